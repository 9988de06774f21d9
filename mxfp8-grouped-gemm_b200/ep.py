"""Expert parallelism: token dispatch and combine across the ranks of a group.

Experts are sharded evenly: every rank holds ``E_local = E / world`` expert
slots, slot ``s`` on rank ``s // E_local``.  Which expert sits in which slot is
a placement (default: expert ``e`` in slot ``e``, i.e. contiguous blocks of
experts per rank; ``balanced_placement`` evens out the expected rows per rank
from expert popularity while keeping ``E_local`` experts per rank).  The
reference delegates this step to torchtitan's MoE token dispatcher (all-to-all
dispatch and combine, expert groups padded to 32 rows for MXFP8:
``port_mxfp8.py:74,214-218,240``); here it is NCCL ``all_to_all_single`` over
NVLink around four sm_100a kernels:

1. ``route``   stable counting sort of the (token, choice) slots by expert slot,
2. ``gather``  rows into send order, all-to-all to the expert owners,
3. ``regroup`` received rows into expert-major groups padded to 32 rows (the
               layout the grouped GEMMs take),
4. ``combine`` results sent back, weighted sum over each token's choices.

A dispatch needs the per-(rank, slot) counts on the host to size the
all-to-all (one small device-to-host copy); ``dispatch_like`` moves more rows
(e.g. the output gradient) along an existing plan without another one.  The
device work is done by an ``ops`` object; the default is the CUDA library, and
there is no CPU path in the library.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _lib


class CudaEpOps:
    """The routing kernels of libmxg.so on the current CUDA stream."""

    def __init__(self):
        self.L = _lib.load()

    def route(self, expert_ids: torch.Tensor, num_experts: int, slot_of_expert=None):
        ids = expert_ids.to(torch.int32).contiguous()
        n_slots = ids.numel()
        k = ids.shape[1] if ids.dim() == 2 else 1
        dev = ids.device
        counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
        send_rows = torch.empty(n_slots, dtype=torch.int32, device=dev)
        slot_pos = torch.empty(n_slots, dtype=torch.int32, device=dev)
        ws = _lib.workspace(self.L.mxg_ep_route_workspace_size(n_slots, num_experts), dev)
        _lib.check(self.L.mxg_ep_route(ids.data_ptr(), _lib.ptr(slot_of_expert), n_slots, k,
                                       num_experts, counts.data_ptr(), send_rows.data_ptr(),
                                       slot_pos.data_ptr(), ws.data_ptr(), ws.numel(),
                                       _lib.stream_ptr(dev)), "mxg_ep_route")
        return counts, send_rows, slot_pos

    def gather(self, src: torch.Tensor, idx: torch.Tensor, n: int) -> torch.Tensor:
        src = src.contiguous()
        out = torch.empty((n,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
        row_bytes = src.element_size()
        for d in src.shape[1:]:
            row_bytes *= d
        _lib.check(self.L.mxg_gather_rows(src.data_ptr() if src.numel() else None, src.shape[0],
                                          row_bytes, idx.data_ptr(), n, out.data_ptr(),
                                          _lib.stream_ptr(src.device)), "mxg_gather_rows")
        return out

    def regroup(self, recv_counts: torch.Tensor, pad: int, m_pad: int, n_recv: int):
        world, e_local = recv_counts.shape
        dev = recv_counts.device
        idx = torch.empty(max(m_pad, 1), dtype=torch.int32, device=dev)
        back = torch.empty(max(n_recv, 1), dtype=torch.int32, device=dev)
        group_rows = torch.empty(e_local, dtype=torch.int32, device=dev)
        _lib.check(self.L.mxg_ep_regroup(recv_counts.contiguous().data_ptr(), world, e_local, pad,
                                         idx.data_ptr(), back.data_ptr(), group_rows.data_ptr(),
                                         _lib.stream_ptr(dev)), "mxg_ep_regroup")
        return idx[:m_pad], back[:n_recv], group_rows

    def combine(self, rows: torch.Tensor, slot_pos: torch.Tensor, weights, n: int, k: int):
        hidden = rows.shape[1]
        out = torch.empty(n, hidden, dtype=torch.bfloat16, device=rows.device)
        w = None if weights is None else weights.to(torch.float32).contiguous()
        _lib.check(self.L.mxg_ep_combine(rows.contiguous().data_ptr(), slot_pos.data_ptr(),
                                         _lib.ptr(w), n, k, hidden, out.data_ptr(),
                                         _lib.stream_ptr(rows.device)), "mxg_ep_combine")
        return out


def balanced_placement(expert_load, world: int, refine_iters: int = 2000) -> np.ndarray:
    """slot_of_expert [E] with exactly E / world experts per rank and the
    expected rows per rank evened out: experts in decreasing load go to the
    least-loaded rank with a free slot, then the most-loaded rank swaps an
    expert for a lighter one of another rank while that lowers the maximum.
    Deterministic, so every rank computes the same map from the same load."""
    load = np.asarray(expert_load, dtype=np.float64)
    E = load.size
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    e_local = E // world
    owner = np.empty(E, dtype=np.int64)
    rank_load = np.zeros(world)
    filled = np.zeros(world, dtype=np.int64)
    for e in np.argsort(-load, kind="stable"):
        free = np.nonzero(filled < e_local)[0]
        r = int(free[np.argmin(rank_load[free])])
        owner[e] = r
        filled[r] += 1
        rank_load[r] += load[e]
    for _ in range(refine_iters):
        r = int(np.argmax(rank_load))
        mine = np.nonzero(owner == r)[0]
        best = None
        for q in range(world):
            if q == r:
                continue
            theirs = np.nonzero(owner == q)[0]
            d = load[mine][:, None] - load[theirs][None, :]          # load moved r -> q
            new_max = np.maximum(rank_load[r] - d, rank_load[q] + d)
            new_max[d <= 0] = np.inf
            i, j = np.unravel_index(np.argmin(new_max), new_max.shape)
            if new_max[i, j] < rank_load[r] - 1e-9 and (best is None or new_max[i, j] < best[0]):
                best = (new_max[i, j], mine[i], theirs[j], q, d[i, j])
        if best is None:
            break
        _, a, b, q, d = best
        owner[a], owner[b] = q, r
        rank_load[r] -= d
        rank_load[q] += d
    slot = np.empty(E, dtype=np.int32)
    for r in range(world):
        members = np.nonzero(owner == r)[0]      # ascending expert id within a rank
        slot[members] = r * e_local + np.arange(members.size)
    return slot


@dataclass
class DispatchPlan:
    send_rows: torch.Tensor     # [n*k] token row of each send position
    slot_pos: torch.Tensor      # [n*k] send position of each (token, choice)
    send_splits: list           # rows sent to each rank
    recv_splits: list           # rows received from each rank
    idx: torch.Tensor           # [M_pad] received row feeding each padded row (-1 = zero pad)
    back: torch.Tensor          # [n_recv] padded local row of each received row
    group_rows: torch.Tensor    # [E_local] padded rows per local expert slot (device int32)
    group_rows_host: list       # same, on the host
    recv_rows: int              # real (unpadded) rows received
    n_tokens: int
    topk: int


class ExpertParallel:
    """Dispatch/combine of routed token rows over a process group."""

    def __init__(self, num_experts: int, group=None, pad: int = 32, ops=None, placement=None):
        self.group = group
        self.world = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split evenly over {self.world} ranks")
        self.num_experts = num_experts
        self.e_local = num_experts // self.world
        self.pad = pad
        self.ops = ops if ops is not None else CudaEpOps()
        self.slot_of_expert = None
        self.placement = None
        if placement is not None:
            p = np.asarray(placement, dtype=np.int32)
            if p.shape != (num_experts,) or not np.array_equal(np.sort(p), np.arange(num_experts)):
                raise ValueError("placement must be a permutation of the expert ids")
            self.placement = p

    def local_experts(self) -> list:
        """Global expert id held in each local slot of this rank."""
        lo = self.rank * self.e_local
        if self.placement is None:
            return list(range(lo, lo + self.e_local))
        inv = np.argsort(self.placement)
        return [int(e) for e in inv[lo:lo + self.e_local]]

    def _a2a(self, inp, out_rows, out_splits=None, in_splits=None):
        if self.world == 1:
            return inp
        out = torch.empty((out_rows,) + tuple(inp.shape[1:]), dtype=inp.dtype, device=inp.device)
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    def dispatch(self, x: torch.Tensor, expert_ids: torch.Tensor):
        """x [n, H] token rows, expert_ids [n, k] global expert of each choice.
        Returns (x_local [M_pad, H] expert-major 32-padded rows of this rank's
        expert slots, plan)."""
        n, k = expert_ids.shape
        slot_map = None
        if self.placement is not None:
            if self.slot_of_expert is None or self.slot_of_expert.device != expert_ids.device:
                self.slot_of_expert = torch.from_numpy(self.placement).to(expert_ids.device)
            slot_map = self.slot_of_expert
        counts, send_rows, slot_pos = self.ops.route(expert_ids, self.num_experts, slot_map)
        recv_counts = self._a2a(counts, counts.numel()).view(self.world, self.e_local)
        host = torch.cat([counts, recv_counts.reshape(-1)]).cpu().view(2, self.world, self.e_local)
        sc = host[0].sum(1).tolist()
        rc_mat = host[1]
        rc = rc_mat.sum(1).tolist()
        per_expert = rc_mat.sum(0).tolist()
        group_rows_host = [(c + self.pad - 1) // self.pad * self.pad for c in per_expert]
        m_pad = int(sum(group_rows_host))
        n_recv = int(sum(rc))
        idx, back, group_rows = self.ops.regroup(recv_counts, self.pad, m_pad, n_recv)
        plan = DispatchPlan(send_rows, slot_pos, sc, rc, idx, back, group_rows, group_rows_host,
                            n_recv, n, k)
        return self.dispatch_like(x, plan), plan

    def dispatch_like(self, x: torch.Tensor, plan: DispatchPlan) -> torch.Tensor:
        """Rows of x [n, H'] moved along an existing plan (same routing)."""
        send_buf = self.ops.gather(x, plan.send_rows, plan.n_tokens * plan.topk)
        recv_buf = self._a2a(send_buf, plan.recv_rows, plan.recv_splits, plan.send_splits)
        return self.ops.gather(recv_buf, plan.idx, plan.idx.numel())

    def combine(self, y_local: torch.Tensor, plan: DispatchPlan, weights=None) -> torch.Tensor:
        """y_local [M_pad, H'] results in the dispatch layout -> [n, H'] =
        sum over each token's choices (weighted when weights [n, k] given)."""
        back_buf = self.ops.gather(y_local, plan.back, plan.recv_rows)
        ret = self._a2a(back_buf, plan.n_tokens * plan.topk, plan.send_splits, plan.recv_splits)
        return self.ops.combine(ret, plan.slot_pos, weights, plan.n_tokens, plan.topk)
