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

import ctypes
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


class CudaP2POps:
    """The NVLink peer-memory exchange kernels of libmxg.so (current stream)."""

    def __init__(self):
        self.L = _lib.load()

    def plan(self, counts_all: torch.Tensor, me: int, pad: int, m_pad: int, n_recv: int):
        world, E = counts_all.shape
        dev = counts_all.device
        e_local = E // world
        slot_start = torch.empty(E + 1, dtype=torch.int32, device=dev)
        dest_base = torch.empty(E, dtype=torch.int32, device=dev)
        group_rows = torch.empty(e_local, dtype=torch.int32, device=dev)
        group_start = torch.empty(e_local + 1, dtype=torch.int32, device=dev)
        back_rank = torch.empty(max(m_pad, 1), dtype=torch.int32, device=dev)
        back_row = torch.empty(max(m_pad, 1), dtype=torch.int32, device=dev)
        ret_order = torch.empty(max(m_pad, 1), dtype=torch.int32, device=dev)
        ws = _lib.workspace(self.L.mxg_ep_p2p_plan_workspace_size(world, E), dev)
        _lib.check(self.L.mxg_ep_p2p_plan(counts_all.contiguous().data_ptr(), world, E, me, pad, m_pad,
                                          slot_start.data_ptr(), dest_base.data_ptr(),
                                          group_rows.data_ptr(), group_start.data_ptr(),
                                          back_rank.data_ptr(), back_row.data_ptr(),
                                          ret_order.data_ptr(), ws.data_ptr(), ws.numel(),
                                          _lib.stream_ptr(dev)), "mxg_ep_p2p_plan")
        return (slot_start, dest_base, group_rows, group_start, back_rank[:m_pad], back_row[:m_pad],
                ret_order[:n_recv])

    def dispatch(self, src, send_rows, slot_start, dest_base, e_local, me, peer_ptrs, capacity_rows,
                 max_blocks=0):
        src = src.contiguous()
        row_bytes = src.element_size() * (src[0].numel() if src.shape[0] else 0)
        _lib.check(self.L.mxg_ep_dispatch_p2p(src.data_ptr() if src.numel() else None, src.shape[0],
                                              row_bytes, send_rows.data_ptr(), send_rows.numel(),
                                              slot_start.data_ptr(), dest_base.data_ptr(),
                                              dest_base.numel(), e_local, me, peer_ptrs.data_ptr(),
                                              capacity_rows, max_blocks,
                                              _lib.stream_ptr(src.device)), "mxg_ep_dispatch_p2p")

    def dispatch_gather(self, src, send_rows, slot_start, dest_base, e_local, me, peer_ptrs, capacity_rows,
                        src2=None, gather_out=None, split_h=0, src_later=None):
        """dispatch of src, with src2's rows put in send order into gather_out
        in the same pass, and (split_h > 0) the rows of local experts >=
        split_h put in send order into src_later instead of being sent."""
        src = src.contiguous()
        row_bytes = src.element_size() * (src[0].numel() if src.shape[0] else 0)
        if src.numel() == 0:
            return
        ptr = lambda t: None if t is None else t.data_ptr()
        _lib.check(self.L.mxg_ep_dispatch_p2p_gather(
            src.data_ptr(), src.shape[0], row_bytes, send_rows.data_ptr(), send_rows.numel(),
            slot_start.data_ptr(), dest_base.data_ptr(), dest_base.numel(), e_local, me, peer_ptrs.data_ptr(),
            capacity_rows, ptr(None if src2 is None else src2.contiguous()), ptr(gather_out), split_h,
            ptr(src_later), _lib.stream_ptr(src.device)), "mxg_ep_dispatch_p2p_gather")

    def ret(self, src, ret_order, back_rank, back_row, peer_ptrs, capacity_rows, max_blocks=0):
        src = src.contiguous()
        row_bytes = src.element_size() * (src[0].numel() if src.shape[0] else 0)
        _lib.check(self.L.mxg_ep_return_p2p(src.data_ptr() if src.numel() else None, row_bytes,
                                            ret_order.data_ptr(), ret_order.numel(),
                                            back_rank.data_ptr(), back_row.data_ptr(),
                                            peer_ptrs.data_ptr(), peer_ptrs.numel(), capacity_rows,
                                            max_blocks, _lib.stream_ptr(src.device)),
                   "mxg_ep_return_p2p")

    def copy_runs(self, src, runs, peer_host, dst_rows):
        """Contiguous row runs (src_row, dst_row, rows, dst_buf: host int64/int32
        arrays) from src to the buffers at peer_host addresses, on the copy
        engines (current stream)."""
        src = src.contiguous()
        row_bytes = src.element_size() * (src[0].numel() if src.shape[0] else 0)
        s_row, d_row, n_rows, d_buf = runs
        addrs = np.ascontiguousarray(peer_host, dtype=np.uint64)
        _lib.check(self.L.mxg_copy_runs(src.data_ptr() if src.numel() else None, src.shape[0], row_bytes,
                                        s_row.ctypes.data, d_row.ctypes.data, n_rows.ctypes.data,
                                        d_buf.ctypes.data, s_row.size, addrs.ctypes.data, addrs.size,
                                        dst_rows, _lib.stream_ptr(src.device)), "mxg_copy_runs")

    def zero_pad_rows(self, buf, back_rank):
        row_bytes = buf.element_size() * (buf[0].numel() if buf.shape[0] else 0)
        _lib.check(self.L.mxg_ep_zero_pad_rows(buf.data_ptr() if buf.numel() else None, row_bytes,
                                               back_rank.data_ptr(), back_rank.numel(),
                                               _lib.stream_ptr(buf.device)), "mxg_ep_zero_pad_rows")


class _CudaMem:
    """A raw device range exposed through the CUDA array interface (no ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


class PeerBuffer:
    """A device buffer of this rank that every rank of the group can write
    (CUDA IPC).  ``ptrs`` holds every rank's address of its own buffer, as
    seen from this process; ``local`` is this rank's buffer as a uint8 tensor."""

    def __init__(self, nbytes: int, group, world: int, rank: int, device: torch.device):
        self.L = _lib.load()
        self.rank, self.world = rank, world
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _lib.check(self.L.mxg_peer_alloc(nbytes, ctypes.byref(own),
                                         ctypes.cast(handle, ctypes.c_void_p)), "mxg_peer_alloc")
        self.own = own.value
        mine = torch.tensor(list(handle), dtype=torch.uint8, device=device)
        every = torch.empty(world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().view(world, 64)
        self.opened = []
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self.own)
                continue
            h = (ctypes.c_uint8 * 64)(*every[r].tolist())
            p = ctypes.c_void_p()
            _lib.check(self.L.mxg_peer_open(ctypes.cast(h, ctypes.c_void_p), ctypes.byref(p)),
                       "mxg_peer_open")
            ptrs.append(p.value)
            self.opened.append(p.value)
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.ptrs_host = np.array(ptrs, dtype=np.uint64)
        self.nbytes = nbytes
        self.local = torch.as_tensor(_CudaMem(self.own, nbytes), device=device)

    def view(self, rows: int, like: torch.Tensor) -> torch.Tensor:
        """This rank's buffer as [rows, *like.shape[1:]] of like.dtype."""
        shape = (rows,) + tuple(like.shape[1:])
        n = like.element_size()
        for d in shape:
            n *= d
        return self.local[:n].view(like.dtype).view(shape)

    def close_peers(self):
        """Unmap the other ranks' buffers."""
        for p in self.opened:
            self.L.mxg_peer_close(ctypes.c_void_p(p))
        self.opened = []

    def free(self):
        """Free this rank's buffer (after every rank has unmapped it)."""
        if self.own:
            self.local = None
            self.L.mxg_peer_free(ctypes.c_void_p(self.own))
            self.own = None


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


def copy_run_tables(counts_all: np.ndarray, me: int, pad: int, first_slot: int = 0):
    """Copy-engine runs of rank ``me`` from the gathered slot counts C
    [world, E] (the layout of ``mxg_ep_p2p_plan``: slot s of rank s // E_local
    holds the rows of every source rank in rank order, groups padded to
    ``pad``).  Returns (dispatch, return) run tables, each (src_row, dst_row,
    rows, dst_rank) of host arrays with empty runs dropped, ordered by
    destination rank starting with me+1 (the ranks then write to different
    peers at the same time):
      dispatch: send positions [pref[me][s], pref[me][s+1]) of slot s (rows of
                the send-order buffer) -> rows [dest_base[s] + pref[me][s], ..)
                of rank s // E_local (only slots with s % E_local >= first_slot);
      return:   padded rows [gs[s] + sum_{r'<r} C[r'][s], .. + C[r][s]) of local
                slot s -> rows [pref[r][s], ..) of rank r's return buffer."""
    C = np.asarray(counts_all, dtype=np.int64)
    W, E = C.shape
    El = E // W
    pref = np.concatenate([np.zeros((W, 1), np.int64), np.cumsum(C, axis=1)], axis=1)
    padded = ((C.sum(0) + pad - 1) // pad * pad).reshape(W, El)
    gs = (np.cumsum(padded, axis=1) - padded).reshape(E)         # padded start of each slot on its owner
    before = np.cumsum(C, axis=0) - C                             # rows of ranks < r in each slot
    order = (me + 1 + np.arange(W)) % W
    slots = (order[:, None] * El + np.arange(first_slot, El)).reshape(-1)  # owners' slots, owner me+1 first
    c = C[me, slots]
    keep = c > 0
    ds = slots[keep]
    dispatch = (pref[me, ds], gs[ds] + before[me, ds], c[keep], ds // El)
    rr = np.repeat(order, El)                                     # source ranks, me+1 first
    ss = np.tile(me * El + np.arange(El), W)                      # my slots
    c = C[rr, ss]
    keep = c > 0
    rr, ss = rr[keep], ss[keep]
    ret = (gs[ss] + before[rr, ss], pref[rr, ss], c[keep], rr)
    i64 = lambda v: np.ascontiguousarray(v, dtype=np.int64)
    i32 = lambda v: np.ascontiguousarray(v, dtype=np.int32)
    return ((i64(dispatch[0]), i64(dispatch[1]), i64(dispatch[2]), i32(dispatch[3])),
            (i64(ret[0]), i64(ret[1]), i64(ret[2]), i32(ret[3])))


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
    # NVLink peer-memory transport only
    slot_start: torch.Tensor | None = None   # [E+1] send-position prefix over slots
    dest_base: torch.Tensor | None = None    # [E] destination row of position p = dest_base[s] + p
    back_rank: torch.Tensor | None = None    # [M_pad] home rank of each padded row (-1: padding)
    back_row: torch.Tensor | None = None     # [M_pad] send position on that rank
    ret_order: torch.Tensor | None = None    # [n_recv] real rows grouped by home rank, rotated
    # copy-engine runs (host arrays: src_row, dst_row, rows, dst_rank), each
    # list of runs ordered by destination rank starting with rank me+1
    runs_dispatch: tuple | None = None       # send-order rows of each slot -> the owner's buffer
    runs_return: tuple | None = None         # padded rows of each (local expert, source rank) -> home
    pregathered: torch.Tensor | None = None  # [n*k, H'] a second tensor already in send order
    pregathered_src: torch.Tensor | None = None  # ... namely this one
    # split dispatch: local expert slots >= split of every owner still to come
    split: int = 0
    later: torch.Tensor | None = None        # [n*k, H] their rows in send order
    runs_later: tuple | None = None          # their copy-engine runs


class ExpertParallel:
    """Dispatch/combine of routed token rows over a process group."""

    def __init__(self, num_experts: int, group=None, pad: int = 32, ops=None, placement=None,
                 transport: str = "auto", max_tokens: int = 0, p2p_max_blocks: int = 0,
                 ce_streams: int = -1):
        """transport: "p2p" (rows written straight into the owners' buffers
        over NVLink, ranks of one node), "nccl" (all_to_all_single), or "auto"
        (p2p on CUDA with more than one rank).  max_tokens sizes the p2p
        receive buffers for batches up to that many tokens per rank (they
        grow on demand, collectively, when a larger batch arrives).
        ce_streams: copy-engine exchanges issue the runs of each destination
        rank on one of this many streams (-1: one per peer), so several copy
        engines move rows at once; 1: every run on the calling stream."""
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
        if transport not in ("auto", "p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        if transport == "auto":
            transport = "p2p" if (self.world > 1 and torch.cuda.is_available() and ops is None) else "nccl"
        self.transport = transport
        self.p2p = CudaP2POps() if transport == "p2p" else None
        self.max_tokens = max_tokens
        self.p2p_max_blocks = p2p_max_blocks
        self.buffers = {}        # name -> PeerBuffer
        self.capacity = {}       # name -> rows
        self._flag = None
        self.marker = None       # optional callable(name): a timing mark on the current stream
        self.ce_streams = (self.world - 1 if ce_streams < 0 else ce_streams)
        self._ce = []            # the copy-engine streams, created on first use

    def _copy_runs(self, src, runs, peer_host, rows):
        """Copy-engine runs (grouped by destination rank, as copy_run_tables
        orders them): each destination's runs on one of the copy-engine
        streams, which start after the calling stream's preceding work and
        which the calling stream then waits for."""
        k = min(self.ce_streams, self.world)
        dst = runs[3]
        if k <= 1 or dst.size == 0:
            self.p2p.copy_runs(src, runs, peer_host, rows)
            return
        cur = torch.cuda.current_stream(src.device)
        if len(self._ce) < k or self._ce[0].device != src.device:
            self._ce = [torch.cuda.Stream(src.device) for _ in range(k)]
        cuts = np.concatenate([[0], np.flatnonzero(np.diff(dst)) + 1, [dst.size]])
        ready = torch.cuda.Event()
        ready.record(cur)
        used = []
        for i, (lo, hi) in enumerate(zip(cuts[:-1], cuts[1:])):
            st = self._ce[i % k]
            if i < k:
                st.wait_event(ready)
                src.record_stream(st)          # read there: keep the block until those copies ran
                used.append(st)
            with torch.cuda.stream(st):
                self.p2p.copy_runs(src, tuple(a[lo:hi] for a in runs), peer_host, rows)
        for st in used:
            cur.wait_stream(st)

    def _mark(self, name):
        if self.marker is not None:
            self.marker(name)

    def close(self):
        """Release the peer buffers (collective: every rank calls it).  Every
        rank unmaps the others' buffers before any rank frees its own."""
        if self.buffers:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            for b in self.buffers.values():
                b.close_peers()
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            for b in self.buffers.values():
                b.free()
            self.buffers, self.capacity = {}, {}

    def _barrier(self, device):
        """Stream-ordered rendezvous: returns on the device once every rank's
        preceding kernels (and their peer stores) have completed."""
        if self._flag is None or self._flag.device != device:
            self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        dist.all_reduce(self._flag, group=self.group)

    def _ensure_buffer(self, name, rows, row_bytes, device):
        """Collective when it (re)allocates: every rank decides from the same
        all-gathered counts."""
        if self.capacity.get(name, (0, 0))[0] >= rows and self.capacity[name][1] == row_bytes:
            return
        old = self.buffers.pop(name, None)
        if old is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            old.close_peers()
            dist.barrier(group=self.group)
            old.free()
        self.buffers[name] = PeerBuffer(max(rows, 1) * row_bytes, self.group, self.world, self.rank, device)
        self.capacity[name] = (max(rows, 1), row_bytes)

    def _ensure_ret(self, name, device):
        need, alloc, row_bytes = self._ret_need
        rows, rb = self.capacity.get(name, (0, 0))
        if rows < need or rb != row_bytes:
            self._ensure_buffer(name, alloc, row_bytes, device)

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

    def dispatch(self, x: torch.Tensor, expert_ids: torch.Tensor, also_gather: torch.Tensor | None = None,
                 split: int = 0):
        """x [n, H] token rows, expert_ids [n, k] global expert of each choice.
        Returns (x_local [M_pad, H] expert-major 32-padded rows of this rank's
        expert slots, plan).  Peer-memory transport only:
          also_gather ([n, H] like x): put its rows in send order in the same
          pass (``plan.pregathered``), for a later ``dispatch_like(...,
          copy_engines=True)`` of that tensor;
          split in (0, E_local): only the rows of every owner's local slots
          below ``split`` arrive now; the rest wait in send order for
          ``dispatch_rest(plan)`` (copy engines), so the owners can start on
          their first ``split`` experts meanwhile (``plan.split`` says whether
          the split was taken)."""
        n, k = expert_ids.shape
        slot_map = None
        if self.placement is not None:
            if self.slot_of_expert is None or self.slot_of_expert.device != expert_ids.device:
                self.slot_of_expert = torch.from_numpy(self.placement).to(expert_ids.device)
            slot_map = self.slot_of_expert
        counts, send_rows, slot_pos = self.ops.route(expert_ids, self.num_experts, slot_map)
        if self.transport == "p2p":
            return self._dispatch_p2p(x, n, k, counts, send_rows, slot_pos, also_gather, split)
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

    def _dispatch_p2p(self, x, n, k, counts, send_rows, slot_pos, also_gather=None, split=0):
        E, W, El, pad = self.num_experts, self.world, self.e_local, self.pad
        # every rank's slot counts plus its number of routing slots n*k: a
        # routing slot whose expert id is out of range is counted nowhere, and
        # every rank sees that from the same gathered table and raises before
        # any peer store
        mine = torch.cat([counts, torch.full((1,), n * k, dtype=torch.int32, device=x.device)])
        Cx = torch.empty(W * (E + 1), dtype=torch.int32, device=x.device)
        dist.all_gather_into_tensor(Cx, mine, group=self.group)   # also: every receiver is idle
        self._mark("x.counts")
        Cx = Cx.view(W, E + 1)
        Chx = Cx.cpu().numpy().astype(np.int64)
        Ch = Chx[:, :E]
        bad = np.nonzero(Ch.sum(1) != Chx[:, E])[0]
        if bad.size:
            lost = ", ".join(f"rank {r}: {int(Chx[r, E] - Ch[r].sum())}" for r in bad)
            raise ValueError(f"expert ids outside [0, {E}): routing slots counted nowhere ({lost})")
        C = Cx[:, :E].contiguous()
        tot = Ch.sum(0).reshape(W, El)                             # rows per (owner, local slot)
        padded = (tot + pad - 1) // pad * pad
        m_pad_all = padded.sum(1)
        m_pad = int(m_pad_all[self.rank])
        recv_rows = int(tot[self.rank].sum())
        sent = Ch.sum(1)                                           # rows each rank sends
        row_bytes = x.element_size() * (x[0].numel() if x.shape[0] else int(np.prod(x.shape[1:])))
        n_cap = max(int(sent.max()) // max(k, 1), self.max_tokens)
        worst = W * n_cap * min(k, El) + El * (pad - 1)
        need = max(int(m_pad_all.max()), 1)
        for name in ("x", "dy"):
            rows, rb = self.capacity.get(name, (0, 0))
            if rows < need or rb != row_bytes:
                self._ensure_buffer(name, max(worst, need), row_bytes, x.device)
        # return buffers ("ret", and any other combine_send names): every
        # rank's n*k rows in send order; sized like the receive buffers, from
        # the gathered counts, so every rank (re)allocates them together
        self._ret_need = (int(sent.max()), max(n_cap * k, int(sent.max())), row_bytes)
        for name in [b for b in self.capacity if b not in ("x", "dy")] or ["ret"]:
            self._ensure_ret(name, x.device)
        slot_start, dest_base, group_rows, _, back_rank, back_row, ret_order = self.p2p.plan(
            C, self.rank, pad, m_pad, recv_rows)
        plan = DispatchPlan(send_rows, slot_pos, None, None, None, None,
                            group_rows, padded[self.rank].tolist(), recv_rows, n, k,
                            slot_start, dest_base, back_rank, back_row, ret_order)
        split = int(split) if 0 < int(split) < El else 0
        like = also_gather is not None and tuple(also_gather.shape) == tuple(x.shape) \
            and also_gather.dtype == x.dtype
        if like or split:
            buf = self.buffers["x"]
            rows, _ = self.capacity["x"]
            local = buf.view(m_pad, x)
            self.p2p.zero_pad_rows(local, plan.back_rank)
            self._mark("x.plan")
            send = torch.empty((n * k,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device) if like else None
            later = torch.empty((n * k,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device) if split else None
            self.p2p.dispatch_gather(x, send_rows, slot_start, dest_base, El, self.rank, buf.ptrs, rows,
                                     also_gather if like else None, send, split, later)
            self._mark("x.send")
            self._barrier(x.device)
            plan.pregathered, plan.pregathered_src = (send, also_gather) if like else (None, None)
            plan.split, plan.later = split, later
        else:
            local = self.dispatch_like(x, plan, "x")
        # host tables built while the rows move
        plan.send_splits = Ch[self.rank].reshape(W, El).sum(1).tolist()
        plan.recv_splits = Ch[:, self.rank * El:(self.rank + 1) * El].sum(1).tolist()
        plan.runs_dispatch, plan.runs_return = copy_run_tables(Ch, self.rank, pad)
        if split:
            plan.runs_later = copy_run_tables(Ch, self.rank, pad, first_slot=split)[0]
        return local, plan

    def dispatch_rest(self, plan: DispatchPlan) -> None:
        """Second half of a split ``dispatch``: the rows of every owner's local
        slots >= plan.split, from their send-order copy, by copy-engine runs
        into the owners' "x" receive buffers (the tensor ``dispatch``
        returned); returns on the current stream once every rank's rows have
        landed.  Collective: every rank calls it after the same dispatch."""
        if not plan.split or plan.later is None:
            raise ValueError("dispatch_rest follows a dispatch(..., split=h) that took the split")
        send = plan.later
        # allocated on the dispatch's stream; the copies may run on another
        send.record_stream(torch.cuda.current_stream(send.device))
        plan.later = None
        rows, _ = self.capacity["x"]
        self._copy_runs(send, plan.runs_later, self.buffers["x"].ptrs_host, rows)
        self._barrier(send.device)

    def dispatch_like(self, x: torch.Tensor, plan: DispatchPlan, buffer: str = "dy",
                      copy_engines: bool = False) -> torch.Tensor:
        """Rows of x [n, H'] moved along an existing plan (same routing).  With
        the p2p transport the result lives in the named receive buffer ("x" is
        the one ``dispatch`` fills) until the next exchange into it.
        copy_engines: gather the rows into send order here, then move each
        slot's run with the copy engines (no SMs taken from kernels running
        beside the exchange) instead of one SM kernel storing to the peers."""
        if plan.back_rank is not None and copy_engines:
            m_pad = plan.back_rank.numel()
            buf = self.buffers[buffer]
            rows, row_bytes = self.capacity[buffer]
            if x.shape[0] and x.element_size() * x[0].numel() != row_bytes:
                self._barrier(x.device)
                raise ValueError("row size differs from the receive buffer's")
            local = buf.view(m_pad, x)
            self.p2p.zero_pad_rows(local, plan.back_rank)
            send = plan.pregathered if plan.pregathered_src is x else None
            if send is None:
                send = self.ops.gather(x, plan.send_rows, plan.n_tokens * plan.topk)
            else:
                # allocated on the stream of the dispatch; the copies below may
                # run on another one: keep the allocator from handing the block
                # out again before they have read it
                send.record_stream(torch.cuda.current_stream(send.device))
            plan.pregathered = plan.pregathered_src = None
            self._copy_runs(send, plan.runs_dispatch, buf.ptrs_host, rows)
            self._barrier(x.device)
            return local
        if plan.back_rank is not None:
            m_pad = plan.back_rank.numel()
            buf = self.buffers[buffer]
            rows, row_bytes = self.capacity[buffer]
            if x.shape[0] and x.element_size() * x[0].numel() != row_bytes:
                # still take part in the closing rendezvous, so the other
                # ranks are not left waiting in it, then fail
                self._barrier(x.device)
                raise ValueError("row size differs from the receive buffer's")
            local = buf.view(m_pad, x)
            self.p2p.zero_pad_rows(local, plan.back_rank)
            if buffer == "x":
                self._mark("x.plan")
            self.p2p.dispatch(x, plan.send_rows, plan.slot_start, plan.dest_base, self.e_local,
                              self.rank, buf.ptrs, rows, self.p2p_max_blocks)
            if buffer == "x":
                self._mark("x.send")
            self._barrier(x.device)
            return local
        send_buf = self.ops.gather(x, plan.send_rows, plan.n_tokens * plan.topk)
        recv_buf = self._a2a(send_buf, plan.recv_rows, plan.recv_splits, plan.send_splits)
        return self.ops.gather(recv_buf, plan.idx, plan.idx.numel())

    def combine(self, y_local: torch.Tensor, plan: DispatchPlan, weights=None) -> torch.Tensor:
        """y_local [M_pad, H'] results in the dispatch layout -> [n, H'] =
        sum over each token's choices (weighted when weights [n, k] given)."""
        return self.combine_finish(self.combine_send(y_local, plan), plan, weights)

    def combine_send(self, y_local: torch.Tensor, plan: DispatchPlan, buffer: str = "ret",
                     copy_engines: bool = False) -> torch.Tensor:
        """First half of ``combine``: every result row back to its home rank.
        Returns this rank's rows in send order [n*k, H'] (with the p2p
        transport: a view of the named return buffer, valid until the next
        combine into it; every rank must use the same buffer names in the
        same order, since a first use allocates collectively).
        copy_engines: the rows of each (local expert, source rank) pair are
        contiguous on both sides, so each moves as one copy-engine run."""
        if plan.back_rank is not None:
            if buffer not in self.buffers:
                self._ensure_ret(buffer, y_local.device)
            buf = self.buffers[buffer]
            rows, row_bytes = self.capacity[buffer]
            if y_local.shape[0] and y_local.element_size() * y_local[0].numel() != row_bytes:
                self._barrier(y_local.device)   # as in dispatch_like: nobody waits for this rank
                raise ValueError("combine rows must have the dispatched rows' size")
            if copy_engines:
                self._copy_runs(y_local, plan.runs_return, buf.ptrs_host, rows)
            else:
                self.p2p.ret(y_local, plan.ret_order, plan.back_rank, plan.back_row, buf.ptrs, rows,
                             self.p2p_max_blocks)
            self._barrier(y_local.device)
            return buf.view(plan.n_tokens * plan.topk, y_local)
        back_buf = self.ops.gather(y_local, plan.back, plan.recv_rows)
        return self._a2a(back_buf, plan.n_tokens * plan.topk, plan.send_splits, plan.recv_splits)

    def return_target(self, plan: DispatchPlan, like: torch.Tensor, buffer: str = "ret"):
        """Where a kernel that produces this rank's result rows (in the
        dispatch layout) stores them so that they land at home: (device array
        of every rank's address of the named return buffer, back_rank,
        back_row, capacity rows).  Peer-memory transport only.  The producer
        is followed by ``return_done``."""
        if plan.back_rank is None:
            raise ValueError("return_target needs the peer-memory transport")
        if buffer not in self.buffers:
            self._ensure_ret(buffer, like.device)
        rows, row_bytes = self.capacity[buffer]
        if like.element_size() * int(np.prod(like.shape[1:])) != row_bytes:
            raise ValueError("result rows must have the dispatched rows' size")
        return self.buffers[buffer].ptrs, plan.back_rank, plan.back_row, rows

    def return_done(self, plan: DispatchPlan, like: torch.Tensor, buffer: str = "ret") -> torch.Tensor:
        """After the producer of ``return_target``: every rank's rows have
        landed; this rank's rows in send order [n*k, H'] (a view of the return
        buffer, as ``combine_send`` returns)."""
        self._barrier(like.device)
        return self.buffers[buffer].view(plan.n_tokens * plan.topk, like)

    def combine_finish(self, ret: torch.Tensor, plan: DispatchPlan, weights=None) -> torch.Tensor:
        """Second half of ``combine``: the weighted sum over each token's choices."""
        return self.ops.combine(ret, plan.slot_pos, weights, plan.n_tokens, plan.topk)
