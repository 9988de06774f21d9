"""Test helpers for expert parallelism: the oracle's dispatch pieces behind the
``ops`` interface ``ExpertParallel`` takes, so its orchestration (count
exchange, split sizes, all-to-alls, combine) can run over ``gloo`` on CPU, and
a spawn-based launcher for world-size-2 process groups."""
import os
import socket
import sys

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

from oracle import ep_oracle  # noqa: E402


class OracleEpOps:
    """CPU stand-in for ``CudaEpOps`` (test only)."""

    def route(self, expert_ids, num_experts, slot_of_expert=None):
        m = None if slot_of_expert is None else slot_of_expert.cpu().numpy()
        c, sr, sp = ep_oracle.route(expert_ids.cpu().numpy(), num_experts, m)
        return torch.from_numpy(c), torch.from_numpy(sr), torch.from_numpy(sp)

    def gather(self, src, idx, n):
        if src.dtype == torch.bfloat16:
            out = ep_oracle.gather(src.view(torch.int16).numpy(), idx.numpy(), n)
            return torch.from_numpy(out).view(torch.bfloat16)
        return torch.from_numpy(ep_oracle.gather(src.numpy(), idx.numpy(), n))

    def regroup(self, recv_counts, pad, m_pad, n_recv):
        idx, back, gr = ep_oracle.regroup(recv_counts.numpy(), pad)
        assert idx.size == m_pad and back.size == n_recv
        return torch.from_numpy(idx), torch.from_numpy(back), torch.from_numpy(gr)

    def combine(self, rows, slot_pos, weights, n, k):
        w = None if weights is None else weights.float().numpy()
        out = ep_oracle.combine(rows.float().numpy(), slot_pos.numpy(), w, n, k)
        return torch.from_numpy(out).to(torch.bfloat16)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_rank_inputs(rank, n, k, num_experts, hidden, seed=0, zipf=None):
    g = np.random.default_rng(seed + 1000 * rank)
    if zipf is None:
        ids = np.stack([g.choice(num_experts, size=k, replace=False) for _ in range(n)]) if n else \
            np.zeros((0, k), np.int64)
    else:
        p = 1.0 / np.arange(1, num_experts + 1) ** zipf
        p /= p.sum()
        perm = g.permutation(num_experts)
        ids = np.stack([perm[g.choice(num_experts, size=k, replace=False, p=p)] for _ in range(n)]) \
            if n else np.zeros((0, k), np.int64)
    x = g.standard_normal((n, hidden)).astype(np.float32)
    w = g.random((n, k)).astype(np.float32)
    return ids.astype(np.int32), x, w
