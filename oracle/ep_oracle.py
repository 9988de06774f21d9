"""CPU oracle for expert-parallel token dispatch/combine.  TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module; the CUDA library never calls it.

The reference does not implement the dispatch itself: its MXFP8 converter
swaps in torchtitan's MoE token dispatcher with groups padded to 32 rows
(reference ``port_mxfp8.py:74,214-218,240``).  torchtitan is neither vendored
nor installed here (and the reference pins no version), so its published
algorithm is restated in numpy:

* routing slots ``(token t, choice j)`` are ordered by global expert id,
  stable in ``t * k + j`` (``argsort(kind="stable")`` of the flattened ids);
* experts are sharded evenly, expert ``e`` on rank ``e // E_local``, so the
  expert-sorted send buffer is already grouped by destination rank;
* the per-(rank, local expert) counts are exchanged first, then the rows;
* the receiver lays rows out expert-major (source rank order inside an
  expert), each expert's group padded with zero rows to a multiple of 32;
* the combine sends results back along the inverse path and sums each
  token's k choices, weighted by the router probabilities.

The functions below are the single-rank pieces plus ``simulate`` which runs
the whole exchange for ``world`` ranks in one process.
"""
from __future__ import annotations

import numpy as np


def route(expert_ids: np.ndarray, num_experts: int, slot_of_expert=None):
    """expert_ids [n, k] -> (counts [E] per expert slot, send_rows [n*k] token
    of each send position, slot_pos [n*k] send position of each slot).  The
    slot of expert e is slot_of_expert[e] (identity when None); slot s lives
    on rank s // E_local."""
    flat = np.asarray(expert_ids, dtype=np.int64).reshape(-1)
    if slot_of_expert is not None:
        flat = np.asarray(slot_of_expert, dtype=np.int64)[flat]
    k = expert_ids.shape[1] if expert_ids.ndim == 2 else 1
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=num_experts).astype(np.int32)
    send_rows = (order // k).astype(np.int32)
    slot_pos = np.empty_like(order)
    slot_pos[order] = np.arange(order.size)
    return counts, send_rows, slot_pos.astype(np.int32)


def gather(src: np.ndarray, idx: np.ndarray, n: int) -> np.ndarray:
    """dst[i] = src[idx[i]]; idx < 0 gives a zero row."""
    out = np.zeros((n,) + src.shape[1:], dtype=src.dtype)
    idx = np.asarray(idx[:n], dtype=np.int64)
    ok = (idx >= 0) & (idx < src.shape[0])
    out[ok] = src[idx[ok]]
    return out


def regroup(recv_counts: np.ndarray, pad: int):
    """recv_counts [world, E_local] rows received from each rank per local
    expert (rows arrive rank-major, expert-minor) -> (idx [M_pad] received row
    feeding each padded row or -1, back [n_recv] padded row of each received
    row, group_rows [E_local] padded group sizes)."""
    world, e_local = recv_counts.shape
    per_expert = recv_counts.sum(0)
    group_rows = ((per_expert + pad - 1) // pad * pad).astype(np.int32)
    starts = np.concatenate([[0], np.cumsum(group_rows)[:-1]]).astype(np.int64)
    m_pad = int(group_rows.sum())
    n_recv = int(recv_counts.sum())
    idx = np.full(m_pad, -1, dtype=np.int32)
    back = np.empty(n_recv, dtype=np.int32)
    src = 0
    fill = np.zeros(e_local, dtype=np.int64)
    for r in range(world):
        for e in range(e_local):
            c = int(recv_counts[r, e])
            dst = starts[e] + fill[e]
            idx[dst:dst + c] = np.arange(src, src + c)
            back[src:src + c] = np.arange(dst, dst + c)
            fill[e] += c
            src += c
    return idx, back, group_rows


def combine(rows: np.ndarray, slot_pos: np.ndarray, weights, n: int, k: int) -> np.ndarray:
    """out[t] = sum_j w[t, j] * rows[slot_pos[t*k + j]] in fp32."""
    r = rows.astype(np.float32)[np.asarray(slot_pos, dtype=np.int64)].reshape(n, k, rows.shape[1])
    w = np.ones((n, k), np.float32) if weights is None else np.asarray(weights, np.float32)
    out = np.zeros((n, r.shape[2]), np.float32)
    for j in range(k):  # same summation order as a per-token loop over choices
        out += w[:, j:j + 1] * r[:, j]
    return out


def simulate(xs, ids, num_experts: int, pad: int = 32, slot_of_expert=None):
    """Run dispatch on ``world = len(xs)`` ranks: xs[r] [n_r, H], ids[r]
    [n_r, k].  Returns per rank (x_local [M_pad, H], recv_counts [world,
    E_local], plan) where plan carries what combine needs."""
    world = len(xs)
    e_local = num_experts // world
    routed = [route(i, num_experts, slot_of_expert) for i in ids]
    send_counts = [c.reshape(world, e_local) for c, _, _ in routed]
    send_bufs = [xs[r][routed[r][1]] for r in range(world)]
    send_off = [np.concatenate([[0], np.cumsum(sc.sum(1))]) for sc in send_counts]
    out = []
    for d in range(world):
        recv_counts = np.stack([send_counts[s][d] for s in range(world)])
        recv = np.concatenate([send_bufs[s][send_off[s][d]:send_off[s][d + 1]] for s in range(world)])
        idx, back, group_rows = regroup(recv_counts, pad)
        out.append((gather(recv, idx, idx.size), recv_counts, dict(back=back, group_rows=group_rows)))
    return out, routed, send_counts


def simulate_combine(ys, routed, send_counts, plans, weights, ns, k):
    """Inverse of ``simulate``: ys[d] [M_pad_d, H'] per expert rank -> per
    source rank [n_r, H'] fp32 combined rows."""
    world = len(ys)
    back_bufs = [ys[d][plans[d]["back"]] for d in range(world)]
    # rows of back_bufs[d] are ordered by source rank s: sizes send_counts[s][d].sum()
    pieces = [[None] * world for _ in range(world)]
    for d in range(world):
        off = 0
        for s in range(world):
            c = int(send_counts[s][d].sum())
            pieces[s][d] = back_bufs[d][off:off + c]
            off += c
    res = []
    for s in range(world):
        ret = np.concatenate(pieces[s])
        res.append(combine(ret, routed[s][2], weights[s], ns[s], k))
    return res


def p2p_plan(counts_all: np.ndarray, me: int, pad: int = 32):
    """The peer-memory exchange tables of rank ``me`` from the all-gathered
    slot counts C [world, E]: the owners' receive buffers use the regroup
    layout above, so send position p of slot s lands on rank s // E_local at
    row dest_base[s] + p, and padded row q of ``me`` returns to
    (back_rank[q], back_row[q]); ret_order lists the real rows by home rank,
    starting with rank me+1 (so that the ranks send to different peers at the
    same time)."""
    C = np.asarray(counts_all, dtype=np.int64)
    W, E = C.shape
    El = E // W
    tot = C.sum(0)
    padded = (tot + pad - 1) // pad * pad
    gs = np.zeros(E, np.int64)
    for d in range(W):
        gs[d * El:(d + 1) * El] = np.concatenate([[0], np.cumsum(padded[d * El:(d + 1) * El])[:-1]])
    pref = np.concatenate([np.zeros((W, 1), np.int64), np.cumsum(C, axis=1)], axis=1)  # [W, E+1]
    src_off = C[:me].sum(0)
    dest_base = gs + src_off - pref[me, :E]
    mine = slice(me * El, (me + 1) * El)
    group_rows = padded[mine]
    group_start = np.concatenate([gs[mine], [padded[mine].sum()]])
    m_pad = int(padded[mine].sum())
    back_rank = np.full(m_pad, -1, np.int64)
    back_row = np.full(m_pad, -1, np.int64)
    for le in range(El):
        s = me * El + le
        q = gs[s]
        for r in range(W):
            c = C[r, s]
            back_rank[q:q + c] = r
            back_row[q:q + c] = pref[r, s] + np.arange(c)
            q += c
    # real rows grouped by home rank, ranks in the order me+1, me+2, ... (mod W)
    ret_order = [q for kk in range(1, W + 1) for q in range(m_pad) if back_rank[q] == (me + kk) % W]
    i32 = lambda a: np.asarray(a, dtype=np.int32)
    return (i32(pref[me]), i32(dest_base), i32(group_rows), i32(group_start), i32(back_rank),
            i32(back_row), i32(ret_order))
