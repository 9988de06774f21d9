"""Expert-parallel routing kernels vs the oracle (bit-exact for the integer
maps and row moves; the weighted combine within one bf16 ulp of the oracle's
fp32 sum; swiglu within 1e-2 relative of a torch fp32 reference), one expert
layer through dispatch -> MXFP8 GEMMs -> combine against fp64, the whole
moe.ExpertFFN step (forward, input gradient and both weight gradients)
against a host restatement, and a world-size-2 NCCL dispatch/combine when
the box has two GPUs."""
import multiprocessing as mp
import os

import numpy as np
import pytest
import torch

from ep_support import free_port, make_rank_inputs
from oracle import ep_oracle
from oracle import mxfp8_oracle as orc_mod

pytestmark = pytest.mark.gpu


def _bf16(x, dev):
    return torch.from_numpy(np.asarray(x, np.float32)).to(torch.bfloat16).to(dev)


def combine_close(got, rows, slot_pos, w, n, k):
    """got within one bf16 ulp of the oracle's fp32 weighted sum, plus the
    fp32 rounding of the k-term sum (FMA vs multiply-then-add) relative to the
    sum of magnitudes, which dominates where the terms cancel."""
    want = ep_oracle.combine(rows, slot_pos, w, n, k)
    mag = ep_oracle.combine(np.abs(rows), slot_pos, None if w is None else np.abs(w), n, k)
    return bool(np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -7 + mag * 2.0 ** -20))


@pytest.mark.parametrize("n,k,E,zipf", [(0, 8, 256, None), (1, 1, 4, None), (1000, 2, 8, 1.2),
                                        (16384, 8, 256, 1.1), (3000, 8, 384, 1.1), (5000, 4, 32, None)])
def test_route_bit_exact(mxg, cuda_dev, n, k, E, zipf):
    ids, _, _ = make_rank_inputs(0, n, k, E, 16, seed=n, zipf=zipf)
    ops = mxg.ep.CudaEpOps()
    c, sr, sp = ops.route(torch.from_numpy(ids).to(cuda_dev), E)
    rc, rsr, rsp = ep_oracle.route(ids, E)
    assert np.array_equal(c.cpu().numpy(), rc)
    assert np.array_equal(sr.cpu().numpy(), rsr)
    assert np.array_equal(sp.cpu().numpy(), rsp)
    assert mxg.device_error() == 0


def test_route_rejects_out_of_range_ids(mxg, cuda_dev):
    ids = torch.tensor([[0, 9]], dtype=torch.int32, device=cuda_dev)
    mxg.ep.CudaEpOps().route(ids, 8)
    with pytest.raises(mxg.MxgError):
        mxg.raise_device_error()


@pytest.mark.parametrize("dtype,width", [(torch.bfloat16, 7168), (torch.uint8, 2048), (torch.bfloat16, 8)])
def test_gather_rows_bit_exact(mxg, cuda_dev, dtype, width):
    g = np.random.default_rng(3)
    src = g.integers(0, 255, size=(300, width * (2 if dtype == torch.bfloat16 else 1)), dtype=np.uint8)
    idx = g.integers(-3, 300, size=517).astype(np.int32)
    s = torch.from_numpy(src).to(cuda_dev).view(dtype)
    out = mxg.ep.CudaEpOps().gather(s, torch.from_numpy(idx).to(cuda_dev), idx.size)
    want = ep_oracle.gather(src, idx, idx.size)
    assert np.array_equal(out.view(torch.uint8).cpu().numpy(), want)


@pytest.mark.parametrize("world,e_local", [(1, 32), (8, 32), (4, 1), (64, 6)])
def test_regroup_bit_exact(mxg, cuda_dev, world, e_local):
    g = np.random.default_rng(world * 100 + e_local)
    rc = g.integers(0, 90, size=(world, e_local)).astype(np.int32)
    rc[0, 0] = 0
    if e_local > 1:
        rc[:, 1] = 0          # an expert nobody routes to
    idx, back, gr = ep_oracle.regroup(rc, 32)
    d_idx, d_back, d_gr = mxg.ep.CudaEpOps().regroup(torch.from_numpy(rc).to(cuda_dev), 32,
                                                     idx.size, back.size)
    assert np.array_equal(d_idx.cpu().numpy(), idx)
    assert np.array_equal(d_back.cpu().numpy(), back)
    assert np.array_equal(d_gr.cpu().numpy(), gr)


@pytest.mark.parametrize("n,k,H,weighted", [(513, 8, 7168, True), (64, 2, 4096, False), (0, 8, 64, True)])
def test_combine_matches_oracle(mxg, cuda_dev, n, k, H, weighted):
    g = np.random.default_rng(n + k)
    rows = g.standard_normal((n * k, H)).astype(np.float32)
    perm = g.permutation(n * k).astype(np.int32)
    w = g.random((n, k)).astype(np.float32) if weighted else None
    rb = _bf16(rows, cuda_dev)
    out = mxg.ep.CudaEpOps().combine(rb, torch.from_numpy(perm).to(cuda_dev),
                                     None if w is None else torch.from_numpy(w).to(cuda_dev), n, k)
    assert combine_close(out.float().cpu().numpy(), rb.float().cpu().numpy(), perm, w, n, k)


@pytest.mark.parametrize("R,I", [(1, 8), (4096, 2048), (777, 1536)])
def test_swiglu(mxg, cuda_dev, R, I):
    gen = torch.Generator(device=cuda_dev).manual_seed(R)
    gu = (torch.randn(R, 2 * I, generator=gen, device=cuda_dev) * 3).to(torch.bfloat16)
    h = mxg.ops.swiglu(gu)
    g, u = gu.float()[:, :I], gu.float()[:, I:]
    ref = torch.nn.functional.silu(g) * u
    err = ((h.float() - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert err <= 1e-2


def test_expert_parallel_world1_matches_oracle(mxg, cuda_dev):
    E, k, H, n = 16, 4, 512, 700
    ids, x, w = make_rank_inputs(0, n, k, E, H, zipf=1.1)
    par = mxg.ExpertParallel(E)
    xb = _bf16(x, cuda_dev)
    x_local, plan = par.dispatch(xb, torch.from_numpy(ids).to(cuda_dev))
    out, routed, sc = ep_oracle.simulate([xb.float().cpu().numpy()], [ids], E)
    assert np.array_equal(x_local.float().cpu().numpy(), out[0][0])
    assert plan.group_rows_host == out[0][2]["group_rows"].tolist()
    y = par.combine(x_local, plan, torch.from_numpy(w).to(cuda_dev))
    # results return along the inverse path: row p of the send order is x[send_rows[p]]
    rows = xb.float().cpu().numpy()[routed[0][1]]
    assert combine_close(y.float().cpu().numpy(), rows, routed[0][2], w, n, k)


def test_expert_layer_through_dispatch(mxg, orc, cuda_dev):
    """dispatch -> rowwise quantize -> grouped fwd (offs = padded group sizes)
    -> combine equals sum_j w_j * deq(x_t) @ deq(W_e).T, fp64 on the dequantised
    operands, rel Frobenius <= 1e-3 against the oracle rounded as the path rounds."""
    E, k, H, N, n = 8, 2, 256, 128, 300
    ids, x, w = make_rank_inputs(0, n, k, E, H, zipf=1.1)
    par = mxg.ExpertParallel(E)
    xb = _bf16(x, cuda_dev)
    x_local, plan = par.dispatch(xb, torch.from_numpy(ids).to(cuda_dev))
    q, s = mxg.quantize_rowwise(x_local)
    gen = torch.Generator(device=cuda_dev).manual_seed(5)
    wb = (torch.randn(E, N, H, generator=gen, device=cuda_dev) * 0.05).to(torch.bfloat16)
    wq, ws = mxg.quantize_rowwise(wb.view(E * N, H))
    wq, ws = wq.view(E, N, H), ws.view(E, N, H // 32)
    y_local = mxg.ops.grouped_fwd(q, wq, plan.group_rows, s, ws, out_dtype=torch.bfloat16, offs_kind=2)
    out = par.combine(y_local, plan, torch.from_numpy(w).to(cuda_dev))
    # oracle: per padded row fwd, then per-token weighted combine
    qn, sn = q.view(torch.uint8).cpu().numpy(), s.cpu().numpy()
    gr = np.array(plan.group_rows_host)
    st = np.concatenate([[0], np.cumsum(gr)[:-1]])
    ref_local = orc.round_to_bf16(orc.grouped_fwd(qn, sn, wq.view(torch.uint8).cpu().numpy(),
                                                  ws.cpu().numpy(), st, st + gr))
    routed = ep_oracle.route(ids, E)
    back = plan.back.cpu().numpy()
    want = ep_oracle.combine(ref_local[back], routed[2], w, n, k)
    err = orc.rel_frobenius(out.float().cpu().numpy().astype(np.float64), want.astype(np.float64))
    assert err <= 1e-2 and orc.rel_frobenius(y_local.float().cpu().numpy(), ref_local) <= 1e-3


@pytest.mark.parametrize("world,k,H", [(4, 3, 1024), (2, 8, 7168), (1, 2, 256)])
def test_p2p_kernels_emulated_ranks(mxg, cuda_dev, world, k, H):
    """The peer-memory plan, dispatch and return kernels with every rank's
    buffers on one GPU (the kernels only store; nothing waits on a peer):
    received rows equal the regroup layout bit for bit, and returned rows
    combine to the oracle's result."""
    E = 4 * world
    ns = [300, 0, 517, 64][:world]
    ins = [make_rank_inputs(r, ns[r], k, E, H, zipf=1.1) for r in range(world)]
    xs = [_bf16(a[1], cuda_dev) for a in ins]
    ep = mxg.ep.CudaEpOps()
    p2p = mxg.ep.CudaP2POps()
    routed = [ep.route(torch.from_numpy(a[0]).to(cuda_dev), E) for a in ins]
    C = torch.stack([rt[0] for rt in routed])
    out, orouted, osc = ep_oracle.simulate([x.float().cpu().numpy() for x in xs], [a[0] for a in ins], E)
    cap = max(o[0].shape[0] for o in out) + 7
    bufs = [torch.full((cap, H), 7.0, dtype=torch.bfloat16, device=cuda_dev) for _ in range(world)]
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=cuda_dev)
    plans = []
    for r in range(world):
        m_pad = out[r][0].shape[0]
        pl = p2p.plan(C, r, 32, m_pad, int(out[r][1].sum()))
        want = ep_oracle.p2p_plan(C.cpu().numpy(), r)
        for got, w in zip(pl, want):
            assert np.array_equal(got.cpu().numpy(), w)
        plans.append(pl)
        p2p.zero_pad_rows(bufs[r][:m_pad], pl[4])
    for r in range(world):
        p2p.dispatch(xs[r], routed[r][1], plans[r][0], plans[r][1], E // world, r, ptrs, cap)
    for d in range(world):
        m_pad = out[d][0].shape[0]
        assert np.array_equal(bufs[d][:m_pad].float().cpu().numpy(), out[d][0])
    assert mxg.device_error() == 0
    # return: every padded row goes home, then the weighted combine
    ret_rows = max(ns) * k   # every rank's return buffer has the same capacity
    rets = [torch.zeros(ret_rows, H, dtype=torch.bfloat16, device=cuda_dev) for r in range(world)]
    rptrs = torch.tensor([t.data_ptr() for t in rets], dtype=torch.int64, device=cuda_dev)
    for d in range(world):
        m_pad = out[d][0].shape[0]
        p2p.ret(bufs[d][:m_pad], plans[d][6], plans[d][4], plans[d][5], rptrs, ret_rows)
    for r in range(world):
        if ns[r] == 0:
            continue
        w = ins[r][2]
        y = ep.combine(rets[r][:ns[r] * k], routed[r][2], torch.from_numpy(w).to(cuda_dev), ns[r], k)
        rows = xs[r].float().cpu().numpy()[orouted[r][1]]
        assert combine_close(y.float().cpu().numpy(), rows, orouted[r][2], w, ns[r], k)


def test_p2p_dispatch_rejects_rows_past_capacity(mxg, cuda_dev):
    """A destination row outside the buffer is skipped and reported, not written."""
    E, k, H = 4, 2, 64
    ids, x, _ = make_rank_inputs(0, 100, k, E, H)
    ep, p2p = mxg.ep.CudaEpOps(), mxg.ep.CudaP2POps()
    c, sr, sp = ep.route(torch.from_numpy(ids).to(cuda_dev), E)
    C = c.view(1, E)
    pl = p2p.plan(C, 0, 32, int(((c.cpu().numpy() + 31) // 32 * 32).sum()), int(c.sum()))
    small = torch.zeros(8, H, dtype=torch.bfloat16, device=cuda_dev)
    guard = torch.zeros(64, H, dtype=torch.bfloat16, device=cuda_dev)
    ptrs = torch.tensor([small.data_ptr()], dtype=torch.int64, device=cuda_dev)
    p2p.dispatch(_bf16(x, cuda_dev), sr, pl[0], pl[1], E, 0, ptrs, 8)
    assert mxg.device_error() == mxg._lib.MXG_ERR_WORKSPACE_TOO_SMALL
    assert torch.all(guard == 0)


def test_p2p_dispatch_skips_unrouted_positions_and_bad_source_rows(mxg, cuda_dev):
    """Routing slots with expert ids -1 and E are counted nowhere, so their
    send positions (past slot_start[E]) stay unwritten: the dispatch must not
    read them even when they hold garbage, and a source row outside the
    source tensor is skipped and reported.  The other rows land as the oracle
    places them."""
    E, k, H, n = 4, 2, 64, 100
    ids, x, _ = make_rank_inputs(0, n, k, E, H)
    ids[5, 0], ids[17, 1], ids[60, 0] = -1, E, E
    ep, p2p = mxg.ep.CudaEpOps(), mxg.ep.CudaP2POps()
    c, sr, sp = ep.route(torch.from_numpy(ids).to(cuda_dev), E)
    assert mxg.device_error() == mxg._lib.MXG_ERR_INVALID_ARGUMENT   # route reports the ids
    routed = int(c.sum())
    assert routed == n * k - 3
    sr[routed:] = 1 << 30                       # garbage past the routed positions
    ok = (ids >= 0) & (ids < E)
    xb = _bf16(x, cuda_dev)
    want, _, _ = ep_oracle.simulate([xb.float().cpu().numpy()], [np.where(ok, ids, 0)], E)
    C = c.view(1, E)
    m_pad = int(((c.cpu().numpy() + 31) // 32 * 32).sum())
    pl = p2p.plan(C, 0, 32, m_pad, routed)
    buf = torch.zeros(m_pad + 8, H, dtype=torch.bfloat16, device=cuda_dev)
    ptrs = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=cuda_dev)
    p2p.dispatch(xb, sr, pl[0], pl[1], E, 0, ptrs, buf.shape[0])
    assert mxg.device_error() == 0
    # the oracle routed the bad slots to expert 0: compare the other experts' rows
    got = buf[:m_pad].float().cpu().numpy()
    gr = pl[2].cpu().numpy()
    g0 = int(gr[0])
    ref_rows = want[0][0]
    ref_g0 = int(((np.sum(np.where(ok, ids, 0) == 0) + 31) // 32) * 32)
    assert np.array_equal(got[g0:], ref_rows[ref_g0:])
    # a source row index outside x: skipped, reported, nothing else disturbed
    sr2 = sr.clone()
    sr2[0] = n + 3
    buf.zero_()
    p2p.dispatch(xb, sr2, pl[0], pl[1], E, 0, ptrs, buf.shape[0])
    assert mxg.device_error() == mxg._lib.MXG_ERR_INVALID_ARGUMENT
    assert torch.all(buf[m_pad:] == 0)


@pytest.mark.parametrize("split", [0, 2])
def test_p2p_dispatch_gather_moves_rows_and_orders_the_second_tensor(mxg, cuda_dev, split):
    """mxg_ep_dispatch_p2p_gather with four ranks emulated on one GPU: the
    first tensor lands exactly as mxg_ep_dispatch_p2p puts it (the oracle's
    layout), the second comes out in send order (src2[send_rows]).  Split at
    local slot 2: the owners receive only the rows of their slots 0 and 1,
    and the rows of slots 2 and 3 come out in send order in the later
    buffer."""
    world, E, k, H = 4, 16, 3, 64
    El = E // world
    ns = [300, 0, 517, 64]
    ins = [make_rank_inputs(r, ns[r], k, E, H, zipf=1.1) for r in range(world)]
    xs = [_bf16(a[1], cuda_dev) for a in ins]
    ys = [_bf16(a[1] * -3.0 + 1.0, cuda_dev) for a in ins]
    ep, p2p = mxg.ep.CudaEpOps(), mxg.ep.CudaP2POps()
    routed = [ep.route(torch.from_numpy(a[0]).to(cuda_dev), E) for a in ins]
    C = torch.stack([rt[0] for rt in routed])
    out, _, _ = ep_oracle.simulate([x.float().cpu().numpy() for x in xs], [a[0] for a in ins], E)
    cap = max(o[0].shape[0] for o in out) + 7
    bufs = [torch.zeros(cap, H, dtype=torch.bfloat16, device=cuda_dev) for _ in range(world)]
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=cuda_dev)
    Ch = C.cpu().numpy().astype(np.int64)
    for r in range(world):
        m_pad = out[r][0].shape[0]
        pl = p2p.plan(C, r, 32, m_pad, int(out[r][1].sum()))
        send = torch.full((ns[r] * k, H), 5.0, dtype=torch.bfloat16, device=cuda_dev)
        later = torch.full((ns[r] * k, H), 7.0, dtype=torch.bfloat16, device=cuda_dev) if split else None
        p2p.dispatch_gather(xs[r], routed[r][1], pl[0], pl[1], El, r, ptrs, cap, ys[r], send, split, later)
        torch.cuda.synchronize()
        sr = routed[r][1].long()
        assert torch.equal(send, ys[r][sr])
        if split:
            pos_slot = np.repeat(np.arange(E), Ch[r])          # slot of each send position
            late = torch.from_numpy(pos_slot % El >= split).to(cuda_dev)
            assert torch.equal(later[late], xs[r][sr][late])
            assert bool((later[~late] == 7.0).all())
    tot = Ch.sum(0).reshape(world, El)
    padded = (tot + 31) // 32 * 32
    for d in range(world):
        m_pad = out[d][0].shape[0]
        want = out[d][0].copy()
        if split:
            want[padded[d, :split].sum():] = 0                   # slots >= split: not sent yet
        assert np.array_equal(bufs[d][:m_pad].float().cpu().numpy(), want)
    assert mxg.device_error() == 0


def test_copy_runs_move_rows_and_refuse_out_of_bounds_runs(mxg, cuda_dev):
    """mxg_copy_runs (copy-engine row runs) between buffers of this GPU: the
    dispatch run tables of four emulated ranks put every row where the
    oracle's layout has it; a run past a destination's end is refused before
    any copy."""
    world, E, k, H = 4, 16, 3, 64
    ns = [300, 0, 517, 64]
    ins = [make_rank_inputs(r, ns[r], k, E, H, zipf=1.1) for r in range(world)]
    xs = [_bf16(a[1], cuda_dev) for a in ins]
    out, routed, _ = ep_oracle.simulate([x.float().cpu().numpy() for x in xs], [a[0] for a in ins], E)
    C = np.stack([rt[0] for rt in routed])
    cap = max(o[0].shape[0] for o in out) + 5
    bufs = [torch.zeros(cap, H, dtype=torch.bfloat16, device=cuda_dev) for _ in range(world)]
    addrs = np.array([b.data_ptr() for b in bufs], dtype=np.uint64)
    p2p = mxg.ep.CudaP2POps()
    for r in range(world):
        send = xs[r][torch.from_numpy(routed[r][1].astype(np.int64)).to(cuda_dev)]
        runs, _ = mxg.ep.copy_run_tables(C, r, 32)
        p2p.copy_runs(send, runs, addrs, cap)
    torch.cuda.synchronize()
    for d in range(world):
        m_pad = out[d][0].shape[0]
        assert np.array_equal(bufs[d][:m_pad].float().cpu().numpy(), out[d][0])
    src = torch.ones(8, H, dtype=torch.bfloat16, device=cuda_dev)
    bad = (np.array([0], np.int64), np.array([cap - 4], np.int64), np.array([8], np.int64), np.array([0], np.int32))
    before = bufs[0].clone()
    with pytest.raises(mxg._lib.MxgError):
        p2p.copy_runs(src, bad, addrs, cap)
    torch.cuda.synchronize()
    assert torch.equal(bufs[0], before)


def _nccl_worker(rank, world, port, q, transport="nccl"):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from conftest import load_pkg
        mxg = load_pkg()
        dev = torch.device("cuda", rank)
        E, k, H = 16, 8, 1024
        ns = [2048, 512]
        par = mxg.ExpertParallel(E, transport=transport)
        all_in = [make_rank_inputs(r, ns[r], k, E, H, zipf=1.1) for r in range(world)]
        ids, x, w = all_in[rank]
        xb = _bf16(x, dev)
        x_local, plan = par.dispatch(xb, torch.from_numpy(ids).to(dev))
        xs = [torch.from_numpy(a[1]).to(torch.bfloat16).float().numpy() for a in all_in]
        out, routed, sc = ep_oracle.simulate(xs, [a[0] for a in all_in], E)
        ok = np.array_equal(x_local.float().cpu().numpy(), out[rank][0])
        y = par.combine(x_local, plan, torch.from_numpy(w).to(dev))
        rows = xs[rank][routed[rank][1]]
        ok2 = combine_close(y.float().cpu().numpy(), rows, routed[rank][2], w, ns[rank], k)
        # a second step with other tokens reuses the buffers
        x2 = _bf16(x * 3, dev)
        x_local2, plan2 = par.dispatch(x2, torch.from_numpy(ids).to(dev))
        ok3 = np.array_equal(x_local2.float().cpu().numpy(),
                             ep_oracle.simulate([torch.from_numpy(a[1] * 3).to(torch.bfloat16).float().numpy()
                                                 for a in all_in], [a[0] for a in all_in], E)[0][rank][0])
        torch.cuda.synchronize()
        par.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if ok and ok2 and ok3 else f"dispatch {ok} combine {ok2} second {ok3}"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_expert_parallel_world2(transport):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q, transport)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def test_route_with_placement_bit_exact(mxg, cuda_dev):
    W = mxg.workloads
    logp = W.zipf_log_popularity(256, 1.1, seed=0)
    ids = W.zipf_topk_sample(16384, logp, 8, seed=1)
    slot = mxg.ep.balanced_placement(W.expected_expert_load(logp, 8), 8)
    c, sr, sp = mxg.ep.CudaEpOps().route(torch.from_numpy(ids).to(cuda_dev), 256,
                                         torch.from_numpy(slot).to(cuda_dev))
    rc, rsr, rsp = ep_oracle.route(ids, 256, slot)
    assert np.array_equal(c.cpu().numpy(), rc)
    assert np.array_equal(sr.cpu().numpy(), rsr)
    assert np.array_equal(sp.cpu().numpy(), rsp)


@pytest.mark.parametrize("R,I", [(1, 8), (4096, 2048), (333, 1536)])
def test_swiglu_bwd_matches_autograd(mxg, cuda_dev, R, I):
    gen = torch.Generator(device=cuda_dev).manual_seed(R + 1)
    gu = (torch.randn(R, 2 * I, generator=gen, device=cuda_dev) * 3).to(torch.bfloat16)
    dh = torch.randn(R, I, generator=gen, device=cuda_dev).to(torch.bfloat16)
    dgu = mxg.ops.swiglu_bwd(gu, dh)
    ref_in = gu.float().requires_grad_(True)
    out = torch.nn.functional.silu(ref_in[:, :I]) * ref_in[:, I:]
    out.backward(dh.float())
    ref = ref_in.grad
    err = ((dgu.float() - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert err <= 1e-2


def _ffn_emulation(x, dy, wgu, wd, ids, p, E):
    """The layer step of moe.ExpertFFN restated on the host: per expert, MXFP8
    (oracle quantiser) operands, fp64 products, bf16 GEMM outputs, SiLU-gated
    product and its gradient in fp64; also the unquantised fp64 result."""
    n, k = ids.shape
    H, I = x.shape[1], wd.shape[2]
    bf = lambda a: orc_mod.bf16_bits_to_f32(orc_mod.f32_to_bf16_bits(a.astype(np.float32))).astype(np.float64)
    q_row = lambda a: orc_mod.dequantize(*orc_mod.quantize_rowwise(orc_mod.f32_to_bf16_bits(a.astype(np.float32))))
    q_col = lambda a: orc_mod.dequantize(*orc_mod.quantize_colwise(orc_mod.f32_to_bf16_bits(a.astype(np.float32))))
    sig = lambda g: 1.0 / (1.0 + np.exp(-g))
    res = {}
    for quant in (True, False):
        out = np.zeros((n, H))
        dx = np.zeros((n, H))
        dwgu = np.zeros((E, 2 * I, H))
        dwd = np.zeros((E, H, I))
        for e in range(E):
            rows = [(t, j) for t in range(n) for j in range(k) if ids[t, j] == e]
            if not rows:
                continue
            T = np.array([t for t, _ in rows])
            pad = (-len(T)) % 32
            xe = np.concatenate([x[T], np.zeros((pad, H))])
            dye = np.concatenate([dy[T], np.zeros((pad, H))])
            if quant:
                gu = bf(q_row(xe) @ q_row(wgu[e]).T)
            else:
                gu = xe @ wgu[e].T
            g, u = gu[:, :I], gu[:, I:]
            h = g * sig(g) * u
            y = bf(q_row(h) @ q_row(wd[e]).T) if quant else h @ wd[e].T
            dh = bf(q_row(dye) @ q_row(np.ascontiguousarray(wd[e].T)).T) if quant else dye @ wd[e]
            s_ = sig(g)
            dgu = np.concatenate([dh * u * s_ * (1 + g * (1 - s_)), dh * g * s_], 1)
            if quant:
                dwd[e] = q_col(dye) @ q_col(h).T
                dwgu[e] = q_col(dgu) @ q_col(xe).T
                dxe = bf(q_row(dgu) @ q_row(np.ascontiguousarray(wgu[e].T)).T)
            else:
                dwd[e] = dye.T @ h
                dwgu[e] = dgu.T @ xe
                dxe = dgu @ wgu[e]
            for r, (t, j) in enumerate(rows):
                out[t] += p[t, j] * y[r]
                dx[t] += dxe[r]
        res[quant] = (out, dx, dwgu, dwd)
    return res


@pytest.mark.parametrize("wgrad_dtype", [torch.bfloat16, torch.float32])
def test_expert_ffn_world1(mxg, cuda_dev, wgrad_dtype):
    """moe.ExpertFFN on one rank: the combined output, the input gradient and
    both weight gradients against a host restatement of the same MXFP8 layer step
    (relative Frobenius <= 3e-2: the fused SwiGLU quantisers round their fp32
    inputs once, the restatement through bf16) and against the unquantised
    fp64 layer (<= 0.12; MXFP8 alone costs ~0.066 here)."""
    E, H, I, n, k = 8, 256, 128, 300, 2
    rng = np.random.default_rng(3)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)
    x, dy = bf(rng.standard_normal((n, H))), bf(rng.standard_normal((n, H)) * 1e-2)
    wgu, wd = bf(rng.standard_normal((E, 2 * I, H)) * 0.05), bf(rng.standard_normal((E, H, I)) * 0.05)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(n)]).astype(np.int32)
    p = rng.random((n, k)) + 0.1
    p = (p / p.sum(1, keepdims=True)).astype(np.float32)
    layer = mxg.moe.ExpertFFN(mxg.ExpertParallel(E), wgu.to(cuda_dev), wd.to(cuda_dev),
                              wgrad_dtype=wgrad_dtype)
    res = layer.step(x.to(cuda_dev), torch.from_numpy(ids).to(cuda_dev),
                     torch.from_numpy(p).to(cuda_dev), dy.to(cuda_dev))
    assert mxg.device_error() == 0
    assert res.dw_gate_up.dtype == wgrad_dtype and res.dw_down.dtype == wgrad_dtype
    ref = _ffn_emulation(x.float().numpy().astype(np.float64), dy.float().numpy().astype(np.float64),
                         wgu.float().numpy().astype(np.float64), wd.float().numpy().astype(np.float64),
                         ids, p.astype(np.float64), E)
    got = [t.float().cpu().numpy().astype(np.float64) for t in (res.out, res.dx, res.dw_gate_up, res.dw_down)]
    for name, g, rq, rf in zip(("out", "dx", "dw_gate_up", "dw_down"), got, ref[True], ref[False]):
        eq, ef = orc_mod.rel_frobenius(g, rq), orc_mod.rel_frobenius(g, rf)
        assert eq <= 3e-2 and ef <= 0.12, (name, eq, ef)


_LAYER_MODES = {  # name -> (comm stream, copy engines, fused returns, split experts, exchanges after
    #                  encodes, copy-engine streams)
    "seq": (False, False, False, 0, False, -1), "sm": (True, False, False, 0, False, -1),
    "ce": (True, True, False, 0, False, -1), "ce_late": (True, True, False, 0, True, -1),
    "ce_2streams": (True, True, False, 0, False, 2), "ce_split": (True, True, False, 2, False, -1),
    "ce_split_late": (True, True, False, 2, True, -1), "ce_split_2streams": (True, True, False, 2, False, 2),
    "fused": (True, False, True, 0, False, -1)}


def _layer_problem(E, H, I, ns, k):
    rng = np.random.default_rng(11)
    f = lambda a: a.astype(np.float32)
    wgu, wd = f(rng.standard_normal((E, 2 * I, H)) * 0.05), f(rng.standard_normal((E, H, I)) * 0.05)
    toks = []
    for n in ns:
        x, dy = f(rng.standard_normal((n, H))), f(rng.standard_normal((n, H)) * 1e-2)
        ids = np.stack([rng.choice(E, k, replace=False) for _ in range(n)]).astype(np.int32)
        p = rng.random((n, k)) + 0.1
        toks.append((x, dy, ids, f(p / p.sum(1, keepdims=True))))
    return wgu, wd, toks


def _layer_worker(rank, world, port, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from conftest import load_pkg
        mxg = load_pkg()
        dev = torch.device("cuda", rank)
        E, H, I, k = 8, 256, 128, 2
        El = E // world
        wgu, wd, toks = _layer_problem(E, H, I, [300, 217], k)
        x, dy, ids, p = toks[rank]
        bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)
        res = {}
        for name, (side, ce, fused, split, late, streams) in _LAYER_MODES.items():
            par = mxg.ExpertParallel(E, transport="p2p", ce_streams=streams)
            layer = mxg.moe.ExpertFFN(par, bf(wgu[rank * El:(rank + 1) * El]), bf(wd[rank * El:(rank + 1) * El]),
                                      comm_stream=torch.cuda.Stream() if side else None, copy_engines=ce,
                                      fused_return=fused, split_experts=split, exchanges_after_encodes=late)
            for _ in range(2):     # the second step reuses the receive buffers
                r = layer.step(bf(x), torch.from_numpy(ids).to(dev), torch.from_numpy(p).to(dev), bf(dy))
            torch.cuda.synchronize()
            assert mxg.device_error() == 0
            res[name] = tuple(t.float().cpu().numpy() for t in (r.out, r.dx, r.dw_gate_up, r.dw_down))
            par.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


def test_expert_ffn_world2_every_exchange_mode():
    """moe.ExpertFFN over two ranks (NVLink peer memory) in every exchange
    mode (sequential SM copies, SM copies beside the GEMMs, copy engines, copy
    engines with the x dispatch split at local expert 2, each copy-engine
    mode with its exchanges started after the encodes too and with its runs
    spread over two streams, returns from the GEMM epilogues): all give the same bytes (the exchange moves rows and
    changes no arithmetic), and those match the host restatement of the whole
    two-rank layer step within the single-rank test's bound."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_layer_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for pr in procs:
        pr.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], dict), res[r]
        base = res[r]["seq"]
        for name, got in res[r].items():
            for a, b, what in zip(base, got, ("out", "dx", "dw_gate_up", "dw_down")):
                assert np.array_equal(a, b), (r, name, what)
    E, H, I, k = 8, 256, 128, 2
    wgu, wd, toks = _layer_problem(E, H, I, [300, 217], k)
    b64 = lambda a: torch.from_numpy(a).to(torch.bfloat16).float().numpy().astype(np.float64)
    x = np.concatenate([b64(t[0]) for t in toks])
    dy = np.concatenate([b64(t[1]) for t in toks])
    ids = np.concatenate([t[2] for t in toks])
    p = np.concatenate([t[3] for t in toks]).astype(np.float64)
    ref = _ffn_emulation(x, dy, b64(wgu), b64(wd), ids, p, E)
    n0 = toks[0][0].shape[0]
    for r, (lo, hi) in enumerate([(0, n0), (n0, x.shape[0])]):
        out, dx, dwgu, dwd = res[r]["seq"]
        El = E // 2
        pairs = ((out, ref[True][0][lo:hi]), (dx, ref[True][1][lo:hi]),
                 (dwgu, ref[True][2][r * El:(r + 1) * El]), (dwd, ref[True][3][r * El:(r + 1) * El]))
        for (g, want), what in zip(pairs, ("out", "dx", "dw_gate_up", "dw_down")):
            e = orc_mod.rel_frobenius(g.astype(np.float64), want)
            assert e <= 3e-2, (r, what, e)
