"""Expert-parallel dispatch/combine on CPU: the oracle's routing pieces against
brute force, and ``ExpertParallel``'s orchestration over a world-size-2
``gloo`` process group with the oracle's pieces injected as its ops."""
import multiprocessing as mp
import os

import numpy as np
import pytest
import torch

from ep_support import OracleEpOps, free_port, make_rank_inputs
from oracle import ep_oracle


def test_route_is_stable_counting_sort():
    ids, _, _ = make_rank_inputs(0, 200, 8, 64, 16, zipf=1.1)
    counts, send_rows, slot_pos = ep_oracle.route(ids, 64)
    assert counts.sum() == ids.size
    # brute force: walk experts in order, slots in (t, j) order
    want = [t for e in range(64) for t in range(ids.shape[0]) for j in range(8) if ids[t, j] == e]
    assert send_rows.tolist() == want
    flat = ids.reshape(-1)
    assert np.all(flat[np.argsort(slot_pos)] == np.sort(flat, kind="stable"))
    assert np.all(send_rows[slot_pos] == np.arange(ids.size) // 8)


def test_regroup_pads_expert_major():
    rc = np.array([[3, 0, 33], [1, 0, 0], [0, 0, 31]], dtype=np.int32)  # 3 ranks x 3 experts
    idx, back, gr = ep_oracle.regroup(rc, 32)
    assert gr.tolist() == [32, 0, 64]
    # received order: r0e0(0..2) r0e2(3..35) r1e0(36) r2e2(37..67)
    assert idx[:4].tolist() == [0, 1, 2, 36] and np.all(idx[4:32] == -1)
    assert idx[32:65].tolist() == list(range(3, 36)) and idx[65:96].tolist() == list(range(37, 68))
    assert np.all(idx[back] == np.arange(back.size))


@pytest.mark.parametrize("world", [1, 2, 4])
def test_simulated_dispatch_combine_roundtrip(world):
    E, k, H = 16, 4, 32
    xs, ids, ws, ns = [], [], [], []
    for r in range(world):
        n = [37, 0, 64, 5][r]
        i, x, w = make_rank_inputs(r, n, k, E, H, zipf=1.1)
        xs.append(x), ids.append(i), ws.append(w), ns.append(n)
    out, routed, send_counts = ep_oracle.simulate(xs, ids, E)
    for d, (xl, rc, plan) in enumerate(out):
        assert xl.shape[0] == plan["group_rows"].sum() and xl.shape[0] % 32 == 0
        e_loc = E // world
        # every non-pad row of local expert le comes from a token routed to it
        starts = np.concatenate([[0], np.cumsum(plan["group_rows"])])
        for le in range(e_loc):
            rows = xl[starts[le]:starts[le + 1]]
            real = int(rc[:, le].sum())
            assert np.all(rows[real:] == 0)
            ge = d * e_loc + le
            srcs = np.concatenate([xs[s][np.nonzero((ids[s] == ge).any(1))[0]] for s in range(world)])
            assert np.array_equal(rows[:real], srcs)
    ys = [o[0] * 2.0 for o in out]
    back = ep_oracle.simulate_combine(ys, routed, send_counts, [o[2] for o in out], ws, ns, k)
    for s in range(world):
        np.testing.assert_allclose(back[s], 2.0 * ws[s].sum(1, keepdims=True) * xs[s], rtol=1e-5, atol=1e-5)


def test_balanced_placement_even_and_balanced():
    from conftest import load_pkg
    ep = load_pkg().ep
    W = load_pkg().workloads
    ids = W.zipf_topk_assign(32768, 256, 8, 1.1, seed=0)
    load = np.bincount(ids.reshape(-1), minlength=256)
    for world in (2, 4, 8):
        slot = ep.balanced_placement(load, world)
        assert np.array_equal(np.sort(slot), np.arange(256))
        per_rank = np.zeros(world)
        np.add.at(per_rank, slot // (256 // world), load)
        contiguous = load.reshape(world, -1).sum(1)
        assert per_rank.max() / per_rank.mean() <= 1.03
        assert per_rank.max() <= contiguous.max()


def test_route_with_placement_matches_permuted_ids():
    ids, _, _ = make_rank_inputs(0, 300, 4, 16, 8, zipf=1.1)
    perm = np.random.default_rng(1).permutation(16).astype(np.int32)
    a = ep_oracle.route(ids, 16, perm)
    b = ep_oracle.route(perm[ids], 16)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)


def _gloo_worker(rank, world, port, q, balanced=False):
    try:
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from conftest import load_pkg
        ep = load_pkg().ep
        E, k, H = 8, 2, 64
        ns = [48, 0] if world == 2 else [48]
        slot = ep.balanced_placement(np.arange(E)[::-1] ** 2, world) if balanced else None
        par = ep.ExpertParallel(E, ops=OracleEpOps(), placement=slot)
        ids, x, w = make_rank_inputs(rank, ns[rank], k, E, H, zipf=1.2)
        xb = torch.from_numpy(x).to(torch.bfloat16)
        x_local, plan = par.dispatch(xb, torch.from_numpy(ids))
        # oracle over all ranks' inputs
        all_in = [make_rank_inputs(r, ns[r], k, E, H, zipf=1.2) for r in range(world)]
        xs = [torch.from_numpy(a[1]).to(torch.bfloat16).float().numpy() for a in all_in]
        out, routed, sc = ep_oracle.simulate(xs, [a[0] for a in all_in], E, slot_of_expert=slot)
        assert np.array_equal(x_local.float().numpy(), out[rank][0]), "dispatch rows"
        again = par.dispatch_like(xb * 2, plan)
        assert np.array_equal(again.float().numpy(), 2 * out[rank][0]), "dispatch_like rows"
        assert plan.group_rows_host == out[rank][2]["group_rows"].tolist()
        y = combined = par.combine(x_local, plan, torch.from_numpy(w))
        want = ep_oracle.simulate_combine([o[0] for o in out], routed, sc, [o[2] for o in out],
                                          [a[2] for a in all_in], ns, k)[rank]
        np.testing.assert_allclose(y.float().numpy(), want, rtol=1e-2, atol=1e-2)
        assert combined.shape == (ns[rank], H)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world,balanced", [(1, False), (2, False), (2, True)])
def test_expert_parallel_gloo(world, balanced):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q, balanced)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert res[r] == "ok", res[r]


class _DroppingOps(OracleEpOps):
    """Routes like the CUDA kernel does with an out-of-range expert id: the
    slot is counted nowhere (its send position is never written)."""

    def route(self, expert_ids, num_experts, slot_of_expert=None):
        ids = expert_ids.cpu().numpy()
        ok = (ids >= 0) & (ids < num_experts)
        c, sr, sp = ep_oracle.route(np.where(ok, ids, 0), num_experts)
        c = np.bincount(ids[ok].reshape(-1), minlength=num_experts).astype(np.int32)
        return torch.from_numpy(c), torch.from_numpy(sr), torch.from_numpy(sp)


def _bad_ids_worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from conftest import load_pkg
        ep = load_pkg().ep
        E, k, H = 8, 2, 64
        par = ep.ExpertParallel(E, ops=_DroppingOps(), transport="p2p")
        ids, x, _ = make_rank_inputs(rank, 16, k, E, H)
        if rank == 1:
            ids[3, 0], ids[9, 1] = E, -1          # two routing slots with no expert
        try:
            par.dispatch(torch.from_numpy(x).to(torch.bfloat16), torch.from_numpy(ids))
            msg = "no error"
        except ValueError as e:
            msg = "raised" if "(rank 1: 2)" in str(e) else str(e)
        dist.barrier()                            # both ranks got here: nobody hangs
        dist.destroy_process_group()
        q.put((rank, msg))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


def test_p2p_dispatch_refuses_unrouted_slots_on_every_rank():
    """An expert id outside [0, E) on one rank makes every rank raise from the
    gathered counts, before any peer store (no rank is left waiting)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_bad_ids_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "raised", 1: "raised"}, res


@pytest.mark.parametrize("world", [1, 3, 4])
def test_p2p_plan_places_rows_like_regroup(world):
    """Every send position lands where the regroup layout puts it, and every
    padded row returns to its own send position."""
    E, k, H = 4 * world, 3, 16
    xs, ids = [], []
    for r in range(world):
        i, x, _ = make_rank_inputs(r, [40, 0, 77, 5][r], k, E, H, zipf=1.1)
        xs.append(x), ids.append(i)
    out, routed, send_counts = ep_oracle.simulate(xs, ids, E)
    C = np.stack([rt[0] for rt in routed])
    bufs = [np.zeros_like(o[0]) for o in out]
    for r in range(world):
        slot_start, dest_base, *_ = ep_oracle.p2p_plan(C, r)
        sr = routed[r][1]
        for p in range(sr.size):
            s = int(np.searchsorted(slot_start, p, side="right") - 1)
            bufs[s // (E // world)][dest_base[s] + p] = xs[r][sr[p]]
    for d in range(world):
        assert np.array_equal(bufs[d], out[d][0])
        _, _, gr, gst, brank, brow, order = ep_oracle.p2p_plan(C, d)
        assert sorted(order.tolist()) == [q for q in range(brank.size) if brank[q] >= 0]
        assert np.array_equal(gr, out[d][2]["group_rows"])
        for q in range(brank.size):
            if brank[q] >= 0:
                r, p = brank[q], brow[q]
                assert np.array_equal(xs[r][routed[r][1][p]], out[d][0][q])
            else:
                assert np.all(out[d][0][q] == 0)


@pytest.mark.parametrize("world", [1, 3, 4])
def test_copy_run_tables_place_rows_like_the_oracle(world):
    """The copy-engine runs of every rank, applied on the host, put each
    routed row where the oracle's regroup layout has it, and the return runs
    bring every padded row's result back to its send position."""
    from conftest import load_pkg
    ep = load_pkg().ep
    E, k, H = 4 * world, 3, 8
    xs, ids = [], []
    for r in range(world):
        i, x, _ = make_rank_inputs(r, [40, 0, 77, 5][r], k, E, H, zipf=1.1)
        xs.append(x), ids.append(i)
    out, routed, _ = ep_oracle.simulate(xs, ids, E)
    C = np.stack([rt[0] for rt in routed])
    bufs = [np.zeros_like(o[0]) for o in out]
    for r in range(world):
        send = xs[r][routed[r][1]]
        (src, dst, rows, rank), _ = ep.copy_run_tables(C, r, 32)
        assert rows.min(initial=1) > 0 and rows.sum() == ids[r].size
        for a, b, c, d in zip(src, dst, rows, rank):
            bufs[d][b:b + c] = send[a:a + c]
    for d in range(world):
        assert np.array_equal(bufs[d], out[d][0])
    for r in range(world):
        back = np.full((ids[r].size, H), np.nan)
        for d in range(world):
            _, (src, dst, rows, rank) = ep.copy_run_tables(C, d, 32)
            for a, b, c, q in zip(src, dst, rows, rank):
                if q == r:
                    back[b:b + c] = out[d][0][a:a + c]
        assert np.array_equal(back, xs[r][routed[r][1]])


@pytest.mark.parametrize("world", [2, 4])
def test_split_dispatch_runs_cover_the_later_slots_once(world):
    """A split dispatch: the rows of local slots below h (the SM kernel's
    share) plus the copy-engine runs of ``copy_run_tables(.., first_slot=h)``
    fill every owner's receive layout exactly as one whole dispatch does, and
    no later run writes a row of a slot below h."""
    from conftest import load_pkg
    ep = load_pkg().ep
    E, k, H = 4 * world, 3, 8
    El = E // world
    xs, ids = [], []
    for r in range(world):
        i, x, _ = make_rank_inputs(r, [40, 0, 77, 5][r], k, E, H, zipf=1.1)
        xs.append(x), ids.append(i)
    out, routed, _ = ep_oracle.simulate(xs, ids, E)
    C = np.stack([rt[0] for rt in routed])
    pref = np.concatenate([np.zeros((world, 1), np.int64), np.cumsum(C, axis=1)], axis=1)
    for h in range(1, El):
        bufs = [np.zeros_like(o[0]) for o in out]
        for r in range(world):
            send = xs[r][routed[r][1]]
            for s in range(E):                        # the SM kernel's share: slots below h
                if s % El < h:
                    (src, dst, rows, rank), _ = ep.copy_run_tables(C, r, 32)
                    for a, b, c, d in zip(src, dst, rows, rank):
                        if pref[r, s] <= a < pref[r, s + 1]:
                            bufs[d][b:b + c] = send[a:a + c]
            (src, dst, rows, rank), _ = ep.copy_run_tables(C, r, 32, first_slot=h)
            slot_of_pos = np.searchsorted(pref[r], src, side="right") - 1
            assert np.all(slot_of_pos % El >= h)
            assert rows.sum() == sum(C[r, s] for s in range(E) if s % El >= h)
            for a, b, c, d in zip(src, dst, rows, rank):
                assert not bufs[d][b:b + c].any()     # each row written once
                bufs[d][b:b + c] = send[a:a + c]
        for d in range(world):
            assert np.array_equal(bufs[d], out[d][0])


@pytest.mark.parametrize("world", [2, 3, 8])
def test_copy_run_tables_group_runs_by_destination(world):
    """The copy-engine exchanges put each destination rank's runs on a
    stream of its own by cutting the run tables where the destination
    changes: every destination must form one contiguous block, in the
    rotated order me+1, me+2, ... (dispatch, the split's later runs and the
    return alike)."""
    from conftest import load_pkg
    ep = load_pkg().ep
    rng = np.random.default_rng(world)
    E = 4 * world
    C = rng.integers(0, 40, size=(world, E))
    C[rng.random((world, E)) < 0.4] = 0
    for me in range(world):
        tables = list(ep.copy_run_tables(C, me, 32)) + [ep.copy_run_tables(C, me, 32, first_slot=2)[0]]
        for (_, _, rows, dst) in tables:
            assert rows.min(initial=1) > 0
            blocks = [int(d) for i, d in enumerate(dst) if i == 0 or dst[i - 1] != d]
            assert len(blocks) == len(set(blocks))
            rot = [(d - me - 1) % world for d in blocks]
            assert rot == sorted(rot)
