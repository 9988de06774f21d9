"""CUDA grouped GEMMs vs the oracle (fp64 ground truth on dequantised
operands).  Tolerance: relative Frobenius error <= 1e-3 for fp32 output, and
for bf16 output against the oracle rounded to bf16 (bf16 rounding alone is
about 1.7e-3 relative)."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

TOL = 1e-3


def u8(t):
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


def dev_u8(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def as_fp8(a, dev):
    return dev_u8(a, dev).view(torch.float8_e4m3fn)


def rand_codes(shape, gen, dev, lo=-6.0, hi=6.0):
    """Random finite e4m3 operands (quantised N(0,1) values)."""
    x = torch.randn(*shape, generator=gen, device=dev).clamp_(lo, hi)
    return x.to(torch.float8_e4m3fn)


def rand_scales(shape, gen, dev, lo=120, hi=134):
    return torch.randint(lo, hi, shape, generator=gen, device=dev, dtype=torch.int32).to(torch.uint8)


def check_fwd(mxg, orc, a, w, offs, a_s, w_s, kind=3, out_dtype=torch.float32, M=None):
    E = w.shape[0]
    M = a.shape[0]
    y = mxg.ops.grouped_fwd(a, w, offs, a_s, w_s, out_dtype=out_dtype, offs_kind=kind)
    assert mxg.device_error() == 0
    st, en = orc.offs_to_bounds(offs.cpu().numpy(), E, M, kind)
    ref = orc.grouped_fwd(u8(a).cpu().numpy(), None if a_s is None else a_s.cpu().numpy(),
                          u8(w).cpu().numpy(), None if w_s is None else w_s.cpu().numpy(), st, en)
    got = y.float().cpu().numpy().astype(np.float64)
    if out_dtype == torch.bfloat16:
        ref = orc.round_to_bf16(ref)
    err = orc.rel_frobenius(got, ref)
    assert err <= TOL, f"rel Frobenius error {err:.3e}"
    return got, ref


def test_cfg0_fwd_fixture(mxg, orc, cuda_dev):
    g = golden("cfg0_small.npz")
    a, w = as_fp8(g["xq"], cuda_dev), as_fp8(g["wq"], cuda_dev)
    a_s, w_s = dev_u8(g["xs"], cuda_dev), dev_u8(g["ws"], cuda_dev)
    offs = dev_u8(g["offs"], cuda_dev)
    for dt in (torch.float32, torch.bfloat16):
        y = mxg.fused_grouped_fwd(a, w, offs, a_s, w_s, out_dtype=dt)
        ref = g["y"] if dt == torch.float32 else orc.round_to_bf16(g["y"])
        err = orc.rel_frobenius(y.float().cpu().numpy(), ref)
        assert err <= TOL, (dt, err)
    assert mxg.device_error() == 0


def test_reference_sanity_fixture_unscaled(mxg, orc, cuda_dev):
    """fused_fwd.py:271-288 shape, unscaled, vs reference_grouped_gemm output."""
    g = golden("ref_sanity.npz")
    a, w = as_fp8(g["a"], cuda_dev), as_fp8(g["w"], cuda_dev)
    offs = dev_u8(g["offs"], cuda_dev)
    y = mxg.fused_grouped_fwd(a, w, offs)
    ref = orc.bf16_bits_to_f32(g["ref_bits"]).astype(np.float64)
    got = y.float().cpu().numpy()
    assert orc.rel_frobenius(got, ref) <= TOL
    assert np.abs(got - ref).max() < 0.5  # the reference's own sanity bound


@pytest.mark.parametrize("t", ["t1", "t2", "t3", "t4"])
def test_known_answer_tests(mxg, orc, cuda_dev, t):
    """scale_correctness.py tests 1-4 through the CUDA path."""
    g = golden("kat_scales.npz")
    a, w = as_fp8(g[f"{t}_a"], cuda_dev), as_fp8(g[f"{t}_w"], cuda_dev)
    a_s, w_s = dev_u8(g[f"{t}_a_scales"], cuda_dev), dev_u8(g[f"{t}_w_scales"], cuda_dev)
    offs = dev_u8(g[f"{t}_offs"], cuda_dev)
    y = mxg.fused_grouped_fwd(a, w, offs, a_s, w_s, out_dtype=torch.float32).cpu().numpy()
    if t == "t2":
        assert np.all(y == 96.0)
    elif t == "t3":
        assert np.all(y == 272.0)
    elif t == "t4":
        for m in range(8):
            assert y[m, 0] == 32.0 * 2.0 ** m + 32.0
    else:
        ref = g["t1_ref_deq"]
        assert np.array_equal(np.isnan(y), np.isnan(ref))
        fin = np.isfinite(ref)
        assert (np.abs(y[fin] - ref[fin]) / np.maximum(np.abs(ref[fin]), 1.0)).max() < 2.0 ** -7


def test_offs_conventions_agree(mxg, orc, cuda_dev):
    gen = torch.Generator(device=cuda_dev).manual_seed(1)
    sizes = [96, 0, 288, 32, 200]
    M, N, K, E = sum(sizes), 192, 256, len(sizes)
    a, w = rand_codes((M, K), gen, cuda_dev), rand_codes((E, N, K), gen, cuda_dev)
    a_s, w_s = rand_scales((M, K // 32), gen, cuda_dev), rand_scales((E, N, K // 32), gen, cuda_dev)
    cum = np.cumsum(sizes).astype(np.int32)
    outs = []
    for kind, offs in ((0, np.concatenate([[0], cum])), (1, cum), (2, np.array(sizes, np.int32)),
                       (3, np.concatenate([[0], cum])), (3, cum), (3, np.array(sizes, np.int32))):
        got, _ = check_fwd(mxg, orc, a, w, dev_u8(offs.astype(np.int32), cuda_dev), a_s, w_s, kind)
        outs.append(got)
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


@pytest.mark.parametrize("sizes,N,K", [
    ([128, 64, 0, 192], 256, 512),          # config 0 split
    ([1], 128, 32),                          # single row, single K block
    ([240, 241, 17, 480, 0, 5], 200, 160),   # ragged groups, N and K not multiples of 128
    ([1000], 384, 96),                       # one group, several token tiles, K < 128
    ([0, 0, 700], 128, 1024),                # leading empty groups
    ([33] * 9, 320, 288),                    # many small groups
    ([100, 60], 132, 64),                    # N*2 bytes not a multiple of 16: direct-store epilogue
])
def test_fwd_ragged(mxg, orc, cuda_dev, sizes, N, K):
    gen = torch.Generator(device=cuda_dev).manual_seed(sum(sizes) + N + K)
    M, E = sum(sizes), len(sizes)
    a, w = rand_codes((M, K), gen, cuda_dev), rand_codes((E, N, K), gen, cuda_dev)
    a_s, w_s = rand_scales((M, K // 32), gen, cuda_dev), rand_scales((E, N, K // 32), gen, cuda_dev)
    offs = dev_u8(np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32), cuda_dev)
    check_fwd(mxg, orc, a, w, offs, a_s, w_s, kind=0, out_dtype=torch.float32)
    check_fwd(mxg, orc, a, w, offs, a_s, w_s, kind=0, out_dtype=torch.bfloat16)


@pytest.mark.parametrize("sizes,N,K", [([300, 0, 517, 64, 1200], 384, 1024), ([96, 2048, 32], 7168, 2048)])
def test_fwd_scatter_rows_land_like_the_regular_output(mxg, cuda_dev, sizes, N, K):
    """The forward whose epilogue stores each output row into another buffer
    (the expert-parallel return written from the GEMM): three destination
    buffers on this GPU stand in for three ranks; every kept row equals the
    regular forward's row bit for bit, dropped rows (back_rank -1) land
    nowhere, and the untouched destination rows keep their fill."""
    gen = torch.Generator(device=cuda_dev).manual_seed(N + K)
    E, M = len(sizes), sum(sizes)
    a, w = rand_codes((M, K), gen, cuda_dev), rand_codes((E, N, K), gen, cuda_dev)
    a_s, w_s = rand_scales((M, K // 32), gen, cuda_dev), rand_scales((E, N, K // 32), gen, cuda_dev)
    offs = torch.tensor(sizes, dtype=torch.int32, device=cuda_dev)
    y = mxg.ops.grouped_fwd(a, w, offs, a_s, w_s, offs_kind=2)
    rng = np.random.default_rng(7)
    ranks = rng.integers(-1, 3, M).astype(np.int32)
    cap = M + 16
    rows = np.full(M, -1, np.int32)
    for r in range(3):
        idx = np.nonzero(ranks == r)[0]
        rows[idx] = rng.permutation(cap)[:idx.size]
    bufs = [torch.full((cap, N), 7.0, dtype=torch.bfloat16, device=cuda_dev) for _ in range(3)]
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=cuda_dev)
    plan = mxg.ops.GroupedFwdPlan(a_s, w_s, offs, E, M, N, K, cuda_dev, offs_kind=2)
    plan.run_scatter(a, w, ptrs, torch.from_numpy(ranks).to(cuda_dev), torch.from_numpy(rows).to(cuda_dev), cap)
    assert mxg.device_error() == 0
    yh = y.view(torch.int16).cpu().numpy()
    for r in range(3):
        got = bufs[r].view(torch.int16).cpu().numpy()
        idx = np.nonzero(ranks == r)[0]
        assert np.array_equal(got[rows[idx]], yh[idx])
        untouched = np.setdiff1d(np.arange(cap), rows[idx])
        assert np.all(bufs[r].float().cpu().numpy()[untouched] == 7.0)


def test_fwd_scatter_rejects_rows_past_capacity(mxg, cuda_dev):
    """A destination row outside its buffer is skipped and reported."""
    gen = torch.Generator(device=cuda_dev).manual_seed(3)
    E, M, N, K = 2, 64, 256, 256
    a, w = rand_codes((M, K), gen, cuda_dev), rand_codes((E, N, K), gen, cuda_dev)
    offs = torch.tensor([32, 32], dtype=torch.int32, device=cuda_dev)
    buf = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda_dev)
    guard = torch.zeros(64, N, dtype=torch.bfloat16, device=cuda_dev)
    ptrs = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=cuda_dev)
    rows = torch.arange(M, dtype=torch.int32, device=cuda_dev)
    rows[5] = M + 3
    plan = mxg.ops.GroupedFwdPlan(None, None, offs, E, M, N, K, cuda_dev, offs_kind=2)
    plan.run_scatter(a, w, ptrs, torch.zeros(M, dtype=torch.int32, device=cuda_dev), rows, M)
    assert mxg.device_error() == mxg._lib.MXG_ERR_WORKSPACE_TOO_SMALL
    assert torch.all(guard == 0)


def test_fwd_uncovered_rows_are_zero(mxg, orc, cuda_dev):
    gen = torch.Generator(device=cuda_dev).manual_seed(5)
    M, N, K = 300, 128, 64
    a, w = rand_codes((M, K), gen, cuda_dev), rand_codes((2, N, K), gen, cuda_dev)
    offs = dev_u8(np.array([0, 100, 250], np.int32), cuda_dev)
    y = mxg.ops.grouped_fwd(a, w, offs, offs_kind=0, out_dtype=torch.float32)
    assert torch.all(y[250:] == 0)
    check_fwd(mxg, orc, a, w, offs, None, None, kind=0)


def test_fwd_ge_dense(mxg, orc, cuda_dev):
    gen = torch.Generator(device=cuda_dev).manual_seed(9)
    M, N, K = 300, 384, 256
    x = rand_codes((M, K), gen, cuda_dev)
    w_kn = rand_codes((K, N), gen, cuda_dev)
    y = mxg.fwd_ge(x, w_kn)
    ref = orc.grouped_fwd(u8(x).cpu().numpy(), None, u8(w_kn).cpu().numpy().T[None].copy(), None, [0], [M])
    assert orc.rel_frobenius(y.float().cpu().numpy(), orc.round_to_bf16(ref)) <= TOL


def check_wgrad(mxg, orc, go, ia, offs, go_s, ia_s, kind=3, out_dtype=torch.float32):
    N, M = go.shape
    K = ia.shape[0]
    dw = mxg.ops.grouped_wgrad(go, ia, offs, go_s, ia_s, out_dtype=out_dtype, offs_kind=kind)
    assert mxg.device_error() == 0
    E = dw.shape[0]
    st, en = orc.offs_to_bounds(offs.cpu().numpy(), E, M, kind)
    ref = orc.grouped_wgrad(u8(go).cpu().numpy(), None if go_s is None else go_s.cpu().numpy(),
                            u8(ia).cpu().numpy(), None if ia_s is None else ia_s.cpu().numpy(), st, en)
    got = dw.float().cpu().numpy()
    if out_dtype == torch.bfloat16:
        ref = orc.round_to_bf16(ref)
    err = orc.rel_frobenius(got, ref)
    assert err <= TOL, f"rel Frobenius error {err:.3e}"
    for e in range(E):
        if en[e] == st[e]:
            assert np.all(got[e] == 0)
    return got


def test_cfg0_wgrad_fixture(mxg, orc, cuda_dev):
    g = golden("cfg0_small.npz")
    go, ia = as_fp8(g["goq"], cuda_dev), as_fp8(g["iaq"], cuda_dev)
    go_s, ia_s = dev_u8(g["gos"], cuda_dev), dev_u8(g["ias"], cuda_dev)
    sizes = dev_u8(g["sizes"], cuda_dev)
    dw = mxg.wgrad_fused(go, ia, sizes, go_s, ia_s, out_dtype=torch.float32)
    assert orc.rel_frobenius(dw.cpu().numpy(), g["dw"]) <= TOL
    assert torch.all(dw[2] == 0)
    data = mxg.wgrad_prepare(go, ia, sizes, go_s, ia_s)
    dw2 = mxg.wgrad_kernel(data, out_dtype=torch.float32)
    assert torch.equal(dw, dw2)
    assert data["flops"] == 2 * 384 * 256 * 512


@pytest.mark.parametrize("sizes,N,K", [
    ([32, 96, 0, 160, 256], 200, 240),
    ([512], 128, 496),
    ([0, 64], 384, 16),
    ([1024, 32, 32], 256, 2048),
    ([64, 32], 128, 112),        # one column tile ending in a 16-column half chunk
    ([96, 32], 160, 48),
    ([256, 0, 2048], 300, 7168),  # many column tiles, rows past the last 128-row block
])
def test_wgrad_ragged(mxg, orc, cuda_dev, sizes, N, K):
    gen = torch.Generator(device=cuda_dev).manual_seed(sum(sizes) + N + K)
    M = sum(sizes)
    go, ia = rand_codes((N, M), gen, cuda_dev), rand_codes((K, M), gen, cuda_dev)
    go_s, ia_s = rand_scales((N, M // 32), gen, cuda_dev), rand_scales((K, M // 32), gen, cuda_dev)
    offs = dev_u8(np.array(sizes, np.int32), cuda_dev)
    check_wgrad(mxg, orc, go, ia, offs, go_s, ia_s, kind=2)
    check_wgrad(mxg, orc, go, ia, offs, go_s, ia_s, kind=2, out_dtype=torch.bfloat16)


def test_bad_offsets_reported(mxg, cuda_dev):
    gen = torch.Generator(device=cuda_dev).manual_seed(2)
    a, w = rand_codes((64, 64), gen, cuda_dev), rand_codes((2, 64, 64), gen, cuda_dev)
    offs = dev_u8(np.array([0, 50, 40], np.int32), cuda_dev)  # decreasing
    y = mxg.ops.grouped_fwd(a, w, offs, offs_kind=0, out_dtype=torch.float32)
    assert mxg.device_error() == mxg._lib.MXG_ERR_BAD_OFFSETS
    assert torch.all(y == 0)
    go, ia = rand_codes((64, 96), gen, cuda_dev), rand_codes((32, 96), gen, cuda_dev)
    mxg.ops.grouped_wgrad(go, ia, dev_u8(np.array([48, 48], np.int32), cuda_dev), offs_kind=2)
    assert mxg.device_error() == mxg._lib.MXG_ERR_BAD_OFFSETS  # not multiples of 32
    assert mxg.device_error() == 0


def test_bounded_wait_times_out_and_context_survives(mxg, orc, cuda_dev):
    """A wait nothing will satisfy gives up after its limit with an error
    status; the next launch on the same context is correct."""
    gen = torch.Generator(device=cuda_dev).manual_seed(4)
    a, w = rand_codes((256, 128), gen, cuda_dev), rand_codes((1, 128, 128), gen, cuda_dev)
    offs = dev_u8(np.array([0, 256], np.int32), cuda_dev)
    L = mxg._lib.load()
    assert L.mxg_debug_inject_stall(20_000_000) == 0  # 20 ms
    mxg.ops.grouped_fwd(a, w, offs, offs_kind=0)
    assert mxg.device_error() == mxg._lib.MXG_ERR_DEVICE_TIMEOUT
    check_fwd(mxg, orc, a, w, offs, None, None, kind=0)
