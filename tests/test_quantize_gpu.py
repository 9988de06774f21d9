"""CUDA quantisers vs the oracle: bytes and E8M0 scales bit-exact."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _bf16_from_bits(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_rowwise_fixture_bit_exact(mxg, orc, cuda_dev):
    g = golden("quant_rceil.npz")
    x = _bf16_from_bits(g["x_bits"], cuda_dev)
    q, s = mxg.quantize_rowwise(x)
    assert np.array_equal(s.cpu().numpy(), g["s"])
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g["q"])


def test_colwise_fixture_bit_exact(mxg, orc, cuda_dev):
    g = golden("cfg0_small.npz")
    for src, qk, sk in (("dy_bits", "goq", "gos"), ("x_bits", "iaq", "ias")):
        x = _bf16_from_bits(g[src], cuda_dev)
        qt, st = mxg.quantize_colwise(x)
        assert np.array_equal(st.cpu().numpy(), g[sk]), src
        assert np.array_equal(qt.view(torch.uint8).cpu().numpy(), g[qk]), src


@pytest.mark.parametrize("shape,scale", [((96, 160), 1.0), ((257, 4096), 3e-4), ((64, 7168), 5e3),
                                         ((1, 32), 1.0), ((4096, 2048), 1.0)])
def test_rowwise_random_bit_exact(mxg, orc, cuda_dev, shape, scale):
    gen = torch.Generator(device=cuda_dev).manual_seed(7)
    x = (torch.randn(*shape, generator=gen, device=cuda_dev) * scale).to(torch.bfloat16)
    q, s = mxg.quantize_rowwise(x)
    oq, os_ = orc.quantize_rowwise(_bits(x))
    assert np.array_equal(s.cpu().numpy(), os_)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), oq)


@pytest.mark.parametrize("shape", [(32, 2), (96, 1030), (2048, 512), (160, 7168), (1056, 2080)])
def test_colwise_random_bit_exact(mxg, orc, cuda_dev, shape):
    gen = torch.Generator(device=cuda_dev).manual_seed(11)
    x = torch.randn(*shape, generator=gen, device=cuda_dev).to(torch.bfloat16)
    x[3 % shape[0], 1] = float("nan")
    x[5 % shape[0], 0] = float("inf")
    qt, st = mxg.quantize_colwise(x)
    oq, os_ = orc.quantize_colwise(_bits(x))
    assert np.array_equal(st.cpu().numpy(), os_)
    assert np.array_equal(qt.view(torch.uint8).cpu().numpy(), oq)


def test_full_size_rowwise_sampled(mxg, orc, cuda_dev):
    """cfg1 activation size (65536 x 7168): sampled rows bit-exact, and the
    dequantised tensor is within half an e4m3 ulp of the input everywhere."""
    gen = torch.Generator(device=cuda_dev).manual_seed(3)
    x = torch.randn(65536, 7168, generator=gen, device=cuda_dev).to(torch.bfloat16)
    q, s = mxg.quantize_rowwise(x)
    rows = torch.randint(0, 65536, (64,), generator=gen, device=cuda_dev).cpu().numpy()
    oq, os_ = orc.quantize_rowwise(_bits(x[torch.from_numpy(rows).to(cuda_dev)]))
    assert np.array_equal(s[rows].cpu().numpy(), os_)
    assert np.array_equal(q.view(torch.uint8)[rows].cpu().numpy(), oq)
    # size-independent property: |deq(q) - x| <= 2^-4 * blockscale-relative
    deq = q.float().view(65536, 224, 32) * torch.exp2(s.float() - 127).unsqueeze(-1)
    err = (deq - x.float().view(65536, 224, 32)).abs()
    bound = torch.exp2(s.float() - 127).unsqueeze(-1) * 16.0  # half ulp at the top binade (448 -> 32/2)
    assert bool((err <= bound).all())


def _special_bf16(shape, gen, dev, scale=1.0):
    x = (torch.randn(*shape, generator=gen, device=dev) * scale).to(torch.bfloat16)
    flat = x.view(-1)
    n = flat.numel()
    idx = torch.randint(0, n, (max(1, n // 500),), generator=gen, device=dev)
    specials = torch.tensor([float("nan"), float("inf"), -float("inf"), 0.0, -0.0, 1e-30, 3e38],
                            device=dev).to(torch.bfloat16)
    flat[idx] = specials[torch.arange(idx.numel(), device=dev) % specials.numel()]
    flat[: 32 * 3] = 0  # an all-zero block in each direction
    return x


@pytest.mark.parametrize("shape,cuts", [((4192, 7168), (0, 1056, 4192)), ((352, 96), (0, 32, 160, 352)),
                                        ((256, 64), (0, 0, 256))])
def test_quantize_dual_rows_in_ranges_match_one_encode(mxg, cuda_dev, shape, cuts):
    """mxg_quantize_dual_rows over consecutive row ranges (cuts at multiples
    of 32 that split the 128-row tiles, an empty range included) writes the
    same bytes as one quantize_dual of the whole tensor; a range outside the
    tensor or off the 32-row grid is refused."""
    gen = torch.Generator(device=cuda_dev).manual_seed(shape[0] * 3 + shape[1])
    x = _special_bf16(shape, gen, cuda_dev)
    q, s, qt, st = mxg.ops.quantize_dual(x)
    out = mxg.ops.dual_outputs(x)
    for t in out:
        t.view(torch.uint8).fill_(0xA5)
    for a, b in zip(cuts, cuts[1:]):
        mxg.ops.quantize_dual_rows(x, a, b, out)
    assert torch.equal(out[0].view(torch.uint8), q.view(torch.uint8)) and torch.equal(out[1], s)
    assert torch.equal(out[2].view(torch.uint8), qt.view(torch.uint8)) and torch.equal(out[3], st)
    for a, b in ((0, shape[0] + 32), (16, 32), (64, 32)):
        with pytest.raises(mxg._lib.MxgError):
            mxg.ops.quantize_dual_rows(x, a, b, out)


@pytest.mark.parametrize("shape", [(32, 32), (64, 96), (4096, 7168), (160, 2048)])
def test_quantize_dual_matches_separate_kernels(mxg, cuda_dev, shape):
    gen = torch.Generator(device=cuda_dev).manual_seed(shape[0] + shape[1])
    x = _special_bf16(shape, gen, cuda_dev)
    q, s, qt, st = mxg.ops.quantize_dual(x)
    q1, s1 = mxg.quantize_rowwise(x)
    qt1, st1 = mxg.quantize_colwise(x)
    assert torch.equal(q.view(torch.uint8), q1.view(torch.uint8)) and torch.equal(s, s1)
    assert torch.equal(qt.view(torch.uint8), qt1.view(torch.uint8)) and torch.equal(st, st1)
    q2, s2, n1, n2 = mxg.ops.quantize_dual(x, colwise=False)
    assert n1 is None and torch.equal(q2.view(torch.uint8), q1.view(torch.uint8))
    _, _, qt3, st3 = mxg.ops.quantize_dual(x, rowwise=False)
    assert torch.equal(qt3.view(torch.uint8), qt1.view(torch.uint8)) and torch.equal(st3, st1)


def test_quantize_dual_bits_match_oracle(mxg, orc, cuda_dev):
    gen = torch.Generator(device=cuda_dev).manual_seed(11)
    x = _special_bf16((96, 160), gen, cuda_dev, scale=50.0)
    q, s, qt, st = mxg.ops.quantize_dual(x)
    bits = _bits(x)
    rq, rs = orc.quantize_rowwise(bits)
    cq, cs = orc.quantize_colwise(bits)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(qt.view(torch.uint8).cpu().numpy(), cq) and np.array_equal(st.cpu().numpy(), cs)


@pytest.mark.parametrize("R,I", [(32, 32), (128, 2048), (96, 1536)])
def test_swiglu_quantize_matches_unfused(mxg, cuda_dev, R, I):
    gen = torch.Generator(device=cuda_dev).manual_seed(R * 7 + I)
    gu = (torch.randn(R, 2 * I, generator=gen, device=cuda_dev) * 4).to(torch.bfloat16)
    fused = mxg.ops.swiglu_quantize(gu)
    ref = mxg.ops.quantize_dual(mxg.ops.swiglu(gu))
    for a, b in zip(fused, ref):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


@pytest.mark.parametrize("R,I", [(32, 32), (128, 2048), (64, 1536)])
def test_swiglu_bwd_quantize_matches_unfused(mxg, cuda_dev, R, I):
    gen = torch.Generator(device=cuda_dev).manual_seed(R * 5 + I)
    gu = (torch.randn(R, 2 * I, generator=gen, device=cuda_dev) * 4).to(torch.bfloat16)
    dh = (torch.randn(R, I, generator=gen, device=cuda_dev) * 1e-2).to(torch.bfloat16)
    fused = mxg.ops.swiglu_bwd_quantize(gu, dh, rowwise=True, colwise=True)
    ref = mxg.ops.quantize_dual(mxg.ops.swiglu_bwd(gu, dh))
    for a, b in zip(fused, ref):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


@pytest.mark.parametrize("shape", [(1056, 2080), (4096, 7168)])
def test_quantize_dual_partial_tiles_bits_match_oracle(mxg, orc, cuda_dev, shape):
    """Both encodings in one pass on shapes with partial 128 x 128 tiles in
    both directions (and whole ones), special values included: bit-exact
    against the oracle."""
    gen = torch.Generator(device=cuda_dev).manual_seed(shape[0] * 3 + shape[1])
    x = _special_bf16(shape, gen, cuda_dev, scale=7.0)
    q, s, qt, st = mxg.ops.quantize_dual(x)
    bits = _bits(x)
    rq, rs = orc.quantize_rowwise(bits)
    cq, cs = orc.quantize_colwise(bits)
    assert np.array_equal(s.cpu().numpy(), rs) and np.array_equal(q.view(torch.uint8).cpu().numpy(), rq)
    assert np.array_equal(st.cpu().numpy(), cs) and np.array_equal(qt.view(torch.uint8).cpu().numpy(), cq)


@pytest.mark.parametrize("R,I", [(128, 2048), (160, 96), (4096, 1536)])
def test_swiglu_bwd_colwise_matches_both_encodings_and_unfused(mxg, cuda_dev, R, I):
    """The column-wise-only SwiGLU-gradient encode (its own TMA-fed kernel)
    equals the column-wise half of the two-direction encode and the
    column-wise encode of the materialised gradient, bit for bit, including
    partial 128 x 64 tiles."""
    gen = torch.Generator(device=cuda_dev).manual_seed(R * 3 + I)
    gu = (torch.randn(R, 2 * I, generator=gen, device=cuda_dev) * 4).to(torch.bfloat16)
    dh = (torch.randn(R, I, generator=gen, device=cuda_dev) * 1e-2).to(torch.bfloat16)
    _, _, qt, st = mxg.ops.swiglu_bwd_quantize(gu, dh)
    _, _, qt2, st2 = mxg.ops.swiglu_bwd_quantize(gu, dh, rowwise=True, colwise=True)
    qt3, st3 = mxg.quantize_colwise(mxg.ops.swiglu_bwd(gu, dh))
    assert torch.equal(qt.view(torch.uint8), qt2.view(torch.uint8)) and torch.equal(st, st2)
    assert torch.equal(qt.view(torch.uint8), qt3.view(torch.uint8)) and torch.equal(st, st3)
