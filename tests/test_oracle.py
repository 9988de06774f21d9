"""The CPU oracle against the golden fixtures generated from the reference's
own code (tests/golden/make_golden.py) and against first principles."""
import math

import numpy as np
import pytest

from conftest import golden


def test_quantizer_matches_rceil_fixture(orc):
    g = golden("quant_rceil.npz")
    q, s = orc.quantize_rowwise(g["x_bits"])
    assert np.array_equal(s, g["s"])
    assert np.array_equal(q, g["q"])


def test_rceil_scale_exhaustive_over_bf16(orc):
    bits = np.arange(0x0001, 0x7F80, dtype=np.uint32)  # every positive finite bf16
    got = orc.rceil_scale_from_amax_bits(bits).astype(np.int64)
    v = orc.bf16_bits_to_f32(bits.astype(np.uint16)).astype(np.float64)
    want = np.clip(np.ceil(np.log2(v / 448.0)), -127, 127).astype(np.int64) + 127
    assert np.array_equal(got, want)
    assert orc.rceil_scale_from_amax_bits(np.array([0, 0x7F80, 0x7FC0]))[...].tolist() == [0, 254, 255]


def test_rceil_scale_pinned_to_third_party_ceil_ue8m0(orc):
    """The RCEIL byte against code this repository did not write: DeepGEMM's
    power-of-two scale rule ``2**ceil(log2(amax / 448))`` as flashinfer ships
    it (``flashinfer.testing.utils._ceil_to_ue8m0``, flashinfer 0.6.11), for
    every positive finite bf16 amax, clamped to the E8M0 range as the
    ``mxfp8_rceil`` recipe does (byte = clamp(exponent, -127, 127) + 127)."""
    fi = pytest.importorskip("flashinfer.testing.utils")
    import torch
    bits = np.arange(0x0001, 0x7F80, dtype=np.uint32)
    got = orc.rceil_scale_from_amax_bits(bits).astype(np.int64)
    amax = torch.from_numpy(bits.astype(np.int32)).to(torch.int16).view(torch.bfloat16)
    sf = fi._ceil_to_ue8m0(amax.float() / 448.0)
    want = torch.log2(sf).round().to(torch.int64).clamp(-127, 127) + 127
    assert np.array_equal(got, want.numpy())


def test_e4m3_elements_pinned_to_torch_cast(orc):
    """Element codes against torch's own float32 -> float8_e4m3fn cast (round
    to nearest even), applied to x * 2**(127 - byte) as the recipe scales
    them, on seeded bf16 blocks spanning many binades (blocks whose scale byte
    is 0 are left to the torchao-restatement fixture: the recipe does not
    scale those)."""
    import torch
    g = np.random.default_rng(7)
    x = g.standard_normal((512, 256)) * np.exp2(g.integers(-60, 60, (512, 1)))
    x[::7, 3] = 0.0
    x[5] = 448.0 * np.exp2(-20)                     # exact powers at the scale boundary
    xb = orc.f32_to_bf16_bits(x.astype(np.float32))
    q, s = orc.quantize_rowwise(xb)
    assert (s > 0).all()
    xf = torch.from_numpy(orc.bf16_bits_to_f32(xb))
    factor = torch.from_numpy(np.exp2(127.0 - s.astype(np.float64)).astype(np.float32))
    scaled = xf.view(512, 8, 32) * factor.view(512, 8, 1)
    want = scaled.to(torch.float8_e4m3fn).view(torch.uint8).reshape(512, 256).numpy()
    assert np.array_equal(q, want)


def test_e4m3_roundtrip_all_codes(orc):
    codes = np.arange(256, dtype=np.uint8)
    vals = orc.E4M3_DECODE[codes]
    finite = ~np.isnan(vals)
    back = orc.e4m3_encode_rne(vals[finite])
    # +0 and -0 both exist; every finite code maps back to itself
    assert np.array_equal(back, codes[finite])
    assert orc.E4M3_DECODE[0x7E] == 448.0 and orc.E4M3_DECODE[0x01] == 2.0 ** -9


def test_e4m3_rne_ties(orc):
    # halfway between 1.0 (code 0x38) and 1.125 (0x39) rounds to even (0x38)
    assert orc.e4m3_encode_rne(np.array([1.0625]))[0] == 0x38
    assert orc.e4m3_encode_rne(np.array([1.1875]))[0] == 0x3A
    assert orc.e4m3_encode_rne(np.array([2.0 ** -10]))[0] == 0x00
    assert orc.e4m3_encode_rne(np.array([-2.0 ** -10 * 3]))[0] == 0x82


def test_oracle_equals_reference_grouped_gemm(orc):
    """reference fused_fwd.py:249-264 (bf16 upcast + per-group matmul) on CPU."""
    g = golden("ref_sanity.npz")
    E, N, K = g["w"].shape
    M = g["a"].shape[0]
    st, en = orc.offs_to_bounds(g["offs"], E, M)
    y = orc.grouped_fwd(g["a"], None, g["w"], None, st, en)
    ref = orc.bf16_bits_to_f32(g["ref_bits"]).astype(np.float64)
    assert np.array_equal(orc.round_to_bf16(y), ref)


def test_oracle_known_answer_tests(orc):
    """scale_correctness.py tests 1-4, inputs as the reference built them."""
    g = golden("kat_scales.npz")
    for t in ("t1", "t2", "t3", "t4"):
        a, w, offs = g[f"{t}_a"], g[f"{t}_w"], g[f"{t}_offs"]
        st, en = orc.offs_to_bounds(offs, w.shape[0], a.shape[0])
        y = orc.grouped_fwd(a, g[f"{t}_a_scales"], w, g[f"{t}_w_scales"], st, en)
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
            rel = np.abs(y[fin] - ref[fin]) / np.maximum(np.abs(ref[fin]), 1.0)
            assert rel.max() < 2.0 ** -7


def test_oracle_cfg0_quantization_and_products(orc):
    g = golden("cfg0_small.npz")
    xq, xs = orc.quantize_rowwise(g["x_bits"])
    assert np.array_equal(xq, g["xq"]) and np.array_equal(xs, g["xs"])
    E, N, K = g["wq"].shape
    wq, ws = orc.quantize_rowwise(g["w_bits"].reshape(E * N, K))
    assert np.array_equal(wq.reshape(E, N, K), g["wq"]) and np.array_equal(ws.reshape(E, N, K // 32), g["ws"])
    goq, gos = orc.quantize_colwise(g["dy_bits"])
    iaq, ias = orc.quantize_colwise(g["x_bits"])
    assert np.array_equal(goq, g["goq"]) and np.array_equal(gos, g["gos"])
    assert np.array_equal(iaq, g["iaq"]) and np.array_equal(ias, g["ias"])
    M = g["xq"].shape[0]
    st, en = orc.offs_to_bounds(g["offs"], E, M)
    y = orc.grouped_fwd(g["xq"], g["xs"], g["wq"], g["ws"], st, en)
    assert orc.rel_frobenius(y, g["y"]) < 1e-12
    dw = orc.grouped_wgrad(g["goq"], g["gos"], g["iaq"], g["ias"], st, en)
    assert orc.rel_frobenius(dw, g["dw"]) < 1e-6
    assert np.all(dw[2] == 0)  # empty group


@pytest.mark.parametrize("kind,offs,want", [
    (0, [0, 128, 192, 192, 384], ([0, 128, 192, 192], [128, 192, 192, 384])),
    (1, [128, 192, 192, 384], ([0, 128, 192, 192], [128, 192, 192, 384])),
    (2, [128, 64, 0, 192], ([0, 128, 192, 192], [128, 192, 192, 384])),
    (3, [0, 128, 192, 192, 384], ([0, 128, 192, 192], [128, 192, 192, 384])),
    (3, [128, 192, 192, 384], ([0, 128, 192, 192], [128, 192, 192, 384])),
    (3, [128, 64, 0, 192], ([0, 128, 192, 192], [128, 192, 192, 384])),
])
def test_offs_conventions(orc, kind, offs, want):
    assert orc.offs_to_bounds(np.array(offs), 4, 384, kind) == tuple(map(list, want))


def test_offs_rejects_inconsistent(orc):
    with pytest.raises(ValueError):
        orc.offs_to_bounds(np.array([1, 128, 192, 192, 384]), 4, 384, 0)
    with pytest.raises(ValueError):
        orc.offs_to_bounds(np.array([128, 64, 0, 100]), 4, 384, 3)
    with pytest.raises(ValueError):
        orc.offs_to_bounds(np.array([0, 300, 200, 384, 384]), 4, 384, 0)


def test_e8m0_helpers_match_reference_semantics(orc):
    # scale_correctness.py:30-45: decode 2^(b-127); encode round(log2(s)) + 127
    assert orc.e8m0_to_float(np.array([127, 128, 126, 129]))[...].tolist() == [1.0, 2.0, 0.5, 4.0]
    assert [orc.e8m0_round_nearest(s) for s in (1.0, 2.0, 0.5, 4.0, 3.0)] == [127, 128, 126, 129, 129]
    assert math.isnan(orc.e8m0_to_float(np.array([255]))[0])
