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


@pytest.mark.parametrize("shape", [(32, 2), (96, 1030), (2048, 512), (160, 7168)])
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
