"""grouped_mm (the MXFP8 autograd grouped matmul) against fp64 products of
the oracle's quantisations of the same bf16 tensors: forward, input gradient
and weight gradient within 1e-3 relative Frobenius (bf16 outputs against the
oracle rounded to bf16)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("sizes,N,K", [([64, 0, 96, 160], 256, 512), ([32, 480], 384, 256)])
def test_grouped_mm_forward_and_backward(mxg, orc, cuda_dev, sizes, N, K):
    gen = torch.Generator(device=cuda_dev).manual_seed(sum(sizes) + N)
    E, M = len(sizes), sum(sizes)
    x = torch.randn(M, K, generator=gen, device=cuda_dev).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(E, N, K, generator=gen, device=cuda_dev) * 0.05).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(M, N, generator=gen, device=cuda_dev).to(torch.bfloat16)
    offs = torch.tensor(sizes, dtype=torch.int32, device=cuda_dev)
    y = mxg.grouped_mm(x, w, offs, out_dtype=torch.float32)
    y.backward(dy.float())
    assert mxg.device_error() == 0

    ends = np.cumsum(sizes)
    st, en = ends - np.array(sizes), ends
    xq, xs = orc.quantize_rowwise(_bits(x))
    wq, ws = orc.quantize_rowwise(_bits(w).reshape(E * N, K))
    ref_y = orc.grouped_fwd(xq, xs, wq.reshape(E, N, K), ws.reshape(E, N, K // 32), st, en)
    assert orc.rel_frobenius(y.detach().cpu().numpy(), ref_y) <= TOL

    dyq, dys = orc.quantize_rowwise(_bits(dy))
    wt = np.ascontiguousarray(_bits(w).reshape(E, N, K).transpose(0, 2, 1)).reshape(E * K, N)
    wtq, wts = orc.quantize_rowwise(wt)
    ref_dx = orc.round_to_bf16(orc.grouped_fwd(dyq, dys, wtq.reshape(E, K, N), wts.reshape(E, K, N // 32), st, en))
    assert orc.rel_frobenius(x.grad.float().cpu().numpy(), ref_dx) <= TOL

    goq, gos = orc.quantize_colwise(_bits(dy))
    iaq, ias = orc.quantize_colwise(_bits(x))
    ref_dw = orc.round_to_bf16(orc.grouped_wgrad(goq, gos, iaq, ias, st, en))
    assert orc.rel_frobenius(w.grad.float().cpu().numpy(), ref_dw) <= TOL
    for e in range(E):
        if sizes[e] == 0:
            assert torch.all(w.grad[e] == 0)
