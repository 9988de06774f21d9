"""Parity at the BASELINE configurations' full sizes.

The oracle cannot recompute a full DSv3 or Mixtral-shaped grouped GEMM in
seconds, so these tests check a seeded random sample of output entries
against fp64 dot products of the dequantised operands (relative Frobenius
<= 1e-3 over the sample, fp32 outputs), plus exact zeros where the result is
zero by construction (padding rows of the forward)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3
SAMPLES = 2048


def _quant_inputs(mxg, rows, K, std, gen, dev, mask=None):
    x = (torch.randn(rows, K, generator=gen, device=dev) * std)
    if mask is not None:
        x[~mask] = 0
    return x.to(torch.bfloat16)


def _deq_rows(orc, q, s):
    return orc.dequantize(q.view(torch.uint8).cpu().numpy(), s.cpu().numpy()).astype(np.float64)


def check_fwd_sampled(mxg, orc, split, N, K, dev, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    mask = torch.from_numpy(split.row_mask()).to(dev)
    x = _quant_inputs(mxg, split.M, K, 1.0, gen, dev, mask)
    w = (torch.randn(split.E, N, K, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    xq, xs = mxg.quantize_rowwise(x)
    del x
    wq, ws = mxg.quantize_rowwise(w.view(split.E * N, K))
    del w
    offs = torch.from_numpy(split.offs_cumulative()).to(dev)
    y = mxg.ops.grouped_fwd(xq, wq.view(split.E, N, K), offs, xs, ws.view(split.E, N, K // 32),
                            out_dtype=torch.float32, offs_kind=mxg._lib.OFFS_CUMULATIVE)
    assert mxg.device_error() == 0
    rng = np.random.default_rng(seed)
    real = np.flatnonzero(split.row_mask())
    r = rng.choice(real, SAMPLES)
    c = rng.integers(0, N, SAMPLES)
    bounds = np.concatenate([[0], np.cumsum(split.padded)])
    e = np.searchsorted(bounds, r, side="right") - 1
    rt, ct, et = (torch.from_numpy(a).to(dev) for a in (r, c, e))
    a_rows = _deq_rows(orc, xq[rt], xs[rt])
    w_rows = _deq_rows(orc, wq[et * N + ct], ws[et * N + ct])
    ref = (a_rows * w_rows).sum(1)
    got = y[rt, ct].cpu().numpy().astype(np.float64)
    err = orc.rel_frobenius(got, ref)
    assert err <= TOL, f"forward sample rel error {err:.3e}"
    pad = np.flatnonzero(~split.row_mask())
    if pad.size:
        assert torch.all(y[torch.from_numpy(pad[:64]).to(dev)] == 0)


def check_wgrad_sampled(mxg, orc, split, N, K, dev, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    mask = torch.from_numpy(split.row_mask()).to(dev)
    dy = _quant_inputs(mxg, split.M, N, 1e-2, gen, dev, mask)
    go, gos = mxg.quantize_colwise(dy)          # [N, M], [N, M/32]
    del dy
    xa = _quant_inputs(mxg, split.M, K, 1.0, gen, dev, mask)
    ia, ias = mxg.quantize_colwise(xa)          # [K, M], [K, M/32]
    del xa
    sizes = torch.from_numpy(split.padded.astype(np.int32)).to(dev)
    dw = mxg.ops.grouped_wgrad(go, ia, sizes, gos, ias, out_dtype=torch.float32,
                               offs_kind=mxg._lib.OFFS_SIZES)
    assert mxg.device_error() == 0
    rng = np.random.default_rng(seed)
    bounds = np.concatenate([[0], np.cumsum(split.padded)])
    got, ref = [], []
    for _ in range(SAMPLES // 64):              # 64 entries per sampled expert
        ex = int(rng.integers(0, split.E))
        t0, t1 = int(bounds[ex]), int(bounds[ex + 1])
        n = torch.from_numpy(rng.integers(0, N, 64)).to(dev)
        k = torch.from_numpy(rng.integers(0, K, 64)).to(dev)
        if t1 == t0:
            ref.append(np.zeros(64))
        else:
            g_rows = _deq_rows(orc, go[n, t0:t1], gos[n, t0 // 32:t1 // 32])
            i_rows = _deq_rows(orc, ia[k, t0:t1], ias[k, t0 // 32:t1 // 32])
            ref.append((g_rows * i_rows).sum(1))
        got.append(dw[ex, n, k].cpu().numpy().astype(np.float64))
    err = orc.rel_frobenius(np.concatenate(got), np.concatenate(ref))
    assert err <= TOL, f"wgrad sample rel error {err:.3e}"


def test_dsv3_configs_full_size(mxg, orc, cuda_dev):
    """Configs 1-2: 32 experts, 65536 routed rows (Dirichlet(1.0) split):
    gate/up forward (N=4096, K=7168), down and gate/up weight gradients."""
    W = mxg.workloads
    split = W.dirichlet_split(65536, 32, 1.0, seed=0)
    check_fwd_sampled(mxg, orc, split, 4096, 7168, cuda_dev, seed=11)
    check_wgrad_sampled(mxg, orc, split, 7168, 2048, cuda_dev, seed=12)
    check_wgrad_sampled(mxg, orc, split, 4096, 7168, cuda_dev, seed=13)
    torch.cuda.empty_cache()


def test_mixtral_config_full_size(mxg, orc, cuda_dev):
    """Config 3: 8 experts, 32768 tokens top-2 from softmax(N(0,1) logits),
    gate/up (N=28672, K=4096) and down (N=4096, K=14336), forward and weight
    gradients."""
    W = mxg.workloads
    split = W.topk_softmax_split(32768, 8, 2, seed=0)
    check_fwd_sampled(mxg, orc, split, 28672, 4096, cuda_dev, seed=21)
    check_fwd_sampled(mxg, orc, split, 4096, 14336, cuda_dev, seed=22)
    check_wgrad_sampled(mxg, orc, split, 28672, 4096, cuda_dev, seed=23)
    check_wgrad_sampled(mxg, orc, split, 4096, 14336, cuda_dev, seed=24)
    torch.cuda.empty_cache()
