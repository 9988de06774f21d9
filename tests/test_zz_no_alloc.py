"""The no-allocation grouped forward, ``mxg_grouped_fwd_noalloc``.

It exists for callers that cannot allocate device memory themselves, such as
a plugin running inside a framework that owns the whole device memory pool,
or host code that must not call cudaMalloc because it can synchronise the
device.  Its scratch is a fixed array built into the library instead of a
caller-provided workspace.  These tests call it through the C ABI and compare
it bit for bit with the regular entry point, ``mxg_grouped_fwd``, on two calls
in a row (the second call finds the first call's data still in the shared
array).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(seed, sizes, N, K, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    M, E = sum(sizes), len(sizes)
    a = torch.randn(M, K, generator=g, device=dev).clamp_(-6, 6).to(torch.float8_e4m3fn)
    w = torch.randn(E, N, K, generator=g, device=dev).clamp_(-6, 6).to(torch.float8_e4m3fn)
    a_s = torch.randint(120, 134, (M, K // 32), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    w_s = torch.randint(120, 134, (E, N, K // 32), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    offs = torch.from_numpy(np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)).to(dev)
    return a, w, a_s, w_s, offs


def _noalloc(mxg, a, w, a_s, w_s, offs, out):
    L = mxg._lib.load()
    M, K = a.shape
    E, N, _ = w.shape
    return L.mxg_grouped_fwd_noalloc(a.data_ptr(), a_s.data_ptr(), w.data_ptr(), w_s.data_ptr(),
                                     offs.data_ptr(), offs.numel(), mxg._lib.OFFS_LEADING_ZERO, E, M,
                                     N, K, out.data_ptr(), mxg._lib.DTYPE_F32,
                                     mxg._lib.stream_ptr(a.device))


def test_noalloc_matches_regular_entry_point_twice(mxg, cuda_dev):
    problems = [_problem(1, [300, 0, 517, 64, 1200], 384, 1024, cuda_dev),
                _problem(2, [96, 2048, 33], 256, 2048, cuda_dev)]
    for a, w, a_s, w_s, offs in problems:
        ref = mxg.ops.grouped_fwd(a, w, offs, a_s, w_s, out_dtype=torch.float32,
                                  offs_kind=mxg._lib.OFFS_LEADING_ZERO)
        out = torch.full_like(ref, float("nan"))
        assert _noalloc(mxg, a, w, a_s, w_s, offs, out) == 0
        torch.cuda.synchronize()
        assert mxg.device_error() == 0
        assert torch.isfinite(out).all()
        # the same kernels on the same inputs: bit-identical, so stale scratch
        # contents from the previous call would show
        assert torch.equal(out, ref)


def test_noalloc_rejects_problems_beyond_its_scratch(mxg, cuda_dev):
    L = mxg._lib.load()
    E, M, N, K = 32, 1 << 20, 4096, 7168
    assert L.mxg_grouped_fwd_workspace_size(E, M, N, K) > (64 << 20)
    dummy = torch.empty(16, dtype=torch.uint8, device=cuda_dev)
    p = dummy.data_ptr()
    rc = L.mxg_grouped_fwd_noalloc(p, None, p, None, p, E + 1, mxg._lib.OFFS_LEADING_ZERO, E, M, N,
                                   K, p, mxg._lib.DTYPE_BF16, mxg._lib.stream_ptr(cuda_dev))
    assert rc == 4  # MXG_ERR_WORKSPACE_TOO_SMALL, returned before any launch
