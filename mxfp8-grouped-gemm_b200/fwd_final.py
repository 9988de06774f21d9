"""Drop-in for the reference's ``fwd_final.py`` dense forward ``fwd_ge``.

Same signature as reference ``fwd_final.py:121-131``: ``x_fp8 [M, K]``,
``w_fp8 [K, N]`` (K x N, N contiguous), unscaled e4m3, bf16 output.  The
Gluon tile keywords are accepted and ignored.  The weight is transposed once
on the device into the K-contiguous layout the tensor cores read.
"""
from __future__ import annotations

import torch

from . import ops


def fwd_ge(x_fp8, w_fp8, BLOCK_M=256, BLOCK_N=256, BLOCK_K=128, NUM_WARPS=4, GROUP_M=4,
           *, out_dtype=torch.bfloat16):
    M, K = x_fp8.shape
    K2, N = w_fp8.shape
    assert K == K2
    return ops.dense_fwd_kn(x_fp8, w_fp8, out_dtype=out_dtype)
