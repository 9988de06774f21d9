"""Differentiable MXFP8 grouped matmul for training.

The reference trains with torchao's ``_MXFP8GroupedMM`` autograd function
swapped in by its converter (``port_mxfp8.py:175-194``, kernels patched in
``patch_kernels.py:25-31``): every grouped GEMM of the MoE layer quantises
its operands to MXFP8 (1x32 blocks along the contraction) and runs in FP8
in the forward and in both backward products.  ``grouped_mm`` is that
function on this library's kernels:

    forward  y[rows of g]  = x[rows of g] @ W[g]^T        x 1x32 along K, W 1x32 along K
    dgrad    dx[rows of g] = dy[rows of g] @ W[g]          dy 1x32 along N, W^T 1x32 along N
    wgrad    dW[g]         = dy[rows of g]^T @ x[rows of g] dy, x 32x1 along the tokens

x [M, K] and W [E, N, K] are bf16; offs gives the groups in any of the three
conventions (group boundaries multiples of 32 rows, as the reference pads
them).  The weight gradient is accumulated in fp32 and returned in W's dtype.
"""
from __future__ import annotations

import torch

from . import _lib, ops


class _GroupedMM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, offs, out_dtype):
        if x.dim() != 2 or w.dim() != 3 or x.shape[1] != w.shape[2]:
            raise ValueError("grouped_mm takes x [M, K] and w [E, N, K]")
        E, N, K = w.shape
        xq, xs = ops.quantize_rowwise(x)
        wq, ws = ops.quantize_rowwise(w.reshape(E * N, K))
        offs = offs.to(device=x.device, dtype=torch.int32).contiguous()
        y = ops.grouped_fwd(xq, wq.view(E, N, K), offs, xs, ws.view(E, N, K // 32),
                            out_dtype=out_dtype)
        ctx.save_for_backward(x, w, offs)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, offs = ctx.saved_tensors
        E, N, K = w.shape
        dy = dy.to(torch.bfloat16).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dyq, dys = ops.quantize_rowwise(dy)                          # along N
            wt = w.transpose(1, 2).contiguous()                          # [E, K, N]
            wtq, wts = ops.quantize_rowwise(wt.view(E * K, N))
            dx = ops.grouped_fwd(dyq, wtq.view(E, K, N), offs, dys, wts.view(E, K, N // 32),
                                 out_dtype=x.dtype)
        if ctx.needs_input_grad[1]:
            goq, gos = ops.quantize_colwise(dy)                          # [N, M]
            iaq, ias = ops.quantize_colwise(x)                           # [K, M]
            kind = _lib.OFFS_LEADING_ZERO if offs.numel() == E + 1 else _lib.OFFS_AUTO
            dw = ops.grouped_wgrad(goq, iaq, offs, gos, ias, out_dtype=torch.float32,
                                   offs_kind=kind, num_groups=E).to(w.dtype)
        return dx, dw, None, None


def grouped_mm(x: torch.Tensor, w: torch.Tensor, offs: torch.Tensor,
               out_dtype=torch.bfloat16) -> torch.Tensor:
    """y = x @ W[g]^T over the row groups of x, MXFP8 forward and backward."""
    return _GroupedMM.apply(x, w, offs, out_dtype)
