"""MXFP8 quantisers (sm_100a kernels): bf16 -> e4m3 + E8M0 scales.

Row-wise (1x32 along the last dim) produces the forward operands; column-wise
(32x1 along tokens, transposed output) produces the token-contiguous wgrad
operands ``go (N, M)`` / ``ia (K, M)`` of reference ``wgrad_fused.py:35-39``.
The reference calls torchao's ``triton_to_mxfp8_dim0/dim1`` with the
``mxfp8_rceil`` recipe for this (``port_mxfp8.py:43-49,207-212``); the names
below mirror those.
"""
from __future__ import annotations

from .ops import quantize_colwise, quantize_rowwise


def to_mxfp8_dim0(x, inner_block_size: int = 32):
    """bf16 [R, C] -> (e4m3 [R, C], uint8 E8M0 [R, C/32])."""
    assert inner_block_size == 32, "MXFP8 uses 32-element blocks"
    return quantize_rowwise(x)


def to_mxfp8_dim1(x, inner_block_size: int = 32):
    """bf16 [R, C] -> (e4m3 [C, R], uint8 E8M0 [C, R/32]) (transposed)."""
    assert inner_block_size == 32, "MXFP8 uses 32-element blocks"
    return quantize_colwise(x)


__all__ = ["quantize_rowwise", "quantize_colwise", "to_mxfp8_dim0", "to_mxfp8_dim1"]
