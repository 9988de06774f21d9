"""Drop-in for the reference's ``fused_fwd.py`` grouped forward.

``fused_grouped_fwd`` keeps the signature of reference ``fused_fwd.py:172-230``.
The Triton tile keywords (BLOCK_M/N/K, GROUP_SIZE_M, num_stages, num_warps)
are accepted for call compatibility and ignored: the sm_100a kernel picks its
own tiles.  Unlike the reference kernel (which reads ``M // E`` rows per
group and never ``offs``, ``fused_fwd.py:48``) group sizes come from ``offs``
and may be uneven or empty.
"""
from __future__ import annotations

import torch

from . import ops


def fused_grouped_fwd(a_fp8, w_fp8, offs,
                      a_scales=None, w_scales=None,
                      BLOCK_M=128, BLOCK_N=128, BLOCK_K=128,
                      GROUP_SIZE_M=8, num_stages=None, num_warps=None,
                      *, out_dtype=torch.bfloat16):
    """Run the fused grouped GEMM.

    Args:
        a_fp8:    [M, K]        torch.float8_e4m3fn
        w_fp8:    [E, N, K]     torch.float8_e4m3fn
        offs:     [E+1] int32 with offs[0] == 0, or [E] cumulative ends, or [E]
                  group sizes (told apart on the device)
        a_scales: [M, K//32]    torch.uint8 E8M0 (scale 1.0 if None)
        w_scales: [E, N, K//32] torch.uint8 E8M0 (scale 1.0 if None)
        out_dtype: torch.bfloat16 (reference) or torch.float32
    Returns:
        C: [M, N] in out_dtype
    """
    return ops.grouped_fwd(a_fp8, w_fp8, offs, a_scales, w_scales, out_dtype=out_dtype)


def reference_grouped_gemm(a_fp8, w_fp8, offs):
    """Name kept from reference ``fused_fwd.py:249-264``: unscaled grouped
    forward, here on the sm_100a kernel (the CPU ground truth lives in the
    test oracle, not in the library)."""
    return ops.grouped_fwd(a_fp8, w_fp8, offs)
