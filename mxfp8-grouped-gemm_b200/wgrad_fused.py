"""Drop-in for the reference's ``wgrad_fused.py`` weight gradient.

``wgrad_fused``, ``wgrad_prepare`` and ``wgrad_kernel`` keep the signatures of
reference ``wgrad_fused.py:34-112``: ``go (N, M)`` and ``ia (K, M)`` are
token-contiguous e4m3, scales ``(N, M//32)`` / ``(K, M//32)`` E8M0, and the
result is ``grad_W[g] = GO[g] @ IA[g]^T`` of shape ``(E, N, K)``.

The reference stacks per-expert copies of both operands before reusing its
forward kernel (``wgrad_fused.py:48-62``) and assumes equal groups
(``:46``).  Here the sm_100a kernel contracts each expert's token range in
place, so ``wgrad_prepare`` makes no copies: it schedules the groups and packs
the scales once on the device, and ``wgrad_kernel`` launches only the
tensor-core kernel.  ``offs`` may be ``[E]`` group sizes (the reference docstring,
``wgrad_fused.py:37``) or ``[E]`` cumulative ends (``e2e_bench.py:42``);
boundaries must be multiples of 32 tokens.
"""
from __future__ import annotations

import torch

from . import ops


def wgrad_fused(go, ia, offs, go_scales=None, ia_scales=None, *, out_dtype=torch.bfloat16,
                **kwargs):
    """One-shot wgrad -> (E, N, K) in out_dtype (bf16 as the reference, or fp32)."""
    return ops.grouped_wgrad(go, ia, offs, go_scales, ia_scales, out_dtype=out_dtype)


def wgrad_prepare(go, ia, offs, go_scales=None, ia_scales=None):
    """Prepare once: schedule the groups and pack the scales on the device
    (no operand copies).  Returns the reference's dict plus the plan."""
    N, M = go.shape
    K = ia.shape[0]
    E = offs.shape[0]
    if (go_scales is None) != (ia_scales is None):
        go_scales = ia_scales = None
    plan = ops.GroupedWgradPlan(go_scales, ia_scales, offs, E, M, N, K, go.device)
    return {
        'A': go, 'B': ia,
        'offs': plan.offs,
        'As': go_scales, 'Bs': ia_scales,
        'E': E, 'N': N, 'K': K, 'M': M,
        'flops': 2 * M * N * K,
        'plan': plan,
    }


def wgrad_kernel(data: dict, *, out_dtype=torch.bfloat16, **kwargs):
    """Run the wgrad kernel on prepared data -> (E, N, K)."""
    plan = data.get('plan')
    if plan is None:
        return ops.grouped_wgrad(data['A'], data['B'], data['offs'], data['As'], data['Bs'],
                                 out_dtype=out_dtype, num_groups=data['E'])
    return plan.run(data['A'], data['B'], out_dtype=out_dtype)
