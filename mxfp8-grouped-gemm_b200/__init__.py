"""mxg: B200-native (sm_100a) MXFP8 grouped GEMM.

Import with ``importlib.import_module("mxfp8-grouped-gemm_b200")`` (the
directory name is not a Python identifier) after putting the repository root
on ``sys.path``.  The compute runs in ``libmxg.so`` (C ABI, ``include/mxg.h``);
build it with ``python mxfp8-grouped-gemm_b200/build.py``.
"""
from . import _lib, autograd, ep, moe, ops, workloads
from .autograd import grouped_mm
from .ep import ExpertParallel
from ._lib import MxgError, device_error, raise_device_error
from .fused_fwd import fused_grouped_fwd, reference_grouped_gemm
from .fwd_final import fwd_ge
from .quantize import quantize_colwise, quantize_rowwise, to_mxfp8_dim0, to_mxfp8_dim1
from .wgrad_fused import wgrad_fused, wgrad_kernel, wgrad_prepare

__all__ = [
    "fused_grouped_fwd", "reference_grouped_gemm", "fwd_ge",
    "wgrad_fused", "wgrad_prepare", "wgrad_kernel",
    "quantize_rowwise", "quantize_colwise", "to_mxfp8_dim0", "to_mxfp8_dim1",
    "grouped_mm", "ExpertParallel", "MxgError", "device_error", "raise_device_error",
    "autograd", "ep", "moe", "ops", "workloads",
]
