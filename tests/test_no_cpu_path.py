"""The package has no CPU path: every compute entry point refuses host
tensors with an error instead of computing something on the CPU."""
import numpy as np
import pytest
import torch


def _fp8(*shape):
    return torch.zeros(*shape, dtype=torch.uint8).view(torch.float8_e4m3fn)


def test_quantisers_refuse_host_tensors(mxg):
    x = torch.zeros(64, 64, dtype=torch.bfloat16)
    for fn in (mxg.quantize_rowwise, mxg.quantize_colwise, mxg.ops.quantize_dual):
        with pytest.raises(ValueError, match="CUDA"):
            fn(x)
    gu = torch.zeros(64, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        mxg.ops.swiglu_quantize(gu)
    with pytest.raises(ValueError, match="CUDA"):
        mxg.ops.swiglu_bwd_quantize(gu, torch.zeros(64, 64, dtype=torch.bfloat16))


def test_gemms_refuse_host_tensors(mxg):
    a, w = _fp8(64, 64), _fp8(2, 32, 64)
    offs = torch.tensor([32, 32], dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        mxg.fused_grouped_fwd(a, w, offs)
    with pytest.raises(ValueError, match="CUDA"):
        mxg.ops.grouped_wgrad(_fp8(32, 64), _fp8(16, 64), offs)
    with pytest.raises(ValueError, match="CUDA"):
        mxg.fwd_ge(a, _fp8(64, 32))


def test_layer_pieces_refuse_host_tensors(mxg):
    with pytest.raises(ValueError, match="CUDA"):
        mxg.ops.swiglu(torch.zeros(4, 64, dtype=torch.bfloat16))
    ids = torch.from_numpy(np.zeros((4, 2), np.int32))
    with pytest.raises((ValueError, RuntimeError)):
        mxg.ExpertParallel(8).dispatch(torch.zeros(4, 64, dtype=torch.bfloat16), ids)
