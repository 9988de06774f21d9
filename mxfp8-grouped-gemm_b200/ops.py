"""Tensor-level wrappers over the C ABI (argument checks, output and
workspace allocation, current-stream launch).  The reference-named drop-in
functions in ``fused_fwd.py``, ``fwd_final.py`` and ``wgrad_fused.py`` are
thin layers over these.
"""
from __future__ import annotations

import torch

from . import _lib

_FP8 = (torch.float8_e4m3fn, torch.uint8)
_SC = (torch.uint8, getattr(torch, "float8_e8m0fnu", torch.uint8))
_OUT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


def _cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def _operand(t: torch.Tensor, name: str) -> torch.Tensor:
    _cuda(t, name)
    if t.dtype not in _FP8:
        raise TypeError(f"{name} must be float8_e4m3fn (or its uint8 bytes), got {t.dtype}")
    return t if t.is_contiguous() else t.contiguous()


def _scales(t, name, shape):
    if t is None:
        return None
    _cuda(t, name)
    if t.dtype not in _SC:
        raise TypeError(f"{name} must hold E8M0 bytes (uint8), got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    return t if t.is_contiguous() else t.contiguous()


def _offs(offs: torch.Tensor, device) -> torch.Tensor:
    if offs.dtype != torch.int32:
        offs = offs.to(torch.int32)
    if offs.device != device:
        offs = offs.to(device, non_blocking=True)
    return offs.contiguous()


def _out_code(dtype) -> int:
    if dtype not in _OUT:
        raise TypeError(f"out_dtype must be torch.bfloat16 or torch.float32, got {dtype}")
    return _OUT[dtype]


# ---------------------------------------------------------------- quantisers
def quantize_rowwise(x: torch.Tensor):
    """MXFP8 1x32 along the last dim: bf16 [R, C] -> (e4m3 [R, C], E8M0 uint8 [R, C/32])."""
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a 2-D bf16 tensor")
    x = x.contiguous()
    R, C = x.shape
    q = torch.empty(R, C, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(R, C // 32, dtype=torch.uint8, device=x.device)
    L = _lib.load()
    _lib.check(L.mxg_quantize_rowwise(x.data_ptr(), R, C, q.data_ptr(), s.data_ptr(),
                                      _lib.stream_ptr(x.device)), "mxg_quantize_rowwise")
    return q, s


def quantize_colwise(x: torch.Tensor):
    """MXFP8 32x1 along the first dim (tokens), transposed output:
    bf16 [R, C] -> (e4m3 [C, R], E8M0 uint8 [C, R/32])."""
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a 2-D bf16 tensor")
    x = x.contiguous()
    R, C = x.shape
    qt = torch.empty(C, R, dtype=torch.float8_e4m3fn, device=x.device)
    st = torch.empty(C, R // 32, dtype=torch.uint8, device=x.device)
    L = _lib.load()
    _lib.check(L.mxg_quantize_colwise(x.data_ptr(), R, C, qt.data_ptr(), st.data_ptr(),
                                      _lib.stream_ptr(x.device)), "mxg_quantize_colwise")
    return qt, st


def _dual_outputs(R, C, device, rowwise, colwise):
    q = s = qt = st = None
    if rowwise:
        q = torch.empty(R, C, dtype=torch.float8_e4m3fn, device=device)
        s = torch.empty(R, C // 32, dtype=torch.uint8, device=device)
    if colwise:
        qt = torch.empty(C, R, dtype=torch.float8_e4m3fn, device=device)
        st = torch.empty(C, R // 32, dtype=torch.uint8, device=device)
    return q, s, qt, st


def quantize_dual(x: torch.Tensor, *, rowwise=True, colwise=True):
    """Both MXFP8 encodings of bf16 x [R, C] in one pass (R, C multiples of
    32): (q [R, C], s [R, C/32], qt [C, R], st [C, R/32]); a direction not
    asked for comes back as None."""
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a 2-D bf16 tensor")
    x = x.contiguous()
    R, C = x.shape
    q, s, qt, st = _dual_outputs(R, C, x.device, rowwise, colwise)
    _lib.check(_lib.load().mxg_quantize_dual(x.data_ptr(), R, C, _lib.ptr(q), _lib.ptr(s),
                                             _lib.ptr(qt), _lib.ptr(st), _lib.stream_ptr(x.device)),
               "mxg_quantize_dual")
    return q, s, qt, st


def quantize_dual_rows(x: torch.Tensor, row_begin: int, row_end: int, out):
    """``quantize_dual`` of rows [row_begin, row_end) of x [R, C] (multiples
    of 32) into out = (q, s, qt, st) laid out for all R rows (``quantize_dual``
    shapes; None entries skip that direction): encoding x range by range
    writes the same bytes as one ``quantize_dual(x)``."""
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a 2-D bf16 tensor")
    x = x.contiguous()
    R, C = x.shape
    q, s, qt, st = out
    for t, shape, name in ((q, (R, C), "q"), (s, (R, C // 32), "s"), (qt, (C, R), "qt"), (st, (C, R // 32), "st")):
        if t is not None and (tuple(t.shape) != shape or not t.is_contiguous() or t.device != x.device):
            raise ValueError(f"{name} must be a contiguous {shape} tensor on {x.device}")
    _lib.check(_lib.load().mxg_quantize_dual_rows(x.data_ptr(), R, C, int(row_begin), int(row_end), _lib.ptr(q),
                                                  _lib.ptr(s), _lib.ptr(qt), _lib.ptr(st),
                                                  _lib.stream_ptr(x.device)), "mxg_quantize_dual_rows")
    return out


def dual_outputs(x: torch.Tensor, *, rowwise=True, colwise=True):
    """Empty (q, s, qt, st) for ``quantize_dual_rows`` of x [R, C]."""
    return _dual_outputs(x.shape[0], x.shape[1], x.device, rowwise, colwise)


def swiglu_quantize(gu: torch.Tensor, *, rowwise=True, colwise=True):
    """MXFP8 encodings of h = silu(g) * u for gu = [g | u] ([R, 2I] bf16)
    without materialising h; same bytes as ``quantize_dual(swiglu(gu))``."""
    _cuda(gu, "gu")
    if gu.dtype != torch.bfloat16 or gu.dim() != 2 or gu.shape[1] % 2:
        raise ValueError("swiglu_quantize takes a [R, 2I] bf16 tensor")
    gu = gu.contiguous()
    R, I = gu.shape[0], gu.shape[1] // 2
    q, s, qt, st = _dual_outputs(R, I, gu.device, rowwise, colwise)
    _lib.check(_lib.load().mxg_swiglu_quantize(gu.data_ptr(), R, I, _lib.ptr(q), _lib.ptr(s),
                                               _lib.ptr(qt), _lib.ptr(st),
                                               _lib.stream_ptr(gu.device)), "mxg_swiglu_quantize")
    return q, s, qt, st


def swiglu_bwd_quantize(gu: torch.Tensor, dh: torch.Tensor, *, rowwise=False, colwise=True):
    """MXFP8 encodings of the SwiGLU input gradient dgu ([R, 2I]) without
    materialising it; same bytes as ``quantize_dual(swiglu_bwd(gu, dh))``."""
    _cuda(gu, "gu")
    _cuda(dh, "dh")
    if gu.dtype != torch.bfloat16 or dh.dtype != torch.bfloat16 or gu.dim() != 2 \
            or dh.shape != (gu.shape[0], gu.shape[1] // 2) or gu.shape[1] % 2:
        raise ValueError("swiglu_bwd_quantize takes gu [R, 2I] and dh [R, I], both bf16")
    gu, dh = gu.contiguous(), dh.contiguous()
    R, I = dh.shape
    q, s, qt, st = _dual_outputs(R, 2 * I, gu.device, rowwise, colwise)
    _lib.check(_lib.load().mxg_swiglu_bwd_quantize(gu.data_ptr(), dh.data_ptr(), R, I, _lib.ptr(q),
                                                   _lib.ptr(s), _lib.ptr(qt), _lib.ptr(st),
                                                   _lib.stream_ptr(gu.device)),
               "mxg_swiglu_bwd_quantize")
    return q, s, qt, st


# ---------------------------------------------------------------- GEMMs
def grouped_fwd(a, w, offs, a_scales=None, w_scales=None, *, out_dtype=torch.bfloat16,
                offs_kind=_lib.OFFS_AUTO, out=None):
    """y[rows of g] = deq(a[rows of g]) @ deq(w[g]).T for every group g.

    a [M, K] e4m3, w [E, N, K] e4m3, a_scales [M, K/32], w_scales [E, N, K/32]
    (uint8 E8M0; None = unit scale), offs int32 in any of the three conventions.
    """
    a = _operand(a, "a_fp8")
    w = _operand(w, "w_fp8")
    M, K = a.shape
    E, N, K2 = w.shape
    assert K == K2, f"K mismatch: {K} vs {K2}"
    if (a_scales is None) != (w_scales is None):
        # the reference applies scales only when both are given (fused_fwd.py:191)
        a_scales = w_scales = None
    a_scales = _scales(a_scales, "a_scales", (M, K // 32))
    w_scales = _scales(w_scales, "w_scales", (E, N, K // 32))
    offs = _offs(offs, a.device)
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    L = _lib.load()
    nbytes = L.mxg_grouped_fwd_workspace_size(E, M, N, K)
    ws = _lib.workspace(nbytes, a.device)
    _lib.check(L.mxg_grouped_fwd(a.data_ptr(), _lib.ptr(a_scales), w.data_ptr(), _lib.ptr(w_scales),
                                 offs.data_ptr(), offs.numel(), offs_kind, E, M, N, K,
                                 out.data_ptr(), _out_code(out.dtype), ws.data_ptr(), ws.numel(),
                                 _lib.stream_ptr(a.device)), "mxg_grouped_fwd")
    return out


def dense_fwd_kn(x, w_kn, *, out_dtype=torch.bfloat16):
    """out[M, N] = x[M, K] @ w[K, N] on e4m3 operands with unit scales."""
    x = _operand(x, "x_fp8")
    w_kn = _operand(w_kn, "w_fp8")
    M, K = x.shape
    K2, N = w_kn.shape
    assert K == K2
    out = torch.empty(M, N, dtype=out_dtype, device=x.device)
    L = _lib.load()
    ws = _lib.workspace(L.mxg_dense_fwd_kn_workspace_size(M, N, K), x.device)
    _lib.check(L.mxg_dense_fwd_kn(x.data_ptr(), w_kn.data_ptr(), M, N, K, out.data_ptr(),
                                  _out_code(out_dtype), ws.data_ptr(), ws.numel(),
                                  _lib.stream_ptr(x.device)), "mxg_dense_fwd_kn")
    return out


def grouped_wgrad(go, ia, offs, go_scales=None, ia_scales=None, *, out_dtype=torch.bfloat16,
                  offs_kind=_lib.OFFS_AUTO, num_groups=None, out=None):
    """dW[g] = deq(go[:, tokens of g]) @ deq(ia[:, tokens of g]).T -> [E, N, K].

    go [N, M] e4m3 and ia [K, M] e4m3 (token-contiguous), go_scales [N, M/32],
    ia_scales [K, M/32]; group boundaries multiples of 32 tokens.
    """
    go = _operand(go, "go")
    ia = _operand(ia, "ia")
    N, M = go.shape
    K, M2 = ia.shape
    assert M == M2, f"token count mismatch: {M} vs {M2}"
    if (go_scales is None) != (ia_scales is None):
        go_scales = ia_scales = None
    go_scales = _scales(go_scales, "go_scales", (N, M // 32))
    ia_scales = _scales(ia_scales, "ia_scales", (K, M // 32))
    offs = _offs(offs, go.device)
    E = num_groups if num_groups is not None else (
        offs.numel() - 1 if offs_kind == _lib.OFFS_LEADING_ZERO else offs.numel())
    if out is None:
        out = torch.empty(E, N, K, dtype=out_dtype, device=go.device)
    L = _lib.load()
    ws = _lib.workspace(L.mxg_grouped_wgrad_workspace_size(E, M, N, K), go.device)
    _lib.check(L.mxg_grouped_wgrad(go.data_ptr(), _lib.ptr(go_scales), ia.data_ptr(),
                                   _lib.ptr(ia_scales), offs.data_ptr(), offs.numel(), offs_kind,
                                   E, M, N, K, out.data_ptr(), _out_code(out.dtype), ws.data_ptr(),
                                   ws.numel(), _lib.stream_ptr(go.device)), "mxg_grouped_wgrad")
    return out


def transpose_u8(x: torch.Tensor) -> torch.Tensor:
    """Byte transpose of a 2-D 1-byte tensor on the device."""
    _cuda(x, "x")
    x = x.contiguous()
    R, C = x.shape
    y = torch.empty(C, R, dtype=x.dtype, device=x.device)
    _lib.check(_lib.load().mxg_transpose_u8(x.data_ptr(), R, C, y.data_ptr(),
                                            _lib.stream_ptr(x.device)), "mxg_transpose_u8")
    return y


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """h = silu(g) * u for bf16 rows gu = [g | u] ([R, 2I] -> [R, I]); the
    activation between the gate/up and down projections of an expert."""
    _cuda(gu, "gu")
    if gu.dtype != torch.bfloat16 or gu.dim() != 2 or gu.shape[1] % 2:
        raise ValueError("swiglu takes a [R, 2I] bf16 tensor")
    gu = gu.contiguous()
    R, I2 = gu.shape
    h = torch.empty(R, I2 // 2, dtype=torch.bfloat16, device=gu.device)
    _lib.check(_lib.load().mxg_swiglu(gu.data_ptr(), R, I2 // 2, h.data_ptr(),
                                      _lib.stream_ptr(gu.device)), "mxg_swiglu")
    return h


def swiglu_bwd(gu: torch.Tensor, dh: torch.Tensor) -> torch.Tensor:
    """Gradient of ``swiglu`` w.r.t. gu = [g | u]: bf16 [R, 2I] from dh [R, I]."""
    _cuda(gu, "gu")
    _cuda(dh, "dh")
    if gu.dtype != torch.bfloat16 or dh.dtype != torch.bfloat16 or gu.dim() != 2 \
            or dh.shape != (gu.shape[0], gu.shape[1] // 2) or gu.shape[1] % 2:
        raise ValueError("swiglu_bwd takes gu [R, 2I] and dh [R, I], both bf16")
    gu, dh = gu.contiguous(), dh.contiguous()
    dgu = torch.empty_like(gu)
    _lib.check(_lib.load().mxg_swiglu_bwd(gu.data_ptr(), dh.data_ptr(), gu.shape[0], dh.shape[1],
                                          dgu.data_ptr(), _lib.stream_ptr(gu.device)),
               "mxg_swiglu_bwd")
    return dgu


class gemm_sm_limit:
    """Context manager: the grouped GEMMs launched inside use at most ``sms``
    SMs (None or 0: all), leaving the rest to kernels on other streams."""

    def __init__(self, sms):
        self.sms = int(sms or 0)

    def __enter__(self):
        L = _lib.load()
        self.prev = L.mxg_get_gemm_sm_limit()
        _lib.check(L.mxg_set_gemm_sm_limit(self.sms), "mxg_set_gemm_sm_limit")
        return self

    def __exit__(self, *exc):
        _lib.load().mxg_set_gemm_sm_limit(self.prev)


# ---------------------------------------------------------------- two-phase plans
class GroupedFwdPlan:
    """Groups and packed scales of one grouped forward, prepared once in a
    workspace owned by the plan; ``run`` launches only the tensor-core kernel."""

    def __init__(self, a_scales, w_scales, offs, num_groups, M, N, K, device,
                 offs_kind=_lib.OFFS_AUTO):
        L = _lib.load()
        self.E, self.M, self.N, self.K = int(num_groups), int(M), int(N), int(K)
        self.a_scales = _scales(a_scales, "a_scales", (M, K // 32))
        self.w_scales = _scales(w_scales, "w_scales", (num_groups, N, K // 32))
        self.offs = _offs(offs, device)
        self.ws = torch.empty(max(L.mxg_grouped_fwd_workspace_size(self.E, M, N, K), 1024),
                              dtype=torch.uint8, device=device)
        _lib.check(L.mxg_grouped_fwd_prepare(_lib.ptr(self.a_scales), _lib.ptr(self.w_scales),
                                             self.offs.data_ptr(), self.offs.numel(), offs_kind,
                                             self.E, M, N, K, self.ws.data_ptr(), self.ws.numel(),
                                             _lib.stream_ptr(device)), "mxg_grouped_fwd_prepare")

    def run(self, a, w, out=None, out_dtype=torch.bfloat16):
        a = _operand(a, "a_fp8")
        w = _operand(w, "w_fp8")
        if out is None:
            out = torch.empty(self.M, self.N, dtype=out_dtype, device=a.device)
        _lib.check(_lib.load().mxg_grouped_fwd_run(
            a.data_ptr(), w.data_ptr(), self.E, self.M, self.N, self.K, out.data_ptr(),
            _out_code(out.dtype), self.ws.data_ptr(), self.ws.numel(), _lib.stream_ptr(a.device)),
            "mxg_grouped_fwd_run")
        return out


    def run_scatter(self, a, w, dst_bufs, back_rank, back_row, dst_rows):
        """The forward with its bf16 output rows stored into other buffers
        (this GPU's or peers'): row q to row back_row[q] of the buffer at
        address dst_bufs[back_rank[q]] (dst_bufs: int64 device tensor of
        addresses; back_rank < 0 drops the row)."""
        a = _operand(a, "a_fp8")
        w = _operand(w, "w_fp8")
        _lib.check(_lib.load().mxg_grouped_fwd_run_scatter(
            a.data_ptr(), w.data_ptr(), self.E, self.M, self.N, self.K, dst_bufs.data_ptr(),
            dst_bufs.numel(), back_rank.data_ptr(), back_row.data_ptr(), dst_rows, self.ws.data_ptr(),
            self.ws.numel(), _lib.stream_ptr(a.device)), "mxg_grouped_fwd_run_scatter")


class GroupedWgradPlan:
    """Groups and packed scales of one grouped weight gradient (the
    counterpart of the reference's wgrad_prepare, without operand copies)."""

    def __init__(self, go_scales, ia_scales, offs, num_groups, M, N, K, device,
                 offs_kind=_lib.OFFS_AUTO):
        L = _lib.load()
        self.E, self.M, self.N, self.K = int(num_groups), int(M), int(N), int(K)
        self.go_scales = _scales(go_scales, "go_scales", (N, M // 32))
        self.ia_scales = _scales(ia_scales, "ia_scales", (K, M // 32))
        self.offs = _offs(offs, device)
        self.ws = torch.empty(max(L.mxg_grouped_wgrad_workspace_size(self.E, M, N, K), 1024),
                              dtype=torch.uint8, device=device)
        _lib.check(L.mxg_grouped_wgrad_prepare(_lib.ptr(self.go_scales), _lib.ptr(self.ia_scales),
                                               self.offs.data_ptr(), self.offs.numel(), offs_kind,
                                               self.E, M, N, K, self.ws.data_ptr(), self.ws.numel(),
                                               _lib.stream_ptr(device)), "mxg_grouped_wgrad_prepare")

    def run(self, go, ia, out=None, out_dtype=torch.bfloat16):
        go = _operand(go, "go")
        ia = _operand(ia, "ia")
        if out is None:
            out = torch.empty(self.E, self.N, self.K, dtype=out_dtype, device=go.device)
        _lib.check(_lib.load().mxg_grouped_wgrad_run(
            go.data_ptr(), ia.data_ptr(), self.E, self.M, self.N, self.K, out.data_ptr(),
            _out_code(out.dtype), self.ws.data_ptr(), self.ws.numel(), _lib.stream_ptr(go.device)),
            "mxg_grouped_wgrad_run")
        return out
