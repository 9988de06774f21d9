"""CPU oracle for the MXFP8 grouped-GEMM hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The CUDA library never calls into it and has no CPU fallback.

It restates, in numpy (bit-exact integer arithmetic) and torch CPU fp32/fp64
(the floating-point contraction), the algorithm of the reference
indianspeedster/mxfp8-grouped-gemm for its one hot path:

* MXFP8 quantisation (1x32 row-wise along K, 32x1 column-wise along tokens),
  e4m3 elements with E8M0 power-of-two block scales.  The reference does not
  vendor its quantiser: it calls torchao's ``triton_to_mxfp8_dim0/dim1`` under
  the ``mxfp8_rceil`` recipe (reference ``port_mxfp8.py:43-49,207-212``,
  ``memory/2026-06-09.md:10,20``).  torchao is absent here, so the published
  RCEIL rule is restated: ``descale = amax/448`` in fp32,
  ``byte = clamp(ceil(log2(descale)), -127, 127) + 127`` (NaN -> 0xFF),
  elements ``e4m3_rne(clamp(x * 2**(127-byte), -448, 448))`` with the factor
  1.0 when ``byte == 0``.
* E8M0 decode ``2**(byte-127)`` (reference ``scale_correctness.py:30-35``) and
  the round-to-nearest E8M0 encoder the reference's known-answer tests use
  (``scale_correctness.py:38-45``).
* Grouped forward ``y[rows of g] = deq(x[rows of g]) @ deq(W[g]).T``
  (reference ``fused_fwd.py:249-264`` unscaled; ``scale_correctness.py:110-137``
  with scales) and grouped weight gradient
  ``dW[g] = deq(go[:, tokens of g]) @ deq(ia[:, tokens of g]).T``
  (reference ``wgrad_fused.py:34-71``), with the ground truth taken in fp64 on
  the fp32-exact dequantised operands.
* The three ``offs`` conventions the reference uses (``fused_fwd.py:7,181``
  ``[E+1]`` leading zero; ``fwd_final.py:170-171`` ``[E]`` cumulative ends;
  ``wgrad_fused.py:37`` ``[E]`` group sizes).

Parity of this restatement is pinned by ``tests/golden`` fixtures generated
by running the reference's own torch code (``reference_grouped_gemm``, the
``scale_correctness.py`` known-answer tests and helpers) in this container.
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
E8M0_BIAS = 127
BLOCK = 32

OFFS_LEADING_ZERO = 0   # [E+1], offs[0] == 0, offs[e+1] = end of group e
OFFS_CUMULATIVE = 1     # [E],   offs[e] = end of group e
OFFS_SIZES = 2          # [E],   offs[e] = number of rows of group e
OFFS_AUTO = 3           # [E]:   cumulative if non-decreasing with last == M, else sizes


# --------------------------------------------------------------------------
# bf16 helpers (bf16 carried as uint16 bit patterns)
# --------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> exact float32 values."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


# --------------------------------------------------------------------------
# E8M0 scales
# --------------------------------------------------------------------------
def e8m0_to_float(b: np.ndarray) -> np.ndarray:
    """E8M0 byte -> 2**(b-127) as float64; 0xFF -> NaN
    (reference ``scale_correctness.py:30-35``; OCP MX v1.0 E8M0)."""
    b = np.asarray(b).astype(np.int64)
    out = np.ldexp(1.0, b - E8M0_BIAS)
    return np.where(b == 255, np.nan, out)


def e8m0_round_nearest(scale: float) -> int:
    """Round-to-nearest E8M0 encoder used by the reference's known-answer
    tests (``scale_correctness.py:38-45``)."""
    import math
    return max(0, min(255, round(math.log2(scale)) + E8M0_BIAS))


def rceil_scale_from_amax_bits(amax_bits: np.ndarray) -> np.ndarray:
    """RCEIL E8M0 byte from the bf16 bit pattern of a block's amax.

    Exact restatement of ``clamp(ceil(log2(amax/448)), -127, 127) + 127``:
    with amax = m * 2**E (m in [1,2)), amax <= 448 * 2**e  <=>
    e >= E - 8 + [m > 1.75].  NaN amax -> 0xFF; +Inf -> 254; 0 -> 0.
    """
    ab = amax_bits.astype(np.uint32)
    f32 = ab << 16
    exp_field = (f32 >> 23).astype(np.int64)
    mant = f32 & 0x7FFFFF
    e = exp_field - 127 - 8 + (mant > 0x600000).astype(np.int64)
    byte = np.clip(e, -E8M0_BIAS, E8M0_BIAS) + E8M0_BIAS
    byte = np.where(ab == 0, 0, byte)
    byte = np.where(ab == 0x7F80, 254, byte)
    byte = np.where(ab > 0x7F80, 255, byte)
    return byte.astype(np.uint8)


def descale_factor(byte: np.ndarray) -> np.ndarray:
    """Multiplier applied to the data before the e4m3 cast:
    1.0 for byte 0, else 2**(127-byte) (2**-128 for 0xFF)."""
    b = byte.astype(np.int64)
    f = np.ldexp(1.0, E8M0_BIAS - b)
    return np.where(b == 0, 1.0, f)


# --------------------------------------------------------------------------
# e4m3 (float8_e4m3fn)
# --------------------------------------------------------------------------
def _e4m3_decode_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float64)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            t[code] = np.nan
        elif e == 0:
            t[code] = s * m * 2.0 ** -9
        else:
            t[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_DECODE = _e4m3_decode_table()


def e4m3_encode_rne(v: np.ndarray) -> np.ndarray:
    """float64 values with |v| <= 448 (or NaN) -> e4m3fn codes, round to
    nearest even; NaN keeps its sign (0x7F / 0xFF) as torch's cast does."""
    v = np.asarray(v, dtype=np.float64)
    sign = np.signbit(v)
    a = np.abs(v)
    nan = np.isnan(v)
    a = np.where(nan, 0.0, a)
    # exponent of the value, floor(log2 a), with subnormals pinned to -6
    _, ex = np.frexp(a)              # a = f * 2**ex, f in [0.5, 1)
    e = np.maximum(ex - 1, -6)
    q = np.rint(np.ldexp(a, 3 - e))  # multiples of 2**(e-3), ties to even
    code = np.where(a == 0, 0, (e + 6) * 8 + q).astype(np.int64)
    code = np.minimum(code, 0x7E)
    code = np.where(nan, 0x7F, code)
    code = code | (sign.astype(np.int64) << 7)
    return code.astype(np.uint8)


# --------------------------------------------------------------------------
# quantisation
# --------------------------------------------------------------------------
def quantize_blocks(bits: np.ndarray):
    """Quantise bf16 bit patterns of shape [..., nblk, 32] block-wise.
    Returns (codes uint8 same shape, scale bytes uint8 [..., nblk])."""
    absb = bits & 0x7FFF
    amax = absb.max(axis=-1)
    scale = rceil_scale_from_amax_bits(amax)
    x = bf16_bits_to_f32(bits).astype(np.float64)
    v = x * descale_factor(scale)[..., None]
    v = np.clip(v, -E4M3_MAX, E4M3_MAX)   # NaN passes through
    return e4m3_encode_rne(v), scale


def quantize_rowwise(bits: np.ndarray):
    """MXFP8 1x32 along the last dim (the reference's dim0 / row-wise cast):
    bf16 bits [R, C] -> (q [R, C] uint8, scales [R, C/32] uint8)."""
    R, C = bits.shape
    assert C % BLOCK == 0
    q, s = quantize_blocks(bits.reshape(R, C // BLOCK, BLOCK))
    return q.reshape(R, C), s


def quantize_colwise(bits: np.ndarray):
    """MXFP8 32x1 along the first dim (tokens), output transposed
    (feature-major, token-contiguous) as the reference's wgrad operands
    ``go (N, M)`` / ``ia (K, M)`` (``wgrad_fused.py:35-39``):
    bf16 bits [R, C] -> (qT [C, R] uint8, scalesT [C, R/32] uint8)."""
    R, C = bits.shape
    assert R % BLOCK == 0
    return quantize_rowwise(np.ascontiguousarray(bits.T))


def dequantize(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """codes [R, C] + scales [R, C/32] -> float64 [R, C] (exact)."""
    R, C = q.shape
    v = E4M3_DECODE[q].reshape(R, C // BLOCK, BLOCK)
    return (v * e8m0_to_float(s)[..., None]).reshape(R, C)


# --------------------------------------------------------------------------
# group metadata
# --------------------------------------------------------------------------
def offs_to_bounds(offs, E: int, M: int, kind: int = OFFS_AUTO):
    """Group boundaries (starts, ends) from any of the reference's offs
    conventions.  Raises ValueError on inconsistent offsets."""
    o = [int(v) for v in np.asarray(offs).reshape(-1)]
    if kind == OFFS_AUTO:
        if len(o) == E + 1:
            kind = OFFS_LEADING_ZERO
        elif len(o) == E:
            mono = all(o[i] <= o[i + 1] for i in range(E - 1))
            if mono and o[-1] == M:
                kind = OFFS_CUMULATIVE
            elif all(v >= 0 for v in o) and sum(o) == M:
                kind = OFFS_SIZES
            else:
                raise ValueError("[E] offs are neither cumulative ends nor sizes summing to M")
        else:
            raise ValueError(f"offs has {len(o)} entries for E={E}")
    if kind == OFFS_LEADING_ZERO:
        if len(o) != E + 1 or o[0] != 0:
            raise ValueError("[E+1] offs must start with 0")
        ends = o[1:]
    elif kind == OFFS_CUMULATIVE:
        if len(o) != E:
            raise ValueError("[E] cumulative offs expected")
        ends = o
    elif kind == OFFS_SIZES:
        if len(o) != E or any(v < 0 for v in o):
            raise ValueError("[E] non-negative group sizes expected")
        ends = list(np.cumsum(o)) if o else []
    else:
        raise ValueError(f"unknown offs kind {kind}")
    starts = [0] + list(ends[:-1])
    for s, e in zip(starts, ends):
        if e < s or e > M:
            raise ValueError("group boundaries must be non-decreasing and <= M")
    return [int(v) for v in starts], [int(v) for v in ends]


# --------------------------------------------------------------------------
# grouped GEMMs (ground truth in fp64 on exact dequantised operands)
# --------------------------------------------------------------------------
def grouped_fwd(a_q, a_s, w_q, w_s, starts, ends, rows=None):
    """y[r, n] = sum_k deq(a)[r, k] * deq(w[g(r)])[n, k] (fp64).

    a_q [M, K] uint8, a_s [M, K/32] uint8 (None -> unit scale 0x7F),
    w_q [E, N, K] uint8, w_s [E, N, K/32].  Rows outside every group are 0.
    ``rows`` optionally restricts the computation to a subset of row indices
    (returns [len(rows), N]) for sampled checks at full problem size.
    """
    M, K = a_q.shape
    E, N, _ = w_q.shape
    if a_s is None:
        a_s = np.full((M, K // BLOCK), E8M0_BIAS, np.uint8)
    if w_s is None:
        w_s = np.full((E, N, K // BLOCK), E8M0_BIAS, np.uint8)
    rows = np.arange(M) if rows is None else np.asarray(rows)
    out = np.zeros((len(rows), N), dtype=np.float64)
    for g in range(E):
        sel = np.nonzero((rows >= starts[g]) & (rows < ends[g]))[0]
        if len(sel) == 0:
            continue
        r = rows[sel]
        a = dequantize(a_q[r], a_s[r])
        w = dequantize(w_q[g], w_s[g])
        out[sel] = a @ w.T
    return out


def grouped_wgrad(go_q, go_s, ia_q, ia_s, starts, ends, experts=None):
    """dW[g] = deq(go)[:, tokens of g] @ deq(ia)[:, tokens of g].T (fp64).

    go_q [N, M] uint8 + go_s [N, M/32]; ia_q [K, M] + ia_s [K, M/32]
    (None -> unit scale).  Returns [len(experts), N, K]; empty groups -> 0.
    """
    N, M = go_q.shape
    K = ia_q.shape[0]
    if go_s is None:
        go_s = np.full((N, M // BLOCK), E8M0_BIAS, np.uint8)
    if ia_s is None:
        ia_s = np.full((K, M // BLOCK), E8M0_BIAS, np.uint8)
    experts = range(len(starts)) if experts is None else experts
    out = np.zeros((len(experts), N, K), dtype=np.float64)
    go = dequantize(go_q, go_s)
    ia = dequantize(ia_q, ia_s)
    for i, g in enumerate(experts):
        s, e = starts[g], ends[g]
        if e > s:
            out[i] = go[:, s:e] @ ia[:, s:e].T
    return out


def rel_frobenius(x, ref) -> float:
    """||x - ref||_F / ||ref||_F (0 when both are zero)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    if den == 0.0:
        return float(num)
    return float(num / den)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float64 -> nearest bf16 value (as float64), via fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, np.float32))).astype(np.float64)


def dequantize_torch(q, s):
    """torch CPU fp32 dequantisation (the reference's own torch path,
    ``scale_correctness.py:110-137`` / ``fused_fwd.py:249-264`` without the
    bf16 rounding): codes uint8 [R, C] + scales uint8 [R, C/32] -> fp32."""
    import torch
    R, C = q.shape
    v = q.contiguous().view(torch.float8_e4m3fn).to(torch.float32).view(R, C // BLOCK, BLOCK)
    sc = torch.exp2(s.to(torch.float32) - float(E8M0_BIAS)).unsqueeze(-1)
    return (v * sc).view(R, C)
