// MXFP8 quantisers for sm_100a: bf16 -> e4m3 elements + E8M0 block scales.
//
// Scale rule (RCEIL, the rounding of the mxfp8_rceil recipe the reference's
// MoE path uses, port_mxfp8.py:207-212): for a block of 32 values with
// amax = max|x|, byte = clamp(ceil(log2(amax / 448)), -127, 127) + 127, NaN
// amax -> 0xFF.  It is evaluated exactly on the bf16 bit pattern of amax
// (amax = m * 2^E, m in [1,2): e = E - 8 + [m > 1.75]), which equals the
// fp32 formula for every bf16 input.  Elements: e4m3_rne(x * 2^(127-byte)),
// the factor being 1.0 for byte 0, saturated to +-448 (hardware satfinite
// conversion), NaN kept as NaN with its sign.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "mxg.h"
#include "mxg_device.cuh"
#include "mxg_internal.h"
#include "mxg_ptx.cuh"

namespace mxg {

// ---------------------------------------------------------------- row-wise
// One thread per 16-byte chunk (8 bf16); four consecutive lanes form one
// 32-element block and reduce its amax with two xor-shuffles.
constexpr int kRowUnroll = 4;

__global__ void __launch_bounds__(256) quant_rowwise_kernel(const uint4* __restrict__ x,
                                                            uint2* __restrict__ q,
                                                            uint8_t* __restrict__ s,
                                                            int64_t nchunks) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t tid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  // every lane of a warp runs the same number of iterations (shuffles below)
  const int64_t base_warp = tid & ~int64_t(31);
  for (int64_t i0 = base_warp; i0 < nchunks; i0 += stride * kRowUnroll) {
    uint4 v[kRowUnroll];
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      const int64_t i = i0 + int64_t(u) * stride + lane;
      if (i < nchunks) {
        v[u] = __ldcs(x + i);
      } else {
        v[u] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      const int64_t i = i0 + int64_t(u) * stride + lane;
      // (per-word maxima here: the SIMD half-word form measured 25% slower
      // in this unrolled loop, unlike in the tiled kernels below)
      uint32_t m = amax2(v[u].x);
      m = max(m, amax2(v[u].y));
      m = max(m, amax2(v[u].z));
      m = max(m, amax2(v[u].w));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
      const uint32_t b = rceil_byte(m);
      const float f = descale_of(b);
      uint32_t c0 = cvt_scaled_e4m3x2(bf16_lo(v[u].x), bf16_hi(v[u].x), f);
      uint32_t c1 = cvt_scaled_e4m3x2(bf16_lo(v[u].y), bf16_hi(v[u].y), f);
      uint32_t c2 = cvt_scaled_e4m3x2(bf16_lo(v[u].z), bf16_hi(v[u].z), f);
      uint32_t c3 = cvt_scaled_e4m3x2(bf16_lo(v[u].w), bf16_hi(v[u].w), f);
      uint32_t lo = c0 | (c1 << 16), hi = c2 | (c3 << 16);
      if (b == 255u) {
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        uint32_t bytes[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t word = j < 2 ? lo : hi;
          const int sh = (j & 1) * 16;
          bytes[2 * j] = fix_nan_byte((word >> sh) & 0xFFu, w[j] & 0xFFFFu);
          bytes[2 * j + 1] = fix_nan_byte((word >> (sh + 8)) & 0xFFu, w[j] >> 16);
        }
        lo = bytes[0] | (bytes[1] << 8) | (bytes[2] << 16) | (bytes[3] << 24);
        hi = bytes[4] | (bytes[5] << 8) | (bytes[6] << 16) | (bytes[7] << 24);
      }
      if (i < nchunks) {
        __stcs(q + i, make_uint2(lo, hi));
        if ((lane & 3) == 0) s[i >> 2] = uint8_t(b);
      }
    }
  }
}

// ---------------------------------------------------------------- column-wise
// x [rows, cols] bf16, blocks of 32 rows.  A thread owns two adjacent columns
// of one 32-row block: 32 coalesced bf16x2 loads (a warp reads 128 contiguous
// bytes per row), in-thread amax, then two 32-byte runs of e4m3 codes written
// to the transposed output qt[col][row0 .. row0+32).
constexpr int kColThreads = 256;
constexpr int kColPerBlock = kColThreads * 2;

__global__ void __launch_bounds__(kColThreads) quant_colwise_kernel(
    const uint32_t* __restrict__ x, int64_t rows, int64_t cols, uint8_t* __restrict__ qt,
    uint8_t* __restrict__ st) {
  const int64_t c = (int64_t(blockIdx.x) * kColThreads + threadIdx.x) * 2;
  const int64_t r0 = int64_t(blockIdx.y) * 32;
  if (c >= cols) return;
  const int64_t ld = cols / 2;  // row stride in bf16x2 words
  uint32_t w[32];
#pragma unroll
  for (int r = 0; r < 32; ++r) w[r] = __ldcs(x + (r0 + r) * ld + c / 2);
  uint32_t m0 = 0, m1 = 0;
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    m0 = max(m0, w[r] & 0x7FFFu);
    m1 = max(m1, (w[r] >> 16) & 0x7FFFu);
  }
  const uint32_t b0 = rceil_byte(m0), b1 = rceil_byte(m1);
  const float f0 = descale_of(b0), f1 = descale_of(b1);
  uint32_t out0[8], out1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    // rows 4j .. 4j+3 of column c (low halves) and column c+1 (high halves)
    uint32_t a01 = cvt_scaled_e4m3x2(bf16_lo(w[4 * j]), bf16_lo(w[4 * j + 1]), f0);
    uint32_t a23 = cvt_scaled_e4m3x2(bf16_lo(w[4 * j + 2]), bf16_lo(w[4 * j + 3]), f0);
    uint32_t b01 = cvt_scaled_e4m3x2(bf16_hi(w[4 * j]), bf16_hi(w[4 * j + 1]), f1);
    uint32_t b23 = cvt_scaled_e4m3x2(bf16_hi(w[4 * j + 2]), bf16_hi(w[4 * j + 3]), f1);
    out0[j] = a01 | (a23 << 16);
    out1[j] = b01 | (b23 << 16);
  }
  if (b0 == 255u || b1 == 255u) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t p0 = 0, p1 = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t wr = w[4 * j + t];
        uint32_t c0 = (out0[j] >> (8 * t)) & 0xFFu, c1 = (out1[j] >> (8 * t)) & 0xFFu;
        if (b0 == 255u) c0 = fix_nan_byte(c0, wr & 0xFFFFu);
        if (b1 == 255u) c1 = fix_nan_byte(c1, wr >> 16);
        p0 |= c0 << (8 * t);
        p1 |= c1 << (8 * t);
      }
      out0[j] = p0;
      out1[j] = p1;
    }
  }
  uint4* d0 = reinterpret_cast<uint4*>(qt + c * rows + r0);
  __stcs(d0, make_uint4(out0[0], out0[1], out0[2], out0[3]));
  __stcs(d0 + 1, make_uint4(out0[4], out0[5], out0[6], out0[7]));
  st[c * (rows / 32) + blockIdx.y] = uint8_t(b0);
  if (c + 1 < cols) {
    uint4* d1 = reinterpret_cast<uint4*>(qt + (c + 1) * rows + r0);
    __stcs(d1, make_uint4(out1[0], out1[1], out1[2], out1[3]));
    __stcs(d1 + 1, make_uint4(out1[4], out1[5], out1[6], out1[7]));
    st[(c + 1) * (rows / 32) + blockIdx.y] = uint8_t(b1);
  }
}

// ---------------------------------------------------------------- fused: both directions
// One pass over a bf16 tensor [rows, cols] (rows a multiple of 32) producing
// the row-wise (1x32) and/or the column-wise (32x1, transposed) encodings,
// each bit-identical to the dedicated kernels above.  A block owns a tile of
// 64 rows x 256 columns: every thread issues eight 16-byte loads at once (a
// warp reads one 512-byte row segment each), encodes the chunks row-wise in
// registers (four lanes per 32-element block, as the row-wise kernel), parks
// them in shared memory, and after a barrier each thread encodes two tile
// columns over 32 rows for the transposed output (the two row halves of a
// column write adjacent 32-byte runs).  The tensor may be computed on the fly from its inputs
// (SwiGLU, and the SwiGLU gradient), rounded to bf16 exactly as the unfused
// kernels round their outputs, so it is never written to memory.
enum { DUAL_PLAIN = 0, DUAL_SWIGLU = 1, DUAL_SWIGLU_GRAD = 2 };
constexpr int kTileRows = 128;                // 32 KiB tiles: kTileRows x kTileCols bf16
constexpr int kTileCols = 16384 / kTileRows;

struct DualArgs {
  const uint4* a;    // x (plain) or gu (swiglu variants), rows of 16-byte chunks
  const uint4* dh;   // swiglu gradient: dh [rows, inter]
  int64_t rows;
  int64_t cols;      // columns of the encoded tensor
  int64_t inter;     // swiglu variants: I
  uint8_t* q;        // row-wise codes [rows, cols] (null: skip)
  uint8_t* s;        // row-wise scales [rows, cols/32]
  uint8_t* qt;       // column-wise codes [cols, rows] (null: skip)
  uint8_t* st;       // column-wise scales [cols, rows/32]
  int64_t row0;      // rows [row0, row_end) are encoded (launch_dual sets them;
  int64_t row_end;   // rows stays the row count the outputs are laid out for)
};

__device__ __forceinline__ uint4 swiglu_chunk(uint4 g, uint4 u) {
  return make_uint4(pack2_bf16(silu_mul(bf16_lo(g.x), bf16_lo(u.x)), silu_mul(bf16_hi(g.x), bf16_hi(u.x))),
                    pack2_bf16(silu_mul(bf16_lo(g.y), bf16_lo(u.y)), silu_mul(bf16_hi(g.y), bf16_hi(u.y))),
                    pack2_bf16(silu_mul(bf16_lo(g.z), bf16_lo(u.z)), silu_mul(bf16_hi(g.z), bf16_hi(u.z))),
                    pack2_bf16(silu_mul(bf16_lo(g.w), bf16_lo(u.w)), silu_mul(bf16_hi(g.w), bf16_hi(u.w))));
}

__device__ __forceinline__ void swiglu_grad_word(uint32_t g, uint32_t u, uint32_t d, uint32_t& dg,
                                                 uint32_t& du) {
  float dg0, du0, dg1, du1;
  silu_mul_grad(bf16_lo(g), bf16_lo(u), bf16_lo(d), dg0, du0);
  silu_mul_grad(bf16_hi(g), bf16_hi(u), bf16_hi(d), dg1, du1);
  dg = pack2_bf16(dg0, dg1);
  du = pack2_bf16(du0, du1);
}

// Row-wise encoding of one 8-element chunk; the four lanes of its 32-element
// block must call this together.
__device__ __forceinline__ void encode_row_chunk(const DualArgs& a, uint4 v, int64_t row,
                                                 int64_t col, bool valid) {
  uint32_t m2 = amax_chunk2(v);
  m2 = max2(m2, __shfl_xor_sync(0xffffffffu, m2, 1));
  m2 = max2(m2, __shfl_xor_sync(0xffffffffu, m2, 2));
  const uint32_t m = halves_max(m2);
  const uint32_t b = rceil_byte(m);
  const float f = descale_of(b);
  uint32_t c0 = cvt_scaled_e4m3x2(bf16_lo(v.x), bf16_hi(v.x), f);
  uint32_t c1 = cvt_scaled_e4m3x2(bf16_lo(v.y), bf16_hi(v.y), f);
  uint32_t c2 = cvt_scaled_e4m3x2(bf16_lo(v.z), bf16_hi(v.z), f);
  uint32_t c3 = cvt_scaled_e4m3x2(bf16_lo(v.w), bf16_hi(v.w), f);
  uint32_t lo = c0 | (c1 << 16), hi = c2 | (c3 << 16);
  if (b == 255u) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t bytes[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t word = j < 2 ? lo : hi;
      const int sh = (j & 1) * 16;
      bytes[2 * j] = fix_nan_byte((word >> sh) & 0xFFu, w[j] & 0xFFFFu);
      bytes[2 * j + 1] = fix_nan_byte((word >> (sh + 8)) & 0xFFu, w[j] >> 16);
    }
    lo = bytes[0] | (bytes[1] << 8) | (bytes[2] << 16) | (bytes[3] << 24);
    hi = bytes[4] | (bytes[5] << 8) | (bytes[6] << 16) | (bytes[7] << 24);
  }
  if (valid) {
    __stcs(reinterpret_cast<uint2*>(a.q + row * a.cols + col), make_uint2(lo, hi));
    if ((threadIdx.x & 3) == 0) a.s[row * (a.cols / 32) + col / 32] = uint8_t(b);
  }
}

// Column pass over a staged tile (rows r0.., tile columns c0..).  Work item =
// (column pair p, 32-row block rb, half h): the two lanes of a pair (h =
// lane & 1) take rows [32rb, 32rb+16) and [32rb+16, 32rb+32) of columns 2p,
// 2p+1, share the block amax with one shuffle, and store their 16 bytes of
// each column side by side, so one store instruction writes whole 32-byte
// sectors of the transposed output.  Block scales go to col_scales.
// SWZ: the tile was staged with rows 16-31 of every 32-row block shifted by
// 16 words (16-byte chunk c stored at c ^ 4), so the two lanes of a pair,
// 16 rows apart, read different banks (register-fed kernel; TMA-fed tiles
// keep the plain layout).
template <int KIND, int NT = 256, bool SWZ = false>
__device__ __forceinline__ void dual_column_pass(const DualArgs& a, const uint32_t (*tile)[kTileCols / 2],
                                                 uint8_t (*col_scales)[kTileRows / 32], int64_t r0,
                                                 int64_t c0, int t) {
  constexpr int R = kTileRows, CW = kTileCols / 2;
  constexpr int kItems = CW * (R / 32) * 2;
#pragma unroll 1
  for (int it = t; it < kItems; it += NT) {
    const int h = it & 1, pcol = (it >> 1) % CW, rblk = (it >> 1) / CW;
    const bool row_ok = r0 + 32 * rblk < a.row_end;
    int64_t col0;
    bool col_ok;
    if (KIND == DUAL_SWIGLU_GRAD) {
      const int64_t j = c0 + 2 * (pcol % (CW / 2));
      col_ok = j < a.inter;
      col0 = pcol < CW / 2 ? j : a.inter + j;
    } else {
      col0 = c0 + 2 * pcol;
      col_ok = col0 < a.cols;
    }
    // (the partner lane always has the same rblk and pcol: same predicate)
    const uint32_t* colp = &tile[32 * rblk + 16 * h][SWZ ? (pcol ^ (h << 4)) : pcol];
    uint32_t w[16];
    uint32_t m2 = 0;  // amax bit patterns of the two columns, one per half
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      w[r] = colp[r * CW];
      m2 = max2(m2, abs2(w[r]));
    }
    m2 = max2(m2, __shfl_xor_sync(0xffffffffu, m2, 1));
    const uint32_t m0 = m2 & 0xFFFFu, m1 = m2 >> 16;
    if (!row_ok || !col_ok) continue;
    const uint32_t b0 = rceil_byte(m0), b1 = rceil_byte(m1);
    const float f0 = descale_of(b0), f1 = descale_of(b1);
    uint32_t o0[4], o1[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a01 = cvt_scaled_e4m3x2(bf16_lo(w[4 * j]), bf16_lo(w[4 * j + 1]), f0);
      const uint32_t a23 = cvt_scaled_e4m3x2(bf16_lo(w[4 * j + 2]), bf16_lo(w[4 * j + 3]), f0);
      const uint32_t b01 = cvt_scaled_e4m3x2(bf16_hi(w[4 * j]), bf16_hi(w[4 * j + 1]), f1);
      const uint32_t b23 = cvt_scaled_e4m3x2(bf16_hi(w[4 * j + 2]), bf16_hi(w[4 * j + 3]), f1);
      o0[j] = a01 | (a23 << 16);
      o1[j] = b01 | (b23 << 16);
      if (b0 == 255u || b1 == 255u) {
        uint32_t p0 = 0, p1 = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t x0 = (o0[j] >> (8 * q)) & 0xFFu, x1 = (o1[j] >> (8 * q)) & 0xFFu;
          if (b0 == 255u) x0 = fix_nan_byte(x0, w[4 * j + q] & 0xFFFFu);
          if (b1 == 255u) x1 = fix_nan_byte(x1, w[4 * j + q] >> 16);
          p0 |= x0 << (8 * q);
          p1 |= x1 << (8 * q);
        }
        o0[j] = p0;
        o1[j] = p1;
      }
    }
    const int64_t rb = r0 + 32 * rblk;
    *reinterpret_cast<uint4*>(a.qt + col0 * a.rows + rb + 16 * h) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
    *reinterpret_cast<uint4*>(a.qt + (col0 + 1) * a.rows + rb + 16 * h) =
        make_uint4(o1[0], o1[1], o1[2], o1[3]);
    if (h == 0) {
      col_scales[2 * pcol][rblk] = uint8_t(b0);
      col_scales[2 * pcol + 1][rblk] = uint8_t(b1);
    }
  }
}

// The tile's column scales leave together: one thread per column writes its
// R/32 consecutive bytes (one word when aligned) instead of single bytes that
// each cost a 32-byte sector on the way to L2.
template <int KIND>
__device__ __forceinline__ void dual_store_col_scales(const DualArgs& a,
                                                      const uint8_t (*col_scales)[kTileRows / 32],
                                                      int64_t r0, int64_t c0, int t) {
  constexpr int R = kTileRows;
  if (t < kTileCols) {
    int64_t gcol;
    if (KIND == DUAL_SWIGLU_GRAD) {
      const int64_t j = c0 + (t % (kTileCols / 2));
      if (j >= a.inter) return;
      gcol = t < kTileCols / 2 ? j : a.inter + j;
    } else {
      gcol = c0 + t;
      if (gcol >= a.cols) return;
    }
    const int64_t rem = (a.row_end - r0) / 32;
    const int nb = int(rem < R / 32 ? rem : R / 32);
    uint8_t* dst = a.st + gcol * (a.rows / 32) + r0 / 32;
    if (R / 32 == 4 && nb == 4 && (reinterpret_cast<uintptr_t>(dst) & 3u) == 0) {
      *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(col_scales[t]);
    } else {
      for (int b = 0; b < nb; ++b) dst[b] = col_scales[t][b];
    }
  }
}

template <int KIND>
__global__ void __launch_bounds__(256, 3) quant_dual_kernel(DualArgs a) {
  constexpr int R = kTileRows, CW = kTileCols / 2;      // tile rows, tile width in bf16x2 words
  constexpr int CPR = kTileCols / 8;                     // 16-byte chunks per tile row
  __shared__ __align__(16) uint32_t tile[R][CW];
  __shared__ __align__(4) uint8_t col_scales[kTileCols][R / 32];  // column pass -> one write per column
  const int64_t r0 = a.row0 + int64_t(blockIdx.y) * R;
  const int t = threadIdx.x;
  // tile columns -> tensor columns: contiguous, except for the gradient where
  // the first half of the tile is dg[j0 + c] and the second du[j0 + c]
  const int64_t c0 = KIND == DUAL_SWIGLU_GRAD ? int64_t(blockIdx.x) * (kTileCols / 2)
                                              : int64_t(blockIdx.x) * kTileCols;
  if (KIND != DUAL_SWIGLU_GRAD) {
    uint4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // all loads first: 128 bytes in flight per thread
      const int k = t + 256 * i;
      const int r = k / CPR, ch = k % CPR;
      const int64_t col = c0 + ch * 8;
      v[i] = make_uint4(0, 0, 0, 0);
      if (col < a.cols && r0 + r < a.row_end) {
        if (KIND == DUAL_PLAIN) {
          v[i] = __ldcs(a.a + ((r0 + r) * a.cols + col) / 8);
        } else {
          const uint4* rowp = a.a + (r0 + r) * (2 * a.inter) / 8;
          v[i] = swiglu_chunk(__ldcs(rowp + col / 8), __ldcs(rowp + (a.inter + col) / 8));
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = t + 256 * i;
      const int r = k / CPR, ch = k % CPR;
      const int64_t col = c0 + ch * 8;
      const bool valid = col < a.cols && r0 + r < a.row_end;
      if (a.q) encode_row_chunk(a, v[i], r0 + r, col, valid);
      *reinterpret_cast<uint4*>(&tile[r][(ch ^ (((r >> 4) & 1) << 2)) * 4]) = v[i];
    }
  } else {
    constexpr int JCPR = CPR / 2;  // input chunks per tile row (each yields a dg and a du chunk)
    uint4 dg[4], du[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = t + 256 * i;
      const int r = k / JCPR, ch = k % JCPR;
      const int64_t j = c0 + ch * 8;
      dg[i] = make_uint4(0, 0, 0, 0);
      du[i] = dg[i];
      if (j < a.inter && r0 + r < a.row_end) {
        const uint4* rowp = a.a + (r0 + r) * (2 * a.inter) / 8;
        const uint4 g = __ldcs(rowp + j / 8), u = __ldcs(rowp + (a.inter + j) / 8);
        const uint4 d = __ldcs(a.dh + ((r0 + r) * a.inter + j) / 8);
        swiglu_grad_word(g.x, u.x, d.x, dg[i].x, du[i].x);
        swiglu_grad_word(g.y, u.y, d.y, dg[i].y, du[i].y);
        swiglu_grad_word(g.z, u.z, d.z, dg[i].z, du[i].z);
        swiglu_grad_word(g.w, u.w, d.w, dg[i].w, du[i].w);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = t + 256 * i;
      const int r = k / JCPR, ch = k % JCPR;
      const int64_t j = c0 + ch * 8;
      const bool valid = j < a.inter && r0 + r < a.row_end;
      if (a.q) {
        encode_row_chunk(a, dg[i], r0 + r, j, valid);
        encode_row_chunk(a, du[i], r0 + r, a.inter + j, valid);
      }
      const int sw = ((r >> 4) & 1) << 2;  // see dual_column_pass<.., SWZ>
      *reinterpret_cast<uint4*>(&tile[r][(ch ^ sw) * 4]) = dg[i];
      *reinterpret_cast<uint4*>(&tile[r][((CW / 8 + ch) ^ sw) * 4]) = du[i];
    }
  }
  if (a.qt == nullptr) return;
  __syncthreads();
  dual_column_pass<KIND, 256, true>(a, tile, col_scales, r0, c0, t);
  __syncthreads();
  dual_store_col_scales<KIND>(a, col_scales, r0, c0, t);
}

// Column-wise encodes through a persistent variant fed by TMA.  Each block
// (two per SM) keeps a ring of tiles in flight in shared memory: one thread
// issues a tile's bulk-tensor loads as soon as its slot is free, and the
// block runs the column pass above on the tile that has landed, so the HBM
// reads never wait for the encode (plain tensors: 5.6 instead of 4.9 TB/s at
// 65536 x 7168).  Plain: three 32 KiB stages of 128 x 128 bf16.  SwiGLU
// gradient: two 48 KiB stages, each 128 rows x 64 of g and u (one 3-D box
// over gu [R, 2, I], so a tile row is g then u, 256 bytes) plus the matching
// 128 x 64 of dh; dg and du are computed in place over g and u, rounded to
// bf16 as the unfused kernel rounds them.  With both encodings the
// register-fed kernel above measured faster (plain: 4.1 vs 3.7-3.9 TB/s), so
// it keeps that case.  Tiles go to blocks round-robin; the waits are bounded.
template <int KIND>
struct TmaTile {
  static constexpr int kStages = KIND == DUAL_SWIGLU_GRAD ? 2 : 3;
  static constexpr uint32_t kInBytes = uint32_t(kTileRows) * kTileCols * 2;   // the 128 x 128 tile
  static constexpr uint32_t kDhBytes = KIND == DUAL_SWIGLU_GRAD ? uint32_t(kTileRows) * kTileCols : 0;
  static constexpr uint32_t kStageBytes = kInBytes + kDhBytes;
  static constexpr size_t kSmemBytes = size_t(kStages) * kStageBytes;
  static constexpr int kColsPerTile = KIND == DUAL_SWIGLU_GRAD ? kTileCols / 2 : kTileCols;
};

struct DualTmaArgs {
  DualArgs a;
  int ncx;     // column tiles
  int ntiles;  // column tiles x row tiles
  int* err;
  uint64_t timeout_ns;
};

constexpr int kQThreads = 256;

template <int KIND>
__global__ void __launch_bounds__(kQThreads, 2)
    quant_dual_tma_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tm_dh,
                          DualTmaArgs p) {
  using T = TmaTile<KIND>;
  constexpr int R = kTileRows, CW = kTileCols / 2, S = T::kStages;
  extern __shared__ __align__(128) uint8_t qsm[];
  __shared__ uint64_t full[S];
  __shared__ int abort_flag;
  __shared__ __align__(4) uint8_t col_scales[kTileCols][R / 32];
  const int t = threadIdx.x;
  const DualArgs& a = p.a;
  const int grid = int(gridDim.x), b = int(blockIdx.x);
  const int my = p.ntiles > b ? (p.ntiles - b + grid - 1) / grid : 0;
  auto tile_of = [&](int slot) { return reinterpret_cast<uint32_t(*)[CW]>(qsm + size_t(slot) * T::kStageBytes); };
  auto dh_of = [&](int slot) {
    return reinterpret_cast<const uint32_t(*)[CW / 2]>(qsm + size_t(slot) * T::kStageBytes + T::kInBytes);
  };
  if (t == 0) {
    for (int i = 0; i < S; ++i) mbar_init(smem_u32(&full[i]), 1);
    abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm);
    if (KIND == DUAL_SWIGLU_GRAD) tma_prefetch_desc(&tm_dh);
  }
  __syncthreads();
  WaitCtl wc{&abort_flag, p.err, p.timeout_ns, 0u};
  auto issue = [&](int j) {  // tile j of this block into slot j % S
    const int tt = b + j * grid;
    const int x = (tt % p.ncx) * T::kColsPerTile, y = (tt / p.ncx) * R;
    const uint32_t bar = smem_u32(&full[j % S]);
    const uint32_t dst = smem_u32(qsm + size_t(j % S) * T::kStageBytes);
    mbar_arrive_expect_tx(bar, T::kStageBytes);
    if (KIND == DUAL_SWIGLU_GRAD) {
      tma_load_3d(dst, &tm, x, 0, y, bar);                    // g and u: [128 rows][2][64]
      tma_load_2d(dst + T::kInBytes, &tm_dh, x, y, bar);      // dh: [128 rows][64]
    } else {
      tma_load_2d(dst, &tm, x, y, bar);
    }
  };
  if (t == 0)
    for (int j = 0; j < S && j < my; ++j) issue(j);
  int i = 0;
  for (; i < my; ++i) {
    const int tt = b + i * grid;
    const int64_t r0 = int64_t(tt / p.ncx) * R, c0 = int64_t(tt % p.ncx) * T::kColsPerTile;
    const bool ok = mbar_wait(smem_u32(&full[i % S]), uint32_t(i / S) & 1u, wc);
    if (__syncthreads_or(!ok)) break;
    uint32_t(*tile)[CW] = tile_of(i % S);
    if (KIND == DUAL_SWIGLU_GRAD) {  // g, u -> dg, du in place (a warp per tile row per step)
      const uint32_t(*dh)[CW / 2] = dh_of(i % S);
#pragma unroll 4
      for (int k = t; k < R * (CW / 2); k += kQThreads) {
        const int r = k / (CW / 2), w = k % (CW / 2);
        uint32_t dg, du;
        swiglu_grad_word(tile[r][w], tile[r][CW / 2 + w], dh[r][w], dg, du);
        tile[r][w] = dg;
        tile[r][CW / 2 + w] = du;
      }
      __syncthreads();
    }
    dual_column_pass<KIND, kQThreads>(a, tile, col_scales, r0, c0, t);
    __syncthreads();
    dual_store_col_scales<KIND>(a, col_scales, r0, c0, t);
    __syncthreads();  // the slot and col_scales are free again
    if (t == 0 && i + S < my) issue(i + S);
  }
  if (i < my && t == 0) {  // gave up: let the loads still in flight land before the block exits
    for (int j = i; j < my && j < i + S; ++j)
      mbar_drain(smem_u32(&full[j % S]), uint32_t(j / S) & 1u, 20000000ull);
  }
}

// Tensor maps (no swizzle, out-of-range elements read as zero).  Plain: bf16
// [rows, cols] with 128 x 128 boxes.  SwiGLU gradient: gu [rows, 2, inter]
// with {64, 2, 128} boxes and dh [rows, inter] with 64 x 128 boxes.
static bool make_quant_tmaps(int kind, const DualArgs& a, CUtensorMap* tm, CUtensorMap* tm_dh) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint32_t estr[3] = {1, 1, 1};
  if (kind == DUAL_PLAIN) {
    cuuint64_t dims[2] = {cuuint64_t(a.cols), cuuint64_t(a.rows)};
    cuuint64_t strides[1] = {cuuint64_t(a.cols) * 2};
    cuuint32_t box[2] = {cuuint32_t(kTileCols), cuuint32_t(kTileRows)};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint4*>(a.a), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  cuuint64_t dims3[3] = {cuuint64_t(a.inter), 2, cuuint64_t(a.rows)};
  cuuint64_t strides3[2] = {cuuint64_t(a.inter) * 2, cuuint64_t(a.inter) * 4};
  cuuint32_t box3[3] = {cuuint32_t(kTileCols / 2), 2, cuuint32_t(kTileRows)};
  if (enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint4*>(a.a), dims3, strides3, box3, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cuuint64_t dims2[2] = {cuuint64_t(a.inter), cuuint64_t(a.rows)};
  cuuint64_t strides2[1] = {cuuint64_t(a.inter) * 2};
  cuuint32_t box2[2] = {cuuint32_t(kTileCols / 2), cuuint32_t(kTileRows)};
  return enc(tm_dh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint4*>(a.dh), dims2, strides2, box2, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KIND>
static int quant_tma_blocks_per_sm() {  // per device and kind: shared-memory attribute set once
  static std::mutex mu;
  static int ready[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lk(mu);
  if (ready[dev] == 0) {
    ready[dev] = -1;
    const size_t smem = TmaTile<KIND>::kSmemBytes;
    if (cudaFuncSetAttribute(quant_dual_tma_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(smem)) == cudaSuccess) {
      int n = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, quant_dual_tma_kernel<KIND>, kQThreads, smem) ==
              cudaSuccess && n > 0)
        ready[dev] = n;
    }
  }
  return ready[dev] > 0 ? ready[dev] : 0;
}

// Column-wise-only plain and SwiGLU-gradient encodes through the TMA kernel;
// returns false (nothing launched) when that path does not apply.
template <int KIND>
static bool launch_dual_tma(const DualArgs& a, void* stream, int* status) {
  if constexpr (KIND == DUAL_SWIGLU) {
    return false;
  } else {
    if (a.q != nullptr || a.row0 != 0 || a.row_end != a.rows) return false;
    if (KIND == DUAL_SWIGLU_GRAD && (a.inter % 32 != 0 || !aligned16(a.dh))) return false;
    const int per_sm = quant_tma_blocks_per_sm<KIND>();
    const int64_t span = KIND == DUAL_SWIGLU_GRAD ? a.inter : a.cols;
    const int64_t ncx = (span + TmaTile<KIND>::kColsPerTile - 1) / TmaTile<KIND>::kColsPerTile;
    const int64_t nry = (a.rows + kTileRows - 1) / kTileRows;
    CUtensorMap tm, tm_dh;
    int* err = device_error_word();
    if (per_sm <= 0 || !err || ncx * nry > INT32_MAX) return false;
    if (!make_quant_tmaps(KIND, a, &tm, &tm_dh)) return false;
    if (KIND == DUAL_PLAIN) tm_dh = tm;  // unused
    DualTmaArgs p{a, int(ncx), int(ncx * nry), err, kWaitLimitNs};
    const int64_t grid = std::min<int64_t>(ncx * nry, int64_t(num_sms()) * per_sm);
    quant_dual_tma_kernel<KIND><<<unsigned(grid), kQThreads, TmaTile<KIND>::kSmemBytes,
                                  (cudaStream_t)stream>>>(tm, tm_dh, p);
    *status = cuda_status(cudaGetLastError());
    return true;
  }
}

// Encodes rows [row0, row_end) of the tensor (row_end < 0: all rows); the
// outputs keep the layout of the whole tensor, so a split encode (rows of some
// groups now, the rest later) writes the same bytes as one over all rows.
template <int KIND>
static int launch_dual(DualArgs a, void* stream, int64_t row0 = 0, int64_t row_end = -1) {
  if (a.rows < 0 || a.cols < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (row_end < 0) row_end = a.rows;
  if (row0 < 0 || row0 > row_end || row_end > a.rows) return MXG_ERR_INVALID_ARGUMENT;
  if (row0 % 32 != 0 || row_end % 32 != 0) return MXG_ERR_BAD_SHAPE;
  a.row0 = row0;
  a.row_end = row_end;
  if ((a.q == nullptr) != (a.s == nullptr) || (a.qt == nullptr) != (a.st == nullptr) ||
      (a.q == nullptr && a.qt == nullptr))
    return MXG_ERR_INVALID_ARGUMENT;
  if (a.rows % 32 != 0 || a.cols % 32 != 0) return MXG_ERR_BAD_SHAPE;
  if ((a.q && !aligned16(a.q)) || (a.qt && !aligned16(a.qt))) return MXG_ERR_MISALIGNED;
  if (row_end == row0 || a.cols == 0) return MXG_OK;
  if ((a.rows + kTileRows - 1) / kTileRows > 65535) return MXG_ERR_BAD_SHAPE;
  int e = check_device();
  if (e) return e;
  int tma_status = MXG_OK;
  if (launch_dual_tma<KIND>(a, stream, &tma_status)) return tma_status;
  const int64_t span = KIND == DUAL_SWIGLU_GRAD ? a.inter : a.cols;
  const int64_t per = KIND == DUAL_SWIGLU_GRAD ? kTileCols / 2 : kTileCols;
  dim3 grid(unsigned((span + per - 1) / per), unsigned((row_end - row0 + kTileRows - 1) / kTileRows));
  quant_dual_kernel<KIND><<<grid, 256, 0, (cudaStream_t)stream>>>(a);
  return cuda_status(cudaGetLastError());
}

// ---------------------------------------------------------------- transpose
// dst [cols, rows] = src [rows, cols]^T for bytes, 64x64 tiles through smem.
__global__ void __launch_bounds__(256) transpose_u8_kernel(const uint8_t* __restrict__ src,
                                                           int64_t rows, int64_t cols,
                                                           uint8_t* __restrict__ dst) {
  __shared__ uint8_t tile[64][65];
  const int64_t r0 = int64_t(blockIdx.y) * 64, c0 = int64_t(blockIdx.x) * 64;
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int r = i / 64, c = i % 64;
    if (r0 + r < rows && c0 + c < cols) tile[r][c] = src[(r0 + r) * cols + c0 + c];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int c = i / 64, r = i % 64;
    if (r0 + r < rows && c0 + c < cols) dst[(c0 + c) * rows + r0 + r] = tile[r][c];
  }
}

}  // namespace mxg

using namespace mxg;

extern "C" int mxg_quantize_rowwise(const void* x_bf16, int64_t rows, int64_t cols, void* q_e4m3,
                                    void* scales_e8m0, void* stream) {
  if (!x_bf16 || !q_e4m3 || !scales_e8m0) return MXG_ERR_INVALID_ARGUMENT;
  if (rows < 0 || cols < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (cols % 32 != 0) return MXG_ERR_BAD_SHAPE;
  if (!aligned16(x_bf16) || !aligned16(q_e4m3)) return MXG_ERR_MISALIGNED;
  if (rows == 0 || cols == 0) return MXG_OK;
  int st = check_device();
  if (st) return st;
  const int64_t nchunks = rows * cols / 8;
  const int threads = 256;
  int64_t want = (nchunks + threads * kRowUnroll - 1) / (threads * kRowUnroll);
  const int64_t cap = int64_t(num_sms()) * 8;
  const int blocks = int(want < cap ? (want < 1 ? 1 : want) : cap);
  quant_rowwise_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint4*>(x_bf16), reinterpret_cast<uint2*>(q_e4m3),
      reinterpret_cast<uint8_t*>(scales_e8m0), nchunks);
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_quantize_colwise(const void* x_bf16, int64_t rows, int64_t cols, void* qt_e4m3,
                                    void* scales_t_e8m0, void* stream) {
  if (!x_bf16 || !qt_e4m3 || !scales_t_e8m0) return MXG_ERR_INVALID_ARGUMENT;
  if (rows < 0 || cols < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (rows % 32 != 0 || cols % 2 != 0) return MXG_ERR_BAD_SHAPE;
  if (!aligned16(x_bf16) || !aligned16(qt_e4m3)) return MXG_ERR_MISALIGNED;
  if (rows == 0 || cols == 0) return MXG_OK;
  if (rows / 32 > 65535) return MXG_ERR_BAD_SHAPE;
  if (cols % 32 == 0) {  // the tiled kernel writes whole 32-byte sectors of qt: faster
    DualArgs a{reinterpret_cast<const uint4*>(x_bf16), nullptr, rows, cols, 0, nullptr, nullptr,
               reinterpret_cast<uint8_t*>(qt_e4m3), reinterpret_cast<uint8_t*>(scales_t_e8m0)};
    return launch_dual<DUAL_PLAIN>(a, stream);
  }
  int st = check_device();
  if (st) return st;
  dim3 grid(unsigned((cols + kColPerBlock - 1) / kColPerBlock), unsigned(rows / 32));
  quant_colwise_kernel<<<grid, kColThreads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint32_t*>(x_bf16), rows, cols, reinterpret_cast<uint8_t*>(qt_e4m3),
      reinterpret_cast<uint8_t*>(scales_t_e8m0));
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_transpose_u8(const void* src, int64_t rows, int64_t cols, void* dst,
                                void* stream) {
  if (!src || !dst || rows < 0 || cols < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (rows == 0 || cols == 0) return MXG_OK;
  if ((rows + 63) / 64 > 65535) return MXG_ERR_BAD_SHAPE;
  int st = check_device();
  if (st) return st;
  dim3 grid(unsigned((cols + 63) / 64), unsigned((rows + 63) / 64));
  transpose_u8_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint8_t*>(src), rows, cols, reinterpret_cast<uint8_t*>(dst));
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_quantize_dual(const void* x_bf16, int64_t rows, int64_t cols, void* q_e4m3,
                                 void* scales_e8m0, void* qt_e4m3, void* scales_t_e8m0,
                                 void* stream) {
  if (!x_bf16) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(x_bf16)) return MXG_ERR_MISALIGNED;
  DualArgs a{reinterpret_cast<const uint4*>(x_bf16), nullptr, rows, cols, 0,
             reinterpret_cast<uint8_t*>(q_e4m3), reinterpret_cast<uint8_t*>(scales_e8m0),
             reinterpret_cast<uint8_t*>(qt_e4m3), reinterpret_cast<uint8_t*>(scales_t_e8m0)};
  return launch_dual<DUAL_PLAIN>(a, stream);
}

extern "C" int mxg_quantize_dual_rows(const void* x_bf16, int64_t rows, int64_t cols, int64_t row_begin,
                                      int64_t row_end, void* q_e4m3, void* scales_e8m0, void* qt_e4m3,
                                      void* scales_t_e8m0, void* stream) {
  if (!x_bf16 || row_end < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(x_bf16)) return MXG_ERR_MISALIGNED;
  DualArgs a{reinterpret_cast<const uint4*>(x_bf16), nullptr, rows, cols, 0,
             reinterpret_cast<uint8_t*>(q_e4m3), reinterpret_cast<uint8_t*>(scales_e8m0),
             reinterpret_cast<uint8_t*>(qt_e4m3), reinterpret_cast<uint8_t*>(scales_t_e8m0)};
  return launch_dual<DUAL_PLAIN>(a, stream, row_begin, row_end);
}

extern "C" int mxg_swiglu_quantize(const void* gu_bf16, int64_t rows, int64_t inter, void* q_e4m3,
                                   void* scales_e8m0, void* qt_e4m3, void* scales_t_e8m0,
                                   void* stream) {
  if (!gu_bf16) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(gu_bf16)) return MXG_ERR_MISALIGNED;
  DualArgs a{reinterpret_cast<const uint4*>(gu_bf16), nullptr, rows, inter, inter,
             reinterpret_cast<uint8_t*>(q_e4m3), reinterpret_cast<uint8_t*>(scales_e8m0),
             reinterpret_cast<uint8_t*>(qt_e4m3), reinterpret_cast<uint8_t*>(scales_t_e8m0)};
  return launch_dual<DUAL_SWIGLU>(a, stream);
}

extern "C" int mxg_swiglu_bwd_quantize(const void* gu_bf16, const void* dh_bf16, int64_t rows,
                                       int64_t inter, void* q_e4m3, void* scales_e8m0,
                                       void* qt_e4m3, void* scales_t_e8m0, void* stream) {
  if (!gu_bf16 || !dh_bf16) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(gu_bf16) || !aligned16(dh_bf16)) return MXG_ERR_MISALIGNED;
  DualArgs a{reinterpret_cast<const uint4*>(gu_bf16), reinterpret_cast<const uint4*>(dh_bf16),
             rows, 2 * inter, inter, reinterpret_cast<uint8_t*>(q_e4m3),
             reinterpret_cast<uint8_t*>(scales_e8m0), reinterpret_cast<uint8_t*>(qt_e4m3),
             reinterpret_cast<uint8_t*>(scales_t_e8m0)};
  return launch_dual<DUAL_SWIGLU_GRAD>(a, stream);
}
