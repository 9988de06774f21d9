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

#include "mxg.h"
#include "mxg_internal.h"

namespace mxg {

__device__ __forceinline__ uint32_t rceil_byte(uint32_t amax_bits16) {
  if (amax_bits16 == 0) return 0u;
  if (amax_bits16 > 0x7F80u) return 255u;
  if (amax_bits16 == 0x7F80u) return 254u;
  const uint32_t f = amax_bits16 << 16;
  const int e = int(f >> 23) - 127 - 8 + ((f & 0x7FFFFFu) > 0x600000u ? 1 : 0);
  const int c = e < -127 ? -127 : (e > 127 ? 127 : e);
  return uint32_t(c + 127);
}

// Multiplier applied before the e4m3 cast: 1.0 for byte 0, else 2^(127-byte)
// built directly as an fp32 bit pattern (subnormal for bytes 254 and 255).
__device__ __forceinline__ float descale_of(uint32_t b) {
  if (b == 0u) return 1.0f;
  if (b <= 253u) return __uint_as_float((254u - b) << 23);
  return __uint_as_float(b == 254u ? 0x00400000u : 0x00200000u);
}

// Two fp32 values -> two e4m3 codes (low byte = first value), round to
// nearest even with saturation to +-448.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  __nv_fp8x2_storage_t s = __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
  return uint32_t(s);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ uint32_t amax2(uint32_t w) {
  const uint32_t a = w & 0x7FFFu, b = (w >> 16) & 0x7FFFu;
  return a > b ? a : b;
}

// NaN-carrying block (scale byte 0xFF): patch the NaN lanes so their codes
// keep the input's sign, as torch's float8_e4m3fn cast does.
__device__ __forceinline__ uint32_t fix_nan_byte(uint32_t code, uint32_t bf16bits) {
  if ((bf16bits & 0x7FFFu) > 0x7F80u) return 0x7Fu | ((bf16bits >> 8) & 0x80u);
  return code;
}

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
      uint32_t m = amax2(v[u].x);
      m = max(m, amax2(v[u].y));
      m = max(m, amax2(v[u].z));
      m = max(m, amax2(v[u].w));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
      const uint32_t b = rceil_byte(m);
      const float f = descale_of(b);
      uint32_t c0 = cvt_e4m3x2(bf16_lo(v[u].x) * f, bf16_hi(v[u].x) * f);
      uint32_t c1 = cvt_e4m3x2(bf16_lo(v[u].y) * f, bf16_hi(v[u].y) * f);
      uint32_t c2 = cvt_e4m3x2(bf16_lo(v[u].z) * f, bf16_hi(v[u].z) * f);
      uint32_t c3 = cvt_e4m3x2(bf16_lo(v[u].w) * f, bf16_hi(v[u].w) * f);
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
    uint32_t a01 = cvt_e4m3x2(bf16_lo(w[4 * j]) * f0, bf16_lo(w[4 * j + 1]) * f0);
    uint32_t a23 = cvt_e4m3x2(bf16_lo(w[4 * j + 2]) * f0, bf16_lo(w[4 * j + 3]) * f0);
    uint32_t b01 = cvt_e4m3x2(bf16_hi(w[4 * j]) * f1, bf16_hi(w[4 * j + 1]) * f1);
    uint32_t b23 = cvt_e4m3x2(bf16_hi(w[4 * j + 2]) * f1, bf16_hi(w[4 * j + 3]) * f1);
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
