// Device-side arithmetic shared by the library's kernels: the MXFP8 element
// and scale rules (RCEIL E8M0, e4m3 RNE with saturation) and the expert FFN
// activation (SwiGLU) with its gradient.  Kernels that must agree bit for bit
// (a quantiser and its fused variants, swiglu and its fused variants) all
// call these.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>

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

// cvt_e4m3x2(lo * f, hi * f), the two products from one packed f32x2
// multiply (each lane rounds exactly as a scalar multiply: the same bits in
// half the multiply instructions).
__device__ __forceinline__ uint32_t cvt_scaled_e4m3x2(float lo, float hi, float f) {
  uint64_t ab, ff, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ab) : "f"(lo), "f"(hi));
  asm("mov.b64 %0, {%1, %1};" : "=l"(ff) : "f"(f));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(ab), "l"(ff));
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
  return cvt_e4m3x2(a, b);
}

__device__ __forceinline__ uint32_t amax2(uint32_t w) {
  const uint32_t a = w & 0x7FFFu, b = (w >> 16) & 0x7FFFu;
  return a > b ? a : b;
}

// |x| bit patterns of both bf16 halves of a word, maxed per half with
// another such pair (one SIMD max per two elements).  The bit patterns of
// non-negative bf16 values order like the values; NaN patterns order above
// +Inf, so a block holding a NaN keeps a NaN amax.
__device__ __forceinline__ uint32_t abs2(uint32_t w) { return w & 0x7FFF7FFFu; }
__device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) { return __vmaxu2(a, b); }

// amax bit pattern of the 8 bf16 values of a 16-byte chunk, still as two halves
__device__ __forceinline__ uint32_t amax_chunk2(uint4 v) {
  return max2(max2(abs2(v.x), abs2(v.y)), max2(abs2(v.z), abs2(v.w)));
}
__device__ __forceinline__ uint32_t halves_max(uint32_t m2) {
  const uint32_t a = m2 & 0xFFFFu, b = m2 >> 16;
  return a > b ? a : b;
}

// NaN-carrying block (scale byte 0xFF): patch the NaN lanes so their codes
// keep the input's sign, as torch's float8_e4m3fn cast does.
__device__ __forceinline__ uint32_t fix_nan_byte(uint32_t code, uint32_t bf16bits) {
  if ((bf16bits & 0x7FFFu) > 0x7F80u) return 0x7Fu | ((bf16bits >> 8) & 0x80u);
  return code;
}

// SwiGLU: h = silu(g) * u = g * sigmoid(g) * u (fp32).
// silu(g) * u.  The divisions use the fast-divide intrinsic (about 2 ulp,
// and 0 once 1 + e^-g passes 2^126, i.e. g < -87): the SwiGLU encoders are
// bound by instruction issue at the power-capped clock, and an IEEE division
// costs several times the rest of the element's work; their results are
// rounded to bf16 (or encoded to e4m3) right after.
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// Gradient of silu_mul w.r.t. g and u for upstream gradient d.
__device__ __forceinline__ void silu_mul_grad(float g, float u, float d, float& dg, float& du) {
  const float sg = __fdividef(1.0f, 1.0f + __expf(-g));
  dg = d * u * sg * (1.0f + g * (1.0f - sg));
  du = d * g * sg;
}

__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace mxg
