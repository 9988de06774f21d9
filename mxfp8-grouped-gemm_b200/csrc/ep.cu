// Expert-parallel token routing kernels for sm_100a (HBM-bound row moves and
// small integer bookkeeping).  Experts are sharded evenly over the ranks:
// global expert e lives on rank e / E_local as local expert e % E_local.
//
//   route:    stable counting sort of the (token, k) routing slots by expert
//             slot (the expert id through an optional placement map) ->
//             per-slot counts, send order (token row of each send position)
//             and the inverse (send position of each slot).
//   gather:   dst[i] = src[idx[i]] (idx < 0 -> zero row), 16-byte vectors.
//   regroup:  rows received from all ranks (ordered by source rank, then
//             local expert) -> expert-major groups padded to `pad` rows, and
//             the inverse map used to send results back.
//   combine:  out[t] = sum_j w[t, j] * rows[inv[t * k + j]] (fp32 sum, bf16 out).
//   swiglu:   h = silu(g) * u for gu = [g | u] rows (bf16 in/out), and its
//             backward dgu = [dg | du] from dh.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "mxg.h"
#include "mxg_device.cuh"
#include "mxg_internal.h"

namespace mxg {

constexpr int kRouteBlock = 1024;  // slots per block in the routing sort

// Per-block expert histograms (stability comes from block order).
// Expert id of slot i mapped through the placement (slot_of_expert may be
// null = identity); -1 for an id outside [0, num_experts).
__device__ __forceinline__ int routed_slot(const int32_t* __restrict__ ids,
                                           const int32_t* __restrict__ slot_of_expert, int64_t i,
                                           int num_experts) {
  const int e = ids[i];
  if (e < 0 || e >= num_experts) return -1;
  return slot_of_expert ? slot_of_expert[e] : e;
}

__global__ void __launch_bounds__(kRouteBlock) route_hist_kernel(const int32_t* __restrict__ ids,
                                                                 const int32_t* __restrict__ slot_of_expert,
                                                                 int64_t n_slots, int num_experts,
                                                                 int32_t* __restrict__ block_hist,
                                                                 int* err) {
  extern __shared__ int32_t h[];
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int64_t i = int64_t(blockIdx.x) * kRouteBlock + threadIdx.x;
  if (i < n_slots) {
    const int e = routed_slot(ids, slot_of_expert, i, num_experts);
    if (e >= 0 && e < num_experts) atomicAdd(&h[e], 1);
    else atomicCAS(err, 0, MXG_ERR_INVALID_ARGUMENT);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x)
    block_hist[int64_t(blockIdx.x) * num_experts + e] = h[e];
}

// block_base[b][e] = sum over experts e' < e of all slots + slots of expert e
// in blocks b' < b; counts[e] = total slots of expert e.  One thread per expert.
__global__ void route_scan_kernel(const int32_t* __restrict__ block_hist, int nblocks,
                                  int num_experts, int32_t* __restrict__ block_base,
                                  int32_t* __restrict__ counts) {
  __shared__ int32_t tot[MXG_EP_MAX_EXPERTS + 1];
  const int e = threadIdx.x;
  int32_t sum = 0;
  if (e < num_experts)
    for (int b = 0; b < nblocks; ++b) sum += block_hist[int64_t(b) * num_experts + e];
  if (e < num_experts) tot[e] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {  // exclusive scan over experts (<= MXG_EP_MAX_EXPERTS entries)
    int32_t run = 0;
    for (int x = 0; x < num_experts; ++x) {
      const int32_t v = tot[x];
      tot[x] = run;
      run += v;
    }
  }
  __syncthreads();
  if (e < num_experts) {
    int32_t run = tot[e];
    counts[e] = sum;
    for (int b = 0; b < nblocks; ++b) {
      block_base[int64_t(b) * num_experts + e] = run;
      run += block_hist[int64_t(b) * num_experts + e];
    }
  }
}

// Stable scatter: within a block, slots keep their order per expert (warp
// match + ballot ranks, then a prefix over the block's warps).
__global__ void __launch_bounds__(kRouteBlock) route_scatter_kernel(
    const int32_t* __restrict__ ids, const int32_t* __restrict__ slot_of_expert, int64_t n_slots,
    int topk, int num_experts,
    const int32_t* __restrict__ block_base, int32_t* __restrict__ send_rows,
    int32_t* __restrict__ slot_pos) {
  extern __shared__ int32_t sm[];  // [32 warps][num_experts] counts, then prefix in place
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int x = threadIdx.x; x < 32 * num_experts; x += blockDim.x) sm[x] = 0;
  __syncthreads();
  const int64_t i = int64_t(blockIdx.x) * kRouteBlock + threadIdx.x;
  int e = -1;
  if (i < n_slots) {
    e = routed_slot(ids, slot_of_expert, i, num_experts);
    if (e >= num_experts) e = -1;
  }
  const unsigned same = __match_any_sync(0xffffffffu, e);
  const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
  if (e >= 0 && rank_in_warp == 0) sm[warp * num_experts + e] = __popc(same);
  __syncthreads();
  for (int x = threadIdx.x; x < num_experts; x += blockDim.x) {  // prefix over warps
    int32_t run = 0;
    for (int w = 0; w < 32; ++w) {
      const int32_t v = sm[w * num_experts + x];
      sm[w * num_experts + x] = run;
      run += v;
    }
  }
  __syncthreads();
  if (e >= 0) {
    const int32_t pos = block_base[int64_t(blockIdx.x) * num_experts + e] +
                        sm[warp * num_experts + e] + rank_in_warp;
    send_rows[pos] = int32_t(i / topk);
    slot_pos[i] = pos;
  } else if (i < n_slots) {
    slot_pos[i] = -1;
  }
}

// dst[i] = src[idx[i]] for 16-byte-multiple rows; idx < 0 or >= src_rows -> zeros.
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint4* __restrict__ src,
                                                          int64_t src_rows, int64_t row_vecs,
                                                          const int32_t* __restrict__ idx,
                                                          int64_t n, uint4* __restrict__ dst) {
  const int64_t total = n * row_vecs;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < total; v += stride) {
    const int64_t r = v / row_vecs, c = v - r * row_vecs;
    const int32_t s = idx[r];
    uint4 val = make_uint4(0, 0, 0, 0);
    if (s >= 0 && s < src_rows) val = __ldg(src + int64_t(s) * row_vecs + c);
    dst[v] = val;
  }
}

// One block per local expert: padded group start, then for every source rank
// the received rows of (rank, expert) in order, then zero padding.
__global__ void regroup_kernel(const int32_t* __restrict__ recv_counts, int world, int e_local,
                               int pad, int32_t* __restrict__ idx, int32_t* __restrict__ back,
                               int32_t* __restrict__ group_rows) {
  const int le = blockIdx.x;
  __shared__ int64_t start_s, src_off_s[MXG_EP_MAX_RANKS];
  __shared__ int32_t rows_s;
  if (threadIdx.x == 0) {
    int64_t start = 0;
    for (int x = 0; x < le; ++x) {
      int64_t c = 0;
      for (int r = 0; r < world; ++r) c += recv_counts[r * e_local + x];
      start += (c + pad - 1) / pad * pad;
    }
    start_s = start;
    int32_t rows = 0;
    int64_t before_rank = 0;  // received rows of ranks < r (all their experts)
    for (int r = 0; r < world; ++r) {
      int64_t within = 0;
      for (int x = 0; x < le; ++x) within += recv_counts[r * e_local + x];
      src_off_s[r] = before_rank + within;
      for (int x = 0; x < e_local; ++x) before_rank += recv_counts[r * e_local + x];
      rows += recv_counts[r * e_local + le];
    }
    rows_s = rows;
    group_rows[le] = (rows + pad - 1) / pad * pad;
  }
  __syncthreads();
  const int64_t start = start_s;
  const int32_t padded = (rows_s + pad - 1) / pad * pad;
  int64_t base = 0;
  for (int r = 0; r < world; ++r) {
    const int32_t c = recv_counts[r * e_local + le];
    for (int j = threadIdx.x; j < c; j += blockDim.x) {
      const int64_t src = src_off_s[r] + j;
      idx[start + base + j] = int32_t(src);
      back[src] = int32_t(start + base + j);
    }
    base += c;
  }
  for (int j = int(base) + threadIdx.x; j < padded; j += blockDim.x) idx[start + j] = -1;
}

// out[t] = sum_j w[t, j] * rows[inv[t * k + j]]; one block of 128 threads per
// token, 8 bf16 (16 bytes) per thread per step.
__global__ void __launch_bounds__(128) combine_kernel(const __nv_bfloat16* __restrict__ rows,
                                                      const int32_t* __restrict__ inv,
                                                      const float* __restrict__ w, int topk,
                                                      int64_t hidden,
                                                      __nv_bfloat16* __restrict__ out) {
  const int64_t t = blockIdx.x;
  for (int64_t c = int64_t(threadIdx.x) * 8; c < hidden; c += int64_t(blockDim.x) * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < topk; ++j) {
      const int32_t p = inv[t * topk + j];
      if (p < 0) continue;
      const float wj = w ? w[t * topk + j] : 1.0f;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(rows + int64_t(p) * hidden + c));
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h2[q]);
        acc[2 * q] += wj * f.x;
        acc[2 * q + 1] += wj * f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) o2[q] = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
    *reinterpret_cast<uint4*>(out + t * hidden + c) = o;
  }
}

// h[r, c] = silu(g[r, c]) * u[r, c] with gu[r] = [g (I) | u (I)]; 8 elements per thread.
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ gu,
                                                     int64_t rows, int64_t inter,
                                                     __nv_bfloat16* __restrict__ h) {
  const int64_t vecs_per_row = inter / 8;
  const int64_t total = rows * vecs_per_row;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < total; v += stride) {
    const int64_t r = v / vecs_per_row, c = (v - r * vecs_per_row) * 8;
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter + c));
    const uint4 uv = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter + inter + c));
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 g = __bfloat1622float2(g2[q]);
      const float2 u = __bfloat1622float2(u2[q]);
      o2[q] = __floats2bfloat162_rn(silu_mul(g.x, u.x), silu_mul(g.y, u.y));
    }
    *reinterpret_cast<uint4*>(h + r * inter + c) = o;
  }
}

// Backward of h = silu(g) * u: dg = dh * u * s * (1 + g * (1 - s)), du = dh *
// silu(g) with s = sigmoid(g); fp32 math, bf16 in/out, 8 elements per thread.
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                                         const __nv_bfloat16* __restrict__ dh,
                                                         int64_t rows, int64_t inter,
                                                         __nv_bfloat16* __restrict__ dgu) {
  const int64_t vecs_per_row = inter / 8;
  const int64_t total = rows * vecs_per_row;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < total; v += stride) {
    const int64_t r = v / vecs_per_row, c = (v - r * vecs_per_row) * 8;
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter + c));
    const uint4 uv = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter + inter + c));
    const uint4 dv = __ldg(reinterpret_cast<const uint4*>(dh + r * inter + c));
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
    const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dv);
    uint4 og, ou;
    __nv_bfloat162* og2 = reinterpret_cast<__nv_bfloat162*>(&og);
    __nv_bfloat162* ou2 = reinterpret_cast<__nv_bfloat162*>(&ou);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 g = __bfloat1622float2(g2[q]);
      const float2 u = __bfloat1622float2(u2[q]);
      const float2 d = __bfloat1622float2(d2[q]);
      float dgx, dux, dgy, duy;
      silu_mul_grad(g.x, u.x, d.x, dgx, dux);
      silu_mul_grad(g.y, u.y, d.y, dgy, duy);
      og2[q] = __floats2bfloat162_rn(dgx, dgy);
      ou2[q] = __floats2bfloat162_rn(dux, duy);
    }
    *reinterpret_cast<uint4*>(dgu + r * 2 * inter + c) = og;
    *reinterpret_cast<uint4*>(dgu + r * 2 * inter + inter + c) = ou;
  }
}

}  // namespace mxg

using namespace mxg;

extern "C" size_t mxg_ep_route_workspace_size(int64_t n_slots, int num_experts) {
  if (n_slots < 0 || num_experts < 1) return 0;
  const int64_t nb = (n_slots + kRouteBlock - 1) / kRouteBlock;
  return size_t(2 * nb * num_experts) * sizeof(int32_t) + 256;
}

extern "C" int mxg_ep_route(const int32_t* expert_ids, const int32_t* slot_of_expert,
                            int64_t n_slots, int topk, int num_experts, int32_t* counts,
                            int32_t* send_rows, int32_t* slot_pos, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (n_slots < 0 || topk < 1 || num_experts < 1 || num_experts > MXG_EP_MAX_EXPERTS)
    return MXG_ERR_INVALID_ARGUMENT;
  // the per-slot arrays may be null when there are no slots
  if (!counts || !workspace || (n_slots > 0 && (!expert_ids || !send_rows || !slot_pos)))
    return MXG_ERR_INVALID_ARGUMENT;
  if (n_slots % topk != 0 || n_slots > INT32_MAX) return MXG_ERR_BAD_SHAPE;
  if (workspace_bytes < mxg_ep_route_workspace_size(n_slots, num_experts))
    return MXG_ERR_WORKSPACE_TOO_SMALL;
  int st = check_device();
  if (st) return st;
  int* err = device_error_word();
  if (!err) return MXG_ERR_CUDA;
  cudaStream_t s = (cudaStream_t)stream;
  if (n_slots == 0) return cuda_status(cudaMemsetAsync(counts, 0, sizeof(int32_t) * num_experts, s));
  const int nb = int((n_slots + kRouteBlock - 1) / kRouteBlock);
  int32_t* hist = reinterpret_cast<int32_t*>(workspace);
  int32_t* base = hist + int64_t(nb) * num_experts;
  route_hist_kernel<<<nb, kRouteBlock, sizeof(int32_t) * num_experts, s>>>(
      expert_ids, slot_of_expert, n_slots, num_experts, hist, err);
  route_scan_kernel<<<1, MXG_EP_MAX_EXPERTS, 0, s>>>(hist, nb, num_experts, base, counts);
  route_scatter_kernel<<<nb, kRouteBlock, sizeof(int32_t) * 32 * num_experts, s>>>(
      expert_ids, slot_of_expert, n_slots, topk, num_experts, base, send_rows, slot_pos);
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_gather_rows(const void* src, int64_t src_rows, int64_t row_bytes,
                               const int32_t* idx, int64_t n, void* dst, void* stream) {
  if (n < 0 || src_rows < 0 || row_bytes < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (row_bytes % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (n == 0 || row_bytes == 0) return MXG_OK;
  if ((!src && src_rows > 0) || !idx || !dst) return MXG_ERR_INVALID_ARGUMENT;
  if ((src && !aligned16(src)) || !aligned16(dst)) return MXG_ERR_MISALIGNED;
  int st = check_device();
  if (st) return st;
  const int64_t vecs = n * (row_bytes / 16);
  const int64_t want = (vecs + 255) / 256;
  const int blocks = int(std::min<int64_t>(want, int64_t(num_sms()) * 16));
  gather_rows_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint4*>(src), src_rows, row_bytes / 16, idx, n,
      reinterpret_cast<uint4*>(dst));
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_ep_regroup(const int32_t* recv_counts, int world, int e_local, int pad,
                              int32_t* idx, int32_t* back, int32_t* group_rows, void* stream) {
  if (!recv_counts || !idx || !back || !group_rows) return MXG_ERR_INVALID_ARGUMENT;
  if (world < 1 || world > MXG_EP_MAX_RANKS || e_local < 1 || e_local > MXG_MAX_GROUPS || pad < 1)
    return MXG_ERR_INVALID_ARGUMENT;
  int st = check_device();
  if (st) return st;
  regroup_kernel<<<e_local, 256, 0, (cudaStream_t)stream>>>(recv_counts, world, e_local, pad, idx,
                                                            back, group_rows);
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_ep_combine(const void* rows, const int32_t* slot_pos, const float* weights,
                              int64_t n_tokens, int topk, int64_t hidden, void* out, void* stream) {
  if (n_tokens < 0 || topk < 1 || hidden < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (hidden % 8 != 0) return MXG_ERR_BAD_SHAPE;
  if (n_tokens == 0 || hidden == 0) return MXG_OK;
  if (!rows || !slot_pos || !out) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(rows) || !aligned16(out)) return MXG_ERR_MISALIGNED;
  if (n_tokens > INT32_MAX) return MXG_ERR_BAD_SHAPE;
  int st = check_device();
  if (st) return st;
  combine_kernel<<<unsigned(n_tokens), 128, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(rows), slot_pos, weights, topk, hidden,
      reinterpret_cast<__nv_bfloat16*>(out));
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_swiglu(const void* gu, int64_t rows, int64_t inter, void* h, void* stream) {
  if (rows < 0 || inter < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (inter % 8 != 0) return MXG_ERR_BAD_SHAPE;
  if (rows == 0 || inter == 0) return MXG_OK;
  if (!gu || !h) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(gu) || !aligned16(h)) return MXG_ERR_MISALIGNED;
  int st = check_device();
  if (st) return st;
  const int64_t vecs = rows * inter / 8;
  const int blocks = int(std::min<int64_t>((vecs + 255) / 256, int64_t(num_sms()) * 16));
  swiglu_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu), rows, inter, reinterpret_cast<__nv_bfloat16*>(h));
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_swiglu_bwd(const void* gu, const void* dh, int64_t rows, int64_t inter, void* dgu,
                              void* stream) {
  if (rows < 0 || inter < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (inter % 8 != 0) return MXG_ERR_BAD_SHAPE;
  if (rows == 0 || inter == 0) return MXG_OK;
  if (!gu || !dh || !dgu) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(gu) || !aligned16(dh) || !aligned16(dgu)) return MXG_ERR_MISALIGNED;
  int st = check_device();
  if (st) return st;
  const int64_t vecs = rows * inter / 8;
  const int blocks = int(std::min<int64_t>((vecs + 255) / 256, int64_t(num_sms()) * 16));
  swiglu_bwd_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<const __nv_bfloat16*>(dh), rows,
      inter, reinterpret_cast<__nv_bfloat16*>(dgu));
  return cuda_status(cudaGetLastError());
}
