// Expert-parallel dispatch and combine over NVLink peer memory (sm_100a).
//
// Every rank exposes receive buffers to the others through CUDA IPC.  A
// dispatch writes each routed token row straight into its final place in the
// owner's buffer -- the expert-major, 32-padded layout the grouped GEMMs read
// -- so there is no send-side gather, no all-to-all staging copy and no
// receive-side regroup.  The combine writes each result row back into the
// token's home rank at the row's send position.  These kernels only store
// (ordinary 16-byte stores to peer addresses); ordering across ranks is left
// to the caller, who runs a collective before (the count exchange: every
// receiver is done with the previous contents) and after (every writer is
// done) each exchange.  No kernel here waits on another rank.
//
// Layout of rank d's receive buffer (shared by every rank's plan):
//   local expert le of rank d occupies padded rows
//     [gstart_d(le), gstart_d(le) + pad(tot(d, le)))
//   where tot(d, le) = sum_r C[r][d*E_l + le] and gstart_d is the exclusive
//   prefix of the padded totals; inside it, the rows sent by rank r come
//   after those of ranks r' < r, in r's send order.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "mxg.h"
#include "mxg_internal.h"

namespace mxg {

__host__ __device__ inline int64_t pad_up(int64_t v, int pad) { return (v + pad - 1) / pad * pad; }

// One block.  counts [world][E] (E = world * e_local expert slots).
// Workspace: pref [world][E + 1] (per-rank exclusive prefix over slots),
// gs [E] (padded start of every slot in its owner's buffer), tot [E].
__global__ void p2p_plan_kernel(const int32_t* __restrict__ C, int world, int E, int me, int pad,
                                int32_t* __restrict__ pref, int32_t* __restrict__ gs,
                                int32_t* __restrict__ tot, int32_t* __restrict__ slot_start,
                                int32_t* __restrict__ dest_base, int32_t* __restrict__ group_rows,
                                int32_t* __restrict__ group_start) {
  const int e_local = E / world;
  for (int s = threadIdx.x; s < E; s += blockDim.x) {
    int32_t t = 0;
    for (int r = 0; r < world; ++r) t += C[r * E + s];
    tot[s] = t;
  }
  for (int r = threadIdx.x; r < world; r += blockDim.x) {
    int32_t run = 0;
    for (int s = 0; s < E; ++s) {
      pref[r * (E + 1) + s] = run;
      run += C[r * E + s];
    }
    pref[r * (E + 1) + E] = run;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < world; d += blockDim.x) {
    int32_t run = 0;
    for (int le = 0; le < e_local; ++le) {
      gs[d * e_local + le] = run;
      run += int32_t(pad_up(tot[d * e_local + le], pad));
    }
    if (d == me) group_start[e_local] = run;
  }
  __syncthreads();
  for (int s = threadIdx.x; s < E; s += blockDim.x) {
    int32_t src_off = 0;  // rows of slot s sent by ranks before me
    for (int r = 0; r < me; ++r) src_off += C[r * E + s];
    dest_base[s] = gs[s] + src_off - pref[me * (E + 1) + s];
  }
  for (int s = threadIdx.x; s <= E; s += blockDim.x) slot_start[s] = pref[me * (E + 1) + s];
  for (int le = threadIdx.x; le < e_local; le += blockDim.x) {
    group_rows[le] = int32_t(pad_up(tot[me * e_local + le], pad));
    group_start[le] = gs[me * e_local + le];
  }
}

// One block per local expert of `me`: for every padded row of its group, the
// rank and send position the result goes back to (-1 on padding rows).
// ret_order lists the real rows grouped by home rank in the order me+1,
// me+2, ..., me (mod world), local experts in order within a rank.
__global__ void p2p_back_kernel(const int32_t* __restrict__ C, int world, int E, int me, int pad,
                                const int32_t* __restrict__ pref, const int32_t* __restrict__ gs,
                                const int32_t* __restrict__ tot, int32_t* __restrict__ back_rank,
                                int32_t* __restrict__ back_row, int32_t* __restrict__ ret_order) {
  const int e_local = E / world;
  const int le = blockIdx.x;
  const int s = me * e_local + le;
  __shared__ int32_t base_s[MXG_EP_MAX_RANKS];
  if (threadIdx.x == 0) {
    // rows from each rank to me, accumulated in the rotated rank order, plus
    // the rows of that rank in my earlier local experts
    int32_t run = 0;
    for (int k = 1; k <= world; ++k) {
      const int r = (me + k) % world;
      int32_t before = 0, all = 0;
      for (int x = 0; x < e_local; ++x) {
        const int32_t c = C[r * E + me * e_local + x];
        if (x < le) before += c;
        all += c;
      }
      base_s[r] = run + before;
      run += all;
    }
  }
  __syncthreads();
  int32_t q0 = gs[s];
  for (int r = 0; r < world; ++r) {
    const int32_t c = C[r * E + s];
    const int32_t p0 = pref[r * (E + 1) + s];
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
      back_rank[q0 + i] = r;
      back_row[q0 + i] = p0 + i;
      ret_order[base_s[r] + i] = q0 + i;
    }
    q0 += c;
  }
  const int32_t end = gs[s] + int32_t(pad_up(tot[s], pad));
  for (int32_t q = q0 + threadIdx.x; q < end; q += blockDim.x) {
    back_rank[q] = -1;
    back_row[q] = -1;
  }
}

constexpr int kCopyThreads = 256;
constexpr int kCopyThreadsExclusive = 1024;
// Shared memory a copy block claims in exclusive mode (unused): more than an
// SM running a persistent GEMM block has left, so the copies only land on the
// SMs the GEMMs were told to leave free.
constexpr int kExclusiveSmem = 120 * 1024;
constexpr int kMaxSlotsSmem = MXG_EP_MAX_EXPERTS + 1;

// One warp copies one row, four 16-byte vectors in flight per lane.  Loads
// and stores are marked streaming (evict-first) so the exchange passes
// through L2 without displacing the operand tiles of GEMMs running beside it.
__device__ __forceinline__ void warp_copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                              int64_t row_vecs, int lane) {
  int64_t v = lane;
  for (; v + 96 < row_vecs; v += 128) {
    const uint4 a = __ldcs(src + v), b = __ldcs(src + v + 32), c = __ldcs(src + v + 64),
                d = __ldcs(src + v + 96);
    __stcs(dst + v, a);
    __stcs(dst + v + 32, b);
    __stcs(dst + v + 64, c);
    __stcs(dst + v + 96, d);
  }
  for (; v < row_vecs; v += 32) __stcs(dst + v, __ldcs(src + v));
}

// Dispatch: send position p (slot s, the largest with slot_start[s] <= p)
// -> row dest_base[s] + p of rank s / e_local.  One warp per row.  Send
// positions are ordered by destination rank; every rank starts with the
// positions of the rank after it (rotation `rot`), so at any moment the ranks
// write to different peers instead of all to the same one.  Only positions
// below slot_start[E] are routed (a routing slot whose expert id was out of
// range is counted nowhere and leaves its send_rows entry unwritten), and a
// source row outside [0, src_rows) is skipped and reported.  With src2, the
// same source row of src2 is also copied to row p of gather_out (local): a
// second tensor put in send order for a later exchange, in the same pass
// while this one is bound by NVLink.  With split_h > 0, positions of slots
// whose local expert index (slot % e_local) is >= split_h are not stored to
// their owner now: their src row goes to row p of src_later (local, send
// order) for a later exchange on the copy engines.
__global__ void __launch_bounds__(kCopyThreadsExclusive) p2p_dispatch_kernel(
    const uint4* __restrict__ src, int64_t src_rows, int64_t row_vecs,
    const int32_t* __restrict__ send_rows, int64_t n_send, const int32_t* __restrict__ slot_start,
    const int32_t* __restrict__ dest_base, int E, int e_local, int me,
    const uint64_t* __restrict__ peer_bufs, int64_t capacity_rows, int* err,
    const uint4* __restrict__ src2, uint4* __restrict__ gather_out, int split_h,
    uint4* __restrict__ src_later) {
  __shared__ int32_t ss[kMaxSlotsSmem];
  for (int i = threadIdx.x; i <= E; i += blockDim.x) ss[i] = slot_start[i];
  __syncthreads();
  const int world = E / e_local;
  const int64_t n_valid = min(n_send, int64_t(ss[E]));
  if (n_valid <= 0) return;
  const int64_t rot = min(int64_t(ss[((me + 1) % world) * e_local]), n_valid);
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n_valid;
       i += warps) {
    const int64_t p = (i + rot) % n_valid;
    int lo = 0, hi = E - 1;  // last slot with ss[s] <= p
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (ss[mid] <= p) lo = mid; else hi = mid - 1;
    }
    const int64_t row = int64_t(dest_base[lo]) + p;
    const int64_t src_row = send_rows[p];
    if (row < 0 || row >= capacity_rows) {
      if (lane == 0) atomicCAS(err, 0, MXG_ERR_WORKSPACE_TOO_SMALL);
      continue;
    }
    if (src_row < 0 || src_row >= src_rows) {
      if (lane == 0) atomicCAS(err, 0, MXG_ERR_INVALID_ARGUMENT);
      continue;
    }
    if (split_h > 0 && lo % e_local >= split_h)
      warp_copy_row(src_later + p * row_vecs, src + src_row * row_vecs, row_vecs, lane);
    else
      warp_copy_row(reinterpret_cast<uint4*>(peer_bufs[lo / e_local]) + row * row_vecs,
                    src + src_row * row_vecs, row_vecs, lane);
    if (src2 != nullptr) warp_copy_row(gather_out + p * row_vecs, src2 + src_row * row_vecs, row_vecs, lane);
  }
  __threadfence_system();
}

// Combine: padded local row q -> send position back_row[q] of rank
// back_rank[q], taking the rows in ret_order (grouped by home rank, starting
// with the rank after this one, as the dispatch does).
__global__ void __launch_bounds__(kCopyThreadsExclusive) p2p_return_kernel(
    const uint4* __restrict__ src, int64_t row_vecs, const int32_t* __restrict__ ret_order,
    int64_t n_rows, const int32_t* __restrict__ back_rank, const int32_t* __restrict__ back_row,
    const uint64_t* __restrict__ peer_bufs, int world, int64_t capacity_rows, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n_rows;
       i += warps) {
    const int64_t q = ret_order[i];
    const int r = back_rank[q];
    if (r < 0) continue;
    const int64_t row = back_row[q];
    if (r >= world || row < 0 || row >= capacity_rows) {
      if (lane == 0) atomicCAS(err, 0, MXG_ERR_WORKSPACE_TOO_SMALL);
      continue;
    }
    warp_copy_row(reinterpret_cast<uint4*>(peer_bufs[r]) + row * row_vecs, src + q * row_vecs,
                  row_vecs, lane);
  }
  __threadfence_system();
}

// Zero the padding rows (back_rank < 0) of a local receive buffer.
__global__ void __launch_bounds__(kCopyThreads) zero_pad_rows_kernel(uint4* __restrict__ buf,
                                                                     int64_t row_vecs,
                                                                     const int32_t* __restrict__ back_rank,
                                                                     int64_t m_pad) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t q = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); q < m_pad;
       q += warps) {
    if (back_rank[q] >= 0) continue;
    for (int64_t v = lane; v < row_vecs; v += 32) buf[q * row_vecs + v] = make_uint4(0, 0, 0, 0);
  }
}

// Launch shape of a peer-copy kernel.  max_blocks <= 0: as many 256-thread
// blocks as the rows need (up to 8 per SM), sharing SMs with whatever runs.
// max_blocks > 0 (exclusive): that many 1024-thread blocks, each claiming
// kExclusiveSmem so it can only run on an SM no GEMM block occupies.
struct CopyLaunch {
  int blocks, threads;
  size_t smem;
};

static CopyLaunch copy_launch(int64_t rows, int max_blocks) {
  if (max_blocks > 0) {
    const int64_t want = (rows + 31) / 32;
    return {int(std::max<int64_t>(1, std::min<int64_t>(want, max_blocks))), kCopyThreadsExclusive,
            size_t(kExclusiveSmem)};
  }
  const int64_t want = (rows + (kCopyThreads / 32) - 1) / (kCopyThreads / 32);
  return {int(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(num_sms()) * 8))), kCopyThreads, 0};
}

template <class K>
static int allow_exclusive_smem(K kernel) {
  return cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kExclusiveSmem + 4096));
}

static int copy_grid(int64_t rows, int max_blocks) { return copy_launch(rows, max_blocks).blocks; }

}  // namespace mxg

using namespace mxg;

extern "C" int mxg_peer_alloc(size_t bytes, void** dptr, void* handle_out) {
  if (!dptr || !handle_out || bytes == 0) return MXG_ERR_INVALID_ARGUMENT;
  int st = check_device();
  if (st) return st;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return MXG_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return MXG_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == MXG_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *dptr = p;
  return MXG_OK;
}

extern "C" int mxg_peer_open(const void* handle, void** dptr) {
  if (!handle || !dptr) return MXG_ERR_INVALID_ARGUMENT;
  int st = check_device();
  if (st) return st;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MXG_ERR_CUDA;
  *dptr = p;
  return MXG_OK;
}

extern "C" int mxg_peer_close(void* dptr) {
  if (!dptr) return MXG_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaIpcCloseMemHandle(dptr));
}

extern "C" int mxg_peer_free(void* dptr) {
  if (!dptr) return MXG_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaFree(dptr));
}

extern "C" size_t mxg_ep_p2p_plan_workspace_size(int world, int num_slots) {
  if (world < 1 || num_slots < 1) return 0;
  return sizeof(int32_t) * (size_t(world) * (num_slots + 1) + 2 * size_t(num_slots)) + 256;
}

extern "C" int mxg_ep_p2p_plan(const int32_t* counts_all, int world, int num_slots, int me, int pad,
                               int64_t m_pad, int32_t* slot_start, int32_t* dest_base,
                               int32_t* group_rows, int32_t* group_start, int32_t* back_rank,
                               int32_t* back_row, int32_t* ret_order, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!counts_all || !slot_start || !dest_base || !group_rows || !group_start || !workspace)
    return MXG_ERR_INVALID_ARGUMENT;
  if (world < 1 || world > MXG_EP_MAX_RANKS || num_slots < 1 || num_slots > MXG_EP_MAX_EXPERTS ||
      num_slots % world != 0 || me < 0 || me >= world || pad < 1 || m_pad < 0)
    return MXG_ERR_INVALID_ARGUMENT;
  if (m_pad > 0 && (!back_rank || !back_row || !ret_order)) return MXG_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < mxg_ep_p2p_plan_workspace_size(world, num_slots))
    return MXG_ERR_WORKSPACE_TOO_SMALL;
  int st = check_device();
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  int32_t* pref = reinterpret_cast<int32_t*>(workspace);
  int32_t* gs = pref + size_t(world) * (num_slots + 1);
  int32_t* tot = gs + num_slots;
  p2p_plan_kernel<<<1, 512, 0, s>>>(counts_all, world, num_slots, me, pad, pref, gs, tot,
                                    slot_start, dest_base, group_rows, group_start);
  if (m_pad > 0)
    p2p_back_kernel<<<num_slots / world, 256, 0, s>>>(counts_all, world, num_slots, me, pad, pref,
                                                      gs, tot, back_rank, back_row, ret_order);
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_ep_dispatch_p2p(const void* src, int64_t src_rows, int64_t row_bytes,
                                   const int32_t* send_rows, int64_t n_send,
                                   const int32_t* slot_start, const int32_t* dest_base,
                                   int num_slots, int e_local, int me, const uint64_t* peer_bufs,
                                   int64_t capacity_rows, int max_blocks, void* stream) {
  if (n_send < 0 || src_rows < 0 || row_bytes < 0 || num_slots < 1 || num_slots > MXG_EP_MAX_EXPERTS ||
      e_local < 1 || num_slots % e_local != 0 || capacity_rows < 0 || me < 0 ||
      me >= num_slots / e_local)
    return MXG_ERR_INVALID_ARGUMENT;
  if (row_bytes % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (n_send == 0 || row_bytes == 0) return MXG_OK;
  if (!src || !send_rows || !slot_start || !dest_base || !peer_bufs) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(src)) return MXG_ERR_MISALIGNED;
  int st = check_device();
  if (st) return st;
  int* err = device_error_word();
  if (!err) return MXG_ERR_CUDA;
  const CopyLaunch cl = copy_launch(n_send, max_blocks);
  if (cl.smem && (st = allow_exclusive_smem(p2p_dispatch_kernel))) return st;
  p2p_dispatch_kernel<<<cl.blocks, cl.threads, cl.smem, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint4*>(src), src_rows, row_bytes / 16, send_rows, n_send, slot_start,
      dest_base, num_slots, e_local, me, peer_bufs, capacity_rows, err, nullptr, nullptr, 0, nullptr);
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_ep_dispatch_p2p_gather(const void* src, int64_t src_rows, int64_t row_bytes,
                                          const int32_t* send_rows, int64_t n_send,
                                          const int32_t* slot_start, const int32_t* dest_base,
                                          int num_slots, int e_local, int me,
                                          const uint64_t* peer_bufs, int64_t capacity_rows,
                                          const void* src2, void* gather_out, int split_h,
                                          void* src_later, void* stream) {
  if (n_send < 0 || src_rows < 0 || row_bytes < 0 || num_slots < 1 || num_slots > MXG_EP_MAX_EXPERTS ||
      e_local < 1 || num_slots % e_local != 0 || capacity_rows < 0 || me < 0 ||
      me >= num_slots / e_local)
    return MXG_ERR_INVALID_ARGUMENT;
  if (row_bytes % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (n_send == 0 || row_bytes == 0) return MXG_OK;
  if (!src || !send_rows || !slot_start || !dest_base || !peer_bufs) return MXG_ERR_INVALID_ARGUMENT;
  if ((src2 == nullptr) != (gather_out == nullptr) || split_h < 0 || split_h > e_local ||
      (split_h > 0 && !src_later))
    return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(src) || (src2 && (!aligned16(src2) || !aligned16(gather_out))) ||
      (split_h > 0 && !aligned16(src_later)))
    return MXG_ERR_MISALIGNED;
  int st = check_device();
  if (st) return st;
  int* err = device_error_word();
  if (!err) return MXG_ERR_CUDA;
  const CopyLaunch cl = copy_launch(n_send, 0);
  p2p_dispatch_kernel<<<cl.blocks, cl.threads, cl.smem, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint4*>(src), src_rows, row_bytes / 16, send_rows, n_send, slot_start,
      dest_base, num_slots, e_local, me, peer_bufs, capacity_rows, err,
      reinterpret_cast<const uint4*>(src2), reinterpret_cast<uint4*>(gather_out), split_h,
      reinterpret_cast<uint4*>(src_later));
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_ep_return_p2p(const void* src, int64_t row_bytes, const int32_t* ret_order,
                                 int64_t n_rows, const int32_t* back_rank, const int32_t* back_row,
                                 const uint64_t* peer_bufs, int world, int64_t capacity_rows,
                                 int max_blocks, void* stream) {
  if (n_rows < 0 || row_bytes < 0 || world < 1 || capacity_rows < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (row_bytes % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (n_rows == 0 || row_bytes == 0) return MXG_OK;
  if (!src || !ret_order || !back_rank || !back_row || !peer_bufs) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(src)) return MXG_ERR_MISALIGNED;
  int st = check_device();
  if (st) return st;
  int* err = device_error_word();
  if (!err) return MXG_ERR_CUDA;
  const CopyLaunch cl = copy_launch(n_rows, max_blocks);
  if (cl.smem && (st = allow_exclusive_smem(p2p_return_kernel))) return st;
  p2p_return_kernel<<<cl.blocks, cl.threads, cl.smem, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint4*>(src), row_bytes / 16, ret_order, n_rows, back_rank, back_row,
      peer_bufs, world, capacity_rows, err);
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_ep_zero_pad_rows(void* buf, int64_t row_bytes, const int32_t* back_rank,
                                    int64_t m_pad, void* stream) {
  if (m_pad < 0 || row_bytes < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (row_bytes % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (m_pad == 0 || row_bytes == 0) return MXG_OK;
  if (!buf || !back_rank) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(buf)) return MXG_ERR_MISALIGNED;
  int st = check_device();
  if (st) return st;
  zero_pad_rows_kernel<<<copy_grid(m_pad, 0), kCopyThreads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<uint4*>(buf), row_bytes / 16, back_rank, m_pad);
  return cuda_status(cudaGetLastError());
}

extern "C" int mxg_copy_runs(const void* src, int64_t src_rows, int64_t row_bytes,
                             const int64_t* src_row, const int64_t* dst_row, const int64_t* rows,
                             const int32_t* dst_buf, int64_t n_runs, const uint64_t* dst_bufs,
                             int n_dst, int64_t dst_rows, void* stream) {
  if (n_runs < 0 || src_rows < 0 || row_bytes < 0 || n_dst < 0 || dst_rows < 0)
    return MXG_ERR_INVALID_ARGUMENT;
  if (n_runs == 0 || row_bytes == 0) return MXG_OK;
  if (!src || !src_row || !dst_row || !rows || !dst_buf || !dst_bufs) return MXG_ERR_INVALID_ARGUMENT;
  for (int64_t i = 0; i < n_runs; ++i) {  // every run in bounds before the first copy
    const int64_t n = rows[i];
    if (n < 0 || src_row[i] < 0 || src_row[i] > src_rows - n || dst_row[i] < 0 ||
        dst_row[i] > dst_rows - n || dst_buf[i] < 0 || dst_buf[i] >= n_dst || dst_bufs[dst_buf[i]] == 0)
      return MXG_ERR_INVALID_ARGUMENT;
  }
  int st = check_device();
  if (st) return st;
  const uint8_t* s8 = reinterpret_cast<const uint8_t*>(src);
  for (int64_t i = 0; i < n_runs; ++i) {
    if (rows[i] == 0) continue;
    uint8_t* d8 = reinterpret_cast<uint8_t*>(dst_bufs[dst_buf[i]]);
    const cudaError_t e = cudaMemcpyAsync(d8 + dst_row[i] * row_bytes, s8 + src_row[i] * row_bytes,
                                          size_t(rows[i] * row_bytes), cudaMemcpyDefault,
                                          (cudaStream_t)stream);
    if (e != cudaSuccess) return MXG_ERR_CUDA;
  }
  return MXG_OK;
}
