// Grouped MXFP8 GEMM for sm_100a (tcgen05 block-scaled MMA on CTA pairs, TMA, TMEM).
//
// One kernel serves both hot-path contractions.  Each computes, per group e,
//     D[i, j] = sum_k A[i, k] * B[j, k]       (both operands K-contiguous)
// with one E8M0 scale per 32 k for every row of A and of B:
//   forward (fused_fwd.py:172-230):  A = W[e] rows (features), B = token rows
//       of x in group e, k = hidden; stored transposed into y[token, feature]
//       ("swap AB": tokens sit on the MMA N side, so a tile's token count can
//       follow the group size exactly instead of padding to 128).
//   wgrad (wgrad_fused.py:34-112):   A = go rows (dW rows), B = ia rows (dW
//       columns), k = the group's token range read in place from the
//       token-contiguous operands; stored row-major into dW[e].
//
// Each cluster of two CTAs (one per SM) works as a pair on 256 A rows x up to
// 240 B rows: every CTA loads its own 128 A rows and half of the B rows, so an
// SM moves a third fewer operand bytes per MMA than a lone CTA would, and the
// leader CTA issues tcgen05.mma.cta_group::2 (M=256) whose accumulator rows
// land in each CTA's own TMEM.  No load uses multicast.
//   warp 4  TMA producer (both CTAs): A 128 x 128 B, B 120 x 128 B (128-byte
//           swizzle) and the pre-packed scale chunks, into a 6-stage ring;
//           completions are counted on the leader's barrier (.cta_group::2).
//   warp 5  TMEM (512 columns, pair allocation); in the leader one thread
//           copies the stage's scale factors to both TMEMs (tcgen05.cp) and
//           issues the MMAs; commits release both CTAs' stages (multicast).
//   warps 0-3 epilogue of each CTA: tcgen05.ld 32x32b, convert, store; the
//           accumulator is double-buffered so the epilogue of tile i overlaps
//           the main loop of tile i+1.
// Every mbarrier wait is bounded (MXG_ERR_DEVICE_TIMEOUT, then unwind).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <mutex>

#include "mxg.h"
#include "mxg_internal.h"
#include "mxg_ptx.cuh"

namespace mxg {

constexpr int kBM = 128;                 // A rows per CTA (a pair covers 256)
constexpr int kBNMax = 240;              // max B rows per pair tile (MMA N) of any mode
constexpr int kBK = 128;                 // contraction bytes per stage
constexpr int kABytes = kBM * kBK;       // 16 KiB
constexpr int kSfaBytes = 512;           // 128 rows x 4 scales, UTCCP layout
constexpr int kSfbBytes = 1024;          // 2 x (128 rows x 4 scales)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccStride = 256;     // accumulator buffer i at column 256*i
// Scale factors live in two TMEM buffers used by alternate stages, so the
// copy for stage s+1 never overwrites columns the MMAs of stage s still read:
// buffer 0 in columns 240-251, buffer 1 in 496-507 (SFA 4 columns, SFB 8).
constexpr uint32_t kSfCol0 = 240, kSfCol1 = 496;
constexpr uint32_t kSfbOff = 4;

enum { MODE_FWD = 0, MODE_WGRAD = 1 };

// Per-mode shape of the kernel.  The wgrad's epilogue writes 128 x N fp32
// (or bf16) per CTA and tile, about as long as a small expert's whole main
// loop, so it runs eight epilogue warps -- two per TMEM lane quarter, each
// with half of the tile's columns -- each staging its stores through one
// 2 KiB slot (16 fp32 or 32 bf16 columns, 64-byte rows per TMA store).
// Together they take the shared memory of four 4 KiB buffers, which is what
// fits beside six pipeline stages of 240-row B tiles (fewer stages starve
// the MMA: the operand loads need about five k-steps of lead).  Against four
// warps with 4 KiB buffers (128-byte rows) it does ~2.4% more work per SM
// cycle on the DSv3 GEMM set, same bytes; under the 1000 W cap the clock
// drops by as much, so sustained throughput is the same.  The forward's bf16
// epilogue is short next to its 56-step main loop and keeps four epilogue
// warps with 4 KiB buffers and 240-row B tiles.
//   warps 0-3 epilogue, 4 TMA producer, 5 MMA issuer, 6-9 epilogue (wgrad)
#ifndef MXG_WGRAD_EPI_WARPS
#define MXG_WGRAD_EPI_WARPS 8
#endif
#ifndef MXG_WGRAD_BN
#define MXG_WGRAD_BN 240
#endif
// staging bytes per wgrad epilogue warp: 2048 (16 fp32 / 32 bf16 columns,
// 64-byte rows per store) or 4096 (32 fp32 columns, 128-byte rows)
#ifndef MXG_WGRAD_EPI_SLOT
#define MXG_WGRAD_EPI_SLOT 2048
#endif
#define MXG_WGRAD_EPI_WARPS_FOR(m) ((m) == MODE_WGRAD ? MXG_WGRAD_EPI_WARPS : 4)
#define MXG_WGRAD_BN_FOR(m) ((m) == MODE_WGRAD ? MXG_WGRAD_BN : 240)
template <int MODE>
struct Cfg {
  static constexpr int kStages = 6;
  static constexpr int kEpiWarps = MXG_WGRAD_EPI_WARPS_FOR(MODE);
  static constexpr int kEpiBytes = MODE == MODE_WGRAD ? MXG_WGRAD_EPI_SLOT : 4096;
  static constexpr int kThreads = 32 * (kEpiWarps + 2);
  static constexpr int kBN = MXG_WGRAD_BN_FOR(MODE);            // max B rows per pair tile
  static constexpr int kBHalf = kBN / 2;                       // B rows each CTA loads
  static constexpr int kBBytes = kBHalf * kBK;
  static constexpr uint32_t kStageTxPerCta = kABytes + kBBytes + kSfaBytes + kSfbBytes;
};
__host__ __device__ constexpr int bn_max(int mode) {
  return mode == MODE_WGRAD ? Cfg<MODE_WGRAD>::kBN : Cfg<MODE_FWD>::kBN;
}
static_assert(Cfg<MODE_FWD>::kBN <= kBNMax && Cfg<MODE_WGRAD>::kBN <= kBNMax, "TMEM columns");

// ---- scheduler output (int32 words in the workspace) ------------------------
//   [0] tiles  [1] A scale chunks  [2] B scale chunks  [3] first row after the
//   last group (forward zero-fill)  [4..7] reserved, then the arrays below.
struct MetaView {
  int* base;
  int E;
  __host__ __device__ int* tile_start() const { return base + 8; }           // E+1
  __host__ __device__ int* g_start() const { return base + 8 + (E + 1); }    // E
  __host__ __device__ int* g_len() const { return g_start() + E; }          // E
  __host__ __device__ int* g_nt() const { return g_len() + E; }             // E
  __host__ __device__ int* g_kb() const { return g_nt() + E; }              // E
  __host__ __device__ int* g_asf() const { return g_kb() + E; }             // E+1
  __host__ __device__ int* g_bsf() const { return g_asf() + E + 1; }        // E+1
  __host__ __device__ static size_t words(int E) { return 8 + 7 * size_t(E) + 3; }
};

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Balanced split of `ext` rows into `nt` tiles of whole 16-row units (each
// at most the mode's B tile rows).  Returns the first row and the row count of tile `i`.
__host__ __device__ inline void split_rows(int ext, int nt, int i, int& n0, int& nlen) {
  const int units = (ext + 15) / 16;
  const int q = units / nt, r = units % nt;
  const int u0 = i * q + (i < r ? i : r);
  const int ul = q + (i < r ? 1 : 0);
  n0 = 16 * u0;
  nlen = min(16 * ul, ext - n0);
}

// ---------------------------------------------------------------- scheduler
struct SchedArgs {
  const int32_t* offs;
  int offs_len;
  int offs_kind;
  int E;
  int M;
  int mode;
  int n_out;   // A-side rows per group
  int n_ext;   // wgrad: B-side rows (dW columns)
  int k_fwd;   // forward contraction length
  int* meta;
  int* err;
};

__device__ int block_excl_scan(int v, int* total, int* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < (blockDim.x >> 5)) warp_sums[lane] = w;
  }
  __syncthreads();
  const int before = (warp ? warp_sums[warp - 1] : 0) + x - v;
  *total = warp_sums[(blockDim.x >> 5) - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(MXG_MAX_GROUPS) schedule_kernel(SchedArgs a) {
  __shared__ int raw[MXG_MAX_GROUPS + 1];
  __shared__ int warp_sums[32];
  __shared__ int kind_s;
  const int tid = threadIdx.x, E = a.E;
  const int L = a.offs ? a.offs_len : 0;
  for (int i = tid; i < L && i <= MXG_MAX_GROUPS; i += blockDim.x) raw[i] = a.offs[i];
  if (tid == 0) kind_s = a.offs ? a.offs_kind : -1;
  __syncthreads();
  bool bad = false;
  int kind = kind_s;
  if (kind == MXG_OFFS_AUTO) {
    if (L == E + 1) {
      kind = MXG_OFFS_LEADING_ZERO;
    } else {
      const bool mono = (tid < E - 1) ? raw[tid] <= raw[tid + 1] : true;
      const bool all_mono = __syncthreads_and(mono);
      if (all_mono && raw[E - 1] == a.M) {
        kind = MXG_OFFS_CUMULATIVE;
      } else {
        int tot;
        (void)block_excl_scan(tid < E ? raw[tid] : 0, &tot, warp_sums);
        const bool nonneg = __syncthreads_and(tid < E ? raw[tid] >= 0 : true);
        kind = (nonneg && tot == a.M) ? MXG_OFFS_SIZES : -2;
      }
    }
  }
  // group starts and lengths
  int start = 0, len = 0;
  if (kind == -1) {  // no offsets: one group of all rows
    start = 0;
    len = (tid == 0) ? a.M : 0;
  } else if (kind == MXG_OFFS_LEADING_ZERO) {
    if (tid < E) {
      start = raw[tid];
      len = raw[tid + 1] - raw[tid];
    }
    if (tid == 0 && raw[0] != 0) bad = true;
  } else if (kind == MXG_OFFS_CUMULATIVE) {
    if (tid < E) {
      start = tid ? raw[tid - 1] : 0;
      len = raw[tid] - start;
    }
  } else if (kind == MXG_OFFS_SIZES) {
    int tot;
    const int sz = tid < E ? raw[tid] : 0;
    start = block_excl_scan(sz, &tot, warp_sums);
    len = sz;
  } else {
    bad = true;
  }
  if (tid < E) {
    if (len < 0 || start < 0 || start + len > a.M) bad = true;
    if (a.mode == MODE_WGRAD && ((start & 31) || (len & 31))) bad = true;
  }
  const bool any_bad = __syncthreads_or(bad);
  // per-group work counts
  int nt = 0, kb = 0, tiles = 0, asf = 0, bsf = 0;
  const int mbp = ceil_div(a.n_out, 2 * kBM);  // pairs of 128-row A blocks
  if (tid < E && !any_bad) {
    if (a.mode == MODE_FWD) {
      nt = ceil_div(len, bn_max(MODE_FWD));
      kb = ceil_div(a.k_fwd, kBK);
    } else {
      nt = ceil_div(a.n_ext, bn_max(MODE_WGRAD));
      kb = ceil_div(len, kBK);
    }
    tiles = mbp * nt;
    asf = 2 * mbp * kb;  // every pair has two A blocks (the second may be past n_out)
    bsf = nt * kb;
  }
  int t_tot, a_tot, b_tot;
  const int t0 = block_excl_scan(tiles, &t_tot, warp_sums);
  const int a0 = block_excl_scan(asf, &a_tot, warp_sums);
  const int b0 = block_excl_scan(bsf, &b_tot, warp_sums);
  MetaView mv{a.meta, E};
  if (tid < E) {
    mv.tile_start()[tid] = t0;
    mv.g_start()[tid] = any_bad ? 0 : start;
    mv.g_len()[tid] = any_bad ? 0 : len;
    mv.g_nt()[tid] = nt;
    mv.g_kb()[tid] = kb;
    mv.g_asf()[tid] = a0;
    mv.g_bsf()[tid] = b0;
  }
  // last group's end = first uncovered row (groups are contiguous from row 0)
  int end_local = (tid < E) ? start + len : 0;
  for (int o = 16; o > 0; o >>= 1) end_local = max(end_local, __shfl_xor_sync(0xffffffffu, end_local, o));
  if ((tid & 31) == 0) warp_sums[tid >> 5] = end_local;
  __syncthreads();
  if (tid == 0) {
    int end_all = 0;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) end_all = max(end_all, warp_sums[w]);
    mv.tile_start()[E] = t_tot;
    mv.g_asf()[E] = a_tot;
    mv.g_bsf()[E] = b_tot;
    a.meta[0] = any_bad ? 0 : t_tot;
    a.meta[1] = any_bad ? 0 : a_tot;
    a.meta[2] = any_bad ? 0 : b_tot;
    a.meta[3] = any_bad ? 0 : end_all;
    if (any_bad) atomicCAS(a.err, 0, MXG_ERR_BAD_OFFSETS);
  }
}

// ---------------------------------------------------------------- scale packing
// Re-lays the row-major E8M0 scales of one operand into 512-byte chunks, one
// per (128 rows, 128 contraction elements): byte (r%32)*16 + (r/32)*4 + kk
// for row r and 32-element block kk -- the shared-memory layout that
// tcgen05.cp 32x128b.warpx4 turns into the TMEM scale-factor layout.  Rows or
// blocks outside the operand are filled with 0x7F (unit scale; those rows and
// steps are never stored or issued).
struct PackArgs {
  const int* meta;
  int E;
  int mode;
  int side;             // 0: A operand (128-row chunks), 1: B operand (2 x 128 rows)
  const uint8_t* src;   // row-major scales, null -> unit scales
  int64_t src_ld;       // bytes per scale row
  uint8_t* dst;
  int n_out;
  int n_ext;
  int k_fwd;
};

// One block per (group, operand row block): thread r owns row r of the block
// and walks that row's scales across the group's contraction range (one
// contiguous run of bytes per thread), writing its word of every chunk.
// A side: 2*mbp blocks of 128 rows per group; B side: one block per N tile
// (<= 240 rows, two 128-row halves).
// Bytes [col, col + 4) of a scale row as one word (0x7F past col_end): an
// aligned load, two joined with a funnel shift when the run is not word
// aligned (used only if the second word still ends inside the row), or byte
// loads at the edges.
__device__ __forceinline__ uint32_t scale_word(const uint8_t* srow, const uint32_t* wp, uint32_t sh,
                                               const uint8_t* row_end, int kb, int col, int col_end) {
  if (col + 4 <= col_end && sh == 0) return __ldg(wp + kb);
  if (col + 4 <= col_end && reinterpret_cast<const uint8_t*>(wp + kb + 2) <= row_end)
    return __funnelshift_r(__ldg(wp + kb), __ldg(wp + kb + 1), sh);
  uint32_t word = 0;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint32_t v = col + kk < col_end ? uint32_t(__ldg(srow + col + kk)) : 0x7Fu;
    word |= v << (8 * kk);
  }
  return word;
}

__device__ __forceinline__ void pack_rows(const PackArgs& p, int bid, int nblk) {
  __shared__ int ustart[MXG_MAX_GROUPS + 1];  // B side: first unit of each group
  MetaView mv{const_cast<int*>(p.meta), p.E};
  const int mbp = ceil_div(p.n_out, 2 * kBM);
  if (p.side == 1) {
    for (int i = threadIdx.x; i <= p.E; i += blockDim.x) ustart[i] = mv.tile_start()[i] / mbp;
    __syncthreads();
  }
  const int units = p.side == 0 ? p.E * 2 * mbp : ustart[p.E];
  // A thread packs rows q, q+32, q+64, q+96 of one 128-row half and stores
  // their four words as one 16-byte vector (a warp writes a whole 512-byte
  // chunk half per k-block instead of scattering 4-byte words).  A block
  // takes one unit at a time; its thread groups split the unit's k-blocks
  // (group ks takes ks, ks + KS, ...), which keeps each thread's chain of
  // dependent loads short.
  const int rows_per_unit = p.side == 0 ? kBM : 2 * kBM;
  const int tpu = rows_per_unit / 4;            // threads per k-block of a unit
  const int KS = int(blockDim.x) / tpu;         // k-split groups per unit
  const int ks = int(threadIdx.x) / tpu, t = int(threadIdx.x) % tpu;
  const int half = t >> 5, q = t & 31;
  const int64_t chunk_bytes = p.side == 0 ? kSfaBytes : kSfbBytes;
  // With 16-byte aligned scale rows a unit's rows are staged through shared
  // memory in slabs of 32 k-blocks (128 bytes of each row), read with
  // coalesced 16-byte loads, instead of each thread walking its rows word by
  // word.  The padding column keeps the chunk reads conflict-free.
  constexpr int kSlab = 32;
  __shared__ uint32_t slab[2 * kBM][kSlab + 1];
  const bool staged = p.mode == MODE_FWD && p.src != nullptr && p.src_ld % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(p.src) & 15u) == 0;
  for (int u = bid; u < units; u += nblk) {
    int e, blk;
    if (p.side == 0) {
      e = u / (2 * mbp);
      blk = u - e * 2 * mbp;
    } else {
      int lo = 0, hi = p.E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ustart[mid] <= u) lo = mid; else hi = mid - 1;
      }
      e = lo;
      blk = u - ustart[e];
    }
    const int kbn = mv.g_kb()[e];
    const int gstart = mv.g_start()[e], glen = mv.g_len()[e];
    int row0, valid, col0, col_end, chunk0;
    if (p.side == 0) {
      row0 = (p.mode == MODE_FWD ? e * p.n_out : 0) + blk * kBM;
      valid = min(kBM, p.n_out - blk * kBM);
      chunk0 = mv.g_asf()[e] + blk * kbn;
    } else {
      const int ext = p.mode == MODE_FWD ? glen : p.n_ext;
      int n0, nlen;
      split_rows(ext, mv.g_nt()[e], blk, n0, nlen);
      row0 = (p.mode == MODE_FWD ? gstart : 0) + n0;
      valid = nlen;
      chunk0 = mv.g_bsf()[e] + blk * kbn;
    }
    if (p.mode == MODE_FWD) {
      col0 = 0;
      col_end = p.k_fwd / 32;
    } else {
      col0 = gstart / 32;
      col_end = (gstart + glen) / 32;
    }
    if (staged) {
      const int halves = p.side == 0 ? 1 : 2;
      const int rows = halves * kBM;
      const int warp = int(threadIdx.x) >> 5, lane = int(threadIdx.x) & 31, nwarps = int(blockDim.x) >> 5;
      for (int kb0 = 0; kb0 < kbn; kb0 += kSlab) {
        const int nkb = min(kSlab, kbn - kb0);
        for (int i = int(threadIdx.x); i < rows * (kSlab / 4); i += int(blockDim.x)) {
          const int r = i / (kSlab / 4), pc = i % (kSlab / 4);
          const int c = col0 + kb0 * 4 + pc * 16;  // byte column of this 16-byte piece
          uint32_t v[4] = {0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu};
          if (r < valid && c < col_end) {
            const uint8_t* src = p.src + int64_t(row0 + r) * p.src_ld + c;
            if (c + 16 <= col_end) {
              const uint4 x = __ldg(reinterpret_cast<const uint4*>(src));
              v[0] = x.x;
              v[1] = x.y;
              v[2] = x.z;
              v[3] = x.w;
            } else {
#pragma unroll
              for (int b = 0; b < 16; ++b) {
                const uint32_t byte = c + b < col_end ? uint32_t(__ldg(src + b)) : 0x7Fu;
                v[b >> 2] = (v[b >> 2] & ~(0xFFu << (8 * (b & 3)))) | (byte << (8 * (b & 3)));
              }
            }
          }
#pragma unroll
          for (int w = 0; w < 4; ++w) slab[r][pc * 4 + w] = v[w];
        }
        __syncthreads();
        // one warp per (k-block, 128-row half): lane q stores rows q, q+32,
        // q+64, q+96 of the half as one 16-byte piece of the chunk
        for (int it = warp; it < nkb * halves; it += nwarps) {
          const int kl = it / halves, h = it - kl * halves;
          const uint4 w4 = make_uint4(slab[h * kBM + lane][kl], slab[h * kBM + lane + 32][kl],
                                      slab[h * kBM + lane + 64][kl], slab[h * kBM + lane + 96][kl]);
          *reinterpret_cast<uint4*>(p.dst + int64_t(chunk0 + kb0 + kl) * chunk_bytes + h * 512 + lane * 16) = w4;
        }
        __syncthreads();  // the slab is reloaded next
      }
      continue;
    }
    // per row j: start of its run, the aligned word pointer and the shift
    const uint8_t* srow[4];
    const uint32_t* wp[4];
    uint32_t sh[4];
    bool live[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = half * kBM + q + 32 * j;
      live[j] = p.src && r < valid;
      srow[j] = live[j] ? p.src + int64_t(row0 + r) * p.src_ld : p.src;
      const uintptr_t a = reinterpret_cast<uintptr_t>(srow[j] + col0);
      wp[j] = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
      sh[j] = uint32_t(a & 3u) * 8u;
    }
    uint4* d = reinterpret_cast<uint4*>(p.dst + int64_t(chunk0) * chunk_bytes + half * 512 + q * 16);
#pragma unroll 4
    for (int kb = ks; kb < kbn; kb += KS) {
      const int col = col0 + kb * 4;
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w[j] = live[j] ? scale_word(srow[j], wp[j], sh[j], srow[j] + p.src_ld, kb, col, col_end)
                       : 0x7F7F7F7Fu;
      d[int64_t(kb) * (chunk_bytes / 16)] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}


// Chunk-parallel variant: one block per chunk at a time, thread r reads the
// four bytes of row r.  Faster than the row walk when the scale rows are not
// word aligned (the wgrad's token-contiguous scales, M/32 bytes per row).
__device__ __forceinline__ void pack_chunks(const PackArgs& p, int bid, int nblk) {
  __shared__ int base_s[MXG_MAX_GROUPS + 1];
  MetaView mv{const_cast<int*>(p.meta), p.E};
  const int* base = p.side == 0 ? mv.g_asf() : mv.g_bsf();
  for (int i = threadIdx.x; i <= p.E; i += blockDim.x) base_s[i] = base[i];
  __syncthreads();
  // one warp per 128-row half of a chunk: lane q packs rows q, q+32, q+64,
  // q+96 into one 16-byte store
  const int halves = p.side == 0 ? 1 : 2;
  const int64_t chunk_bytes = p.side == 0 ? kSfaBytes : kSfbBytes;
  const int total = base_s[p.E] * halves;
  const int lane = threadIdx.x & 31;
  const int warps = int(nblk * blockDim.x) >> 5;
  for (int item = int(bid * blockDim.x + threadIdx.x) >> 5; item < total; item += warps) {
    const int c = item / halves, half = item - c * halves;
    int lo = 0, hi = p.E - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (base_s[mid] <= c) lo = mid; else hi = mid - 1;
    }
    const int e = lo;
    const int local = c - base_s[e];
    const int kbn = mv.g_kb()[e];
    const int blk = local / kbn, kb = local - blk * kbn;
    const int gstart = mv.g_start()[e], glen = mv.g_len()[e];
    int row0, valid, col0, col_end;
    if (p.side == 0) {
      row0 = (p.mode == MODE_FWD ? e * p.n_out : 0) + blk * kBM;
      valid = min(kBM, p.n_out - blk * kBM);
    } else {
      const int ext = p.mode == MODE_FWD ? glen : p.n_ext;
      int n0, nlen;
      split_rows(ext, mv.g_nt()[e], blk, n0, nlen);
      row0 = (p.mode == MODE_FWD ? gstart : 0) + n0;
      valid = nlen;
    }
    if (p.mode == MODE_FWD) {
      col0 = kb * 4;
      col_end = p.k_fwd / 32;
    } else {
      col0 = gstart / 32 + kb * 4;
      col_end = (gstart + glen) / 32;
    }
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = half * kBM + lane + 32 * j;
      uint32_t word = 0x7F7F7F7Fu;
      if (p.src && r < valid) {  // one word, or two joined by a funnel shift, or bytes at the edges
        const uint8_t* srow = p.src + int64_t(row0 + r) * p.src_ld;
        const uintptr_t a = reinterpret_cast<uintptr_t>(srow + col0);
        word = scale_word(srow, reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3)), uint32_t(a & 3u) * 8u,
                          srow + p.src_ld, 0, col0, col_end);
      }
      w[j] = word;
    }
    *reinterpret_cast<uint4*>(p.dst + int64_t(c) * chunk_bytes + half * 512 + lane * 16) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Both operands' scales in one launch: blocks [0, blocks0) pack the A side,
// the rest the B side, so the two run side by side with one kernel boundary
// between the scheduler and the GEMM instead of two.
struct PackPair {
  PackArgs side[2];
  int blocks0;
};

__global__ void __launch_bounds__(256) pack_scales_kernel(PackPair pp) {
  const bool second = int(blockIdx.x) >= pp.blocks0;
  pack_rows(pp.side[second ? 1 : 0], second ? int(blockIdx.x) - pp.blocks0 : int(blockIdx.x),
            second ? int(gridDim.x) - pp.blocks0 : pp.blocks0);
}

__global__ void __launch_bounds__(256) pack_scales_chunk_kernel(PackPair pp) {
  const bool second = int(blockIdx.x) >= pp.blocks0;
  pack_chunks(pp.side[second ? 1 : 0], second ? int(blockIdx.x) - pp.blocks0 : int(blockIdx.x),
              second ? int(gridDim.x) - pp.blocks0 : pp.blocks0);
}


// ---------------------------------------------------------------- GEMM kernel (CTA pairs)
struct GemmArgs {
  const int* meta;
  void* out;
  int out_dtype;
  int E;
  int n_out;     // A rows per group (forward: features N; wgrad: dW rows N)
  int n_ext;     // wgrad: dW columns K
  int k_fwd;     // forward contraction K
  int64_t ldo;   // output row stride in elements
  int* err;
  uint64_t timeout_ns;
  int stall_test;
  int fwd_tma_store;    // forward output row stride is 16-byte aligned: store via TMA
  int wgrad_tma_store;  // wgrad output row stride is 16-byte aligned: store via TMA
  // forward, bf16, scatter mode (non-null scatter_bufs): output row q leaves
  // for row back_row[q] of buffer scatter_bufs[back_rank[q]] (this GPU's or
  // a peer's memory, plain stores), nothing is written to `out`
  const uint64_t* scatter_bufs;
  const int32_t* back_rank;
  const int32_t* back_row;
  int scatter_nbufs;
  int64_t scatter_rows;
};

template <int S, int EW, int BB, int EB>
struct __align__(1024) SmemT {
  static constexpr int kStages = S;
  uint8_t a[S][kABytes];
  uint8_t b[S][BB];
  uint8_t sfa[S][kSfaBytes];
  uint8_t sfb[S][kSfbBytes];
  alignas(1024) uint8_t epi[EW][EB];    // per epilogue warp: staging (4 KiB: two 2 KiB slots), swizzled
  uint64_t full[S];            // leader: both CTAs' loads of the stage landed
  uint64_t empty[S];           // each CTA: the pair MMA finished reading the stage
  uint64_t acc_full[2];        // each CTA: accumulator buffer complete
  uint64_t acc_empty[2];       // leader: both CTAs' epilogues drained the buffer
  uint64_t drain;
  uint64_t never;
  uint32_t tmem_base;
  int abort_flag;
  int num_tiles;
  // first tile of each group (the per-tile binary search); the other
  // per-group fields are read from the scheduler's table in global memory
  int tile_start[MXG_MAX_GROUPS + 1];
};
template <int MODE>
using SmemOf = SmemT<Cfg<MODE>::kStages, Cfg<MODE>::kEpiWarps, Cfg<MODE>::kBBytes, Cfg<MODE>::kEpiBytes>;
template <int MODE>
constexpr size_t smem_bytes() { return sizeof(SmemOf<MODE>) + 1024; }
// swizzled tiles must start on 1024-byte boundaries (the swizzle pattern is
// taken from address bits 4-9)
template <class L>
constexpr bool layout_ok() {
  return offsetof(L, a) % 1024 == 0 && offsetof(L, b) % 1024 == 0 && offsetof(L, epi) % 1024 == 0 &&
         kABytes % 1024 == 0 && sizeof(L::b[0]) % 1024 == 0;
}
static_assert(layout_ok<SmemOf<MODE_FWD>>() && layout_ok<SmemOf<MODE_WGRAD>>(), "tile alignment");
static_assert(smem_bytes<MODE_FWD>() <= 232448 && smem_bytes<MODE_WGRAD>() <= 232448,
              "shared memory budget");

struct TileInfo {
  int e, mb, nt, n0, nlen, kb_count, klen, k0, a_row, b_row, sfa0, sfb0;
};

// Walks one CTA's pair tiles in increasing order (t = pair, pair + npairs,
// ...) and decodes tile t as seen by CTA `rank` of the pair: its own 128-row
// A block (mb = 2 * pair block + rank) and the pair's B rows [b_row, b_row +
// nlen).  The current group's fields stay cached, so the next tile costs one
// division; a binary search over the groups' first tiles happens only for
// the first tile (a per-tile search and the table loads cost ~700 cycles).
template <int MODE>
struct TileWalker {
  int e = -1, ts = 0, te = 0, nt_count = 1, q = 0, r = 0, kb = 0, gstart = 0, glen = 0, asf = 0,
      bsf = 0, ext = 0;

  template <class SL>
  __device__ __forceinline__ void enter(const SL& s, const GemmArgs& g, int grp) {
    e = grp;
    ts = s.tile_start[grp];
    te = s.tile_start[grp + 1];
    const MetaView mv{const_cast<int*>(g.meta), g.E};
    nt_count = max(__ldg(mv.g_nt() + grp), 1);
    gstart = __ldg(mv.g_start() + grp);
    glen = __ldg(mv.g_len() + grp);
    kb = __ldg(mv.g_kb() + grp);
    asf = __ldg(mv.g_asf() + grp);
    bsf = __ldg(mv.g_bsf() + grp);
    ext = MODE == MODE_FWD ? glen : g.n_ext;
    const int units = (ext + 15) / 16;  // split_rows' balanced split, per group
    q = units / nt_count;
    r = units - q * nt_count;
  }

  template <class SL>
  __device__ __forceinline__ TileInfo at(const SL& s, const GemmArgs& g, int t, int rank) {
    if (e < 0 || t < ts) {
      int lo = 0, hi = g.E - 1;  // last group whose first tile is <= t
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s.tile_start[mid] <= t) lo = mid; else hi = mid - 1;
      }
      enter(s, g, lo);
    }
    while (t >= te) enter(s, g, e + 1);  // groups without tiles are passed over
    TileInfo ti;
    ti.e = e;
    const int local = t - ts;
    const int mbp = local / nt_count;
    ti.nt = local - mbp * nt_count;
    ti.mb = 2 * mbp + rank;
    const int u0 = ti.nt * q + min(ti.nt, r);
    const int ul = q + (ti.nt < r ? 1 : 0);
    ti.n0 = 16 * u0;
    ti.nlen = min(16 * ul, ext - ti.n0);
    ti.kb_count = kb;
    if (MODE == MODE_FWD) {
      ti.klen = g.k_fwd;
      ti.k0 = 0;
      ti.a_row = e * g.n_out + ti.mb * kBM;
      ti.b_row = gstart + ti.n0;
    } else {
      ti.klen = glen;
      ti.k0 = gstart;
      ti.a_row = ti.mb * kBM;
      ti.b_row = ti.n0;
    }
    ti.sfa0 = asf + ti.mb * ti.kb_count;
    ti.sfb0 = bsf + ti.nt * ti.kb_count;
    return ti;
  }

  // For a whole warp: every field broadcast from lane 0, so the compiler can
  // keep tile coordinates in uniform registers.
  template <class SL>
  __device__ __forceinline__ TileInfo at_warp(const SL& s, const GemmArgs& g, int t, int rank) {
    TileInfo ti = at(s, g, t, rank);
    ti.e = __shfl_sync(0xffffffffu, ti.e, 0);
    ti.mb = __shfl_sync(0xffffffffu, ti.mb, 0);
    ti.nt = __shfl_sync(0xffffffffu, ti.nt, 0);
    ti.n0 = __shfl_sync(0xffffffffu, ti.n0, 0);
    ti.nlen = __shfl_sync(0xffffffffu, ti.nlen, 0);
    ti.kb_count = __shfl_sync(0xffffffffu, ti.kb_count, 0);
    ti.klen = __shfl_sync(0xffffffffu, ti.klen, 0);
    ti.k0 = __shfl_sync(0xffffffffu, ti.k0, 0);
    ti.a_row = __shfl_sync(0xffffffffu, ti.a_row, 0);
    ti.b_row = __shfl_sync(0xffffffffu, ti.b_row, 0);
    ti.sfa0 = __shfl_sync(0xffffffffu, ti.sfa0, 0);
    ti.sfb0 = __shfl_sync(0xffffffffu, ti.sfb0, 0);
    return ti;
  }
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Epilogue store of 32 accumulator columns [c0, c0+32) held by this thread
// (TMEM lane = `row` of this CTA's 128-row block).
template <int MODE>
__device__ __forceinline__ void store_chunk(const GemmArgs& g, const TileInfo& ti, int row, int c0,
                                            const uint32_t (&v)[32], bool zero) {
  const int ncols = min(32, ti.nlen - c0);
  if (MODE == MODE_FWD) {
    const int f = ti.mb * kBM + row;
    if (f >= g.n_out) return;
    const int64_t tok0 = int64_t(ti.b_row) + c0;
    if (g.out_dtype == MXG_DTYPE_BF16) {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + tok0 * g.ldo + f;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) o[int64_t(j) * g.ldo] = __float2bfloat16_rn(zero ? 0.f : __uint_as_float(v[j]));
    } else {
      float* o = reinterpret_cast<float*>(g.out) + tok0 * g.ldo + f;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) o[int64_t(j) * g.ldo] = zero ? 0.f : __uint_as_float(v[j]);
    }
  } else {
    const int r = ti.mb * kBM + row;
    if (r >= g.n_out) return;
    const int64_t off = (int64_t(ti.e) * g.n_out + r) * g.ldo + ti.n0 + c0;
    if (g.out_dtype == MXG_DTYPE_F32) {
      float* o = reinterpret_cast<float*>(g.out) + off;
      if (ncols == 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 q = zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                          : make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                        __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
          *reinterpret_cast<float4*>(o + j) = q;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) o[j] = zero ? 0.f : __uint_as_float(v[j]);
      }
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + off;
      if (ncols == 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 q;
          if (zero) {
            q = make_uint4(0, 0, 0, 0);
          } else {
            q.x = pack_bf16x2(__uint_as_float(v[j]), __uint_as_float(v[j + 1]));
            q.y = pack_bf16x2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
            q.z = pack_bf16x2(__uint_as_float(v[j + 4]), __uint_as_float(v[j + 5]));
            q.w = pack_bf16x2(__uint_as_float(v[j + 6]), __uint_as_float(v[j + 7]));
          }
          *reinterpret_cast<uint4*>(o + j) = q;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) o[j] = __float2bfloat16_rn(zero ? 0.f : __uint_as_float(v[j]));
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(Cfg<MODE>::kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmSFA,
                        const __grid_constant__ CUtensorMap tmSFB,
                        const __grid_constant__ CUtensorMap tmOut,
                        const __grid_constant__ CUtensorMap tmOut16,
                        const __grid_constant__ CUtensorMap tmOutAux, GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  using SL = SmemOf<MODE>;
  constexpr int kStages = Cfg<MODE>::kStages, kEpiWarps = Cfg<MODE>::kEpiWarps;
  constexpr int kThreads = Cfg<MODE>::kThreads;
  SL& s = *reinterpret_cast<SL*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = int(cluster_ctarank());
  const int pair = int(cluster_id_x());
  const int npairs = int(num_clusters_x());

  MetaView mv{const_cast<int*>(g.meta), g.E};
  for (int i = threadIdx.x; i <= g.E; i += kThreads) s.tile_start[i] = mv.tile_start()[i];
  if (threadIdx.x == 0) {
    s.num_tiles = g.meta[0];
    s.abort_flag = 0;
  }
  if (warp == 4 && lane == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&s.full[i]), 1);
      mbar_init(smem_u32(&s.empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s.acc_full[i]), 1);
      mbar_init(smem_u32(&s.acc_empty[i]), 2 * kEpiWarps);  // one arrival per epilogue warp, both CTAs
    }
    mbar_init(smem_u32(&s.drain), 1);
    mbar_init(smem_u32(&s.never), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmSFA);
    tma_prefetch_desc(&tmSFB);
  }
  if (warp == 5) {
    tmem_alloc_pair(smem_u32(&s.tmem_base), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  const int num_tiles = s.num_tiles;
  WaitCtl wc{&s.abort_flag, g.err, g.timeout_ns, mapa_shared(smem_u32(&s.abort_flag), rank ^ 1)};

  if (warp == 4) {
    // ------------------------------------------------------------ producer (both CTAs)
    // The whole warp runs the loop (tile fields stay warp-uniform); one
    // elected lane issues the copies.
    uint32_t stage = 0, phase = 0, armed = 0, armed_par = 0;
    bool ok = true;
    TileWalker<MODE> walk;
    for (int t = pair; t < num_tiles && ok; t += npairs) {
      const TileInfo ti = walk.at_warp(s, g, t, rank);
      const int half = int((uint32_t(ti.nlen + 15) & ~15u) >> 1);
      for (int kb = 0; kb < ti.kb_count; ++kb) {
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&s.empty[stage]), phase ^ 1u, wc))) {
          ok = false;
          break;
        }
        if (elect_one_sync()) {
          const uint32_t fb_local = smem_u32(&s.full[stage]);
          if (rank == 0) mbar_arrive_expect_tx(fb_local, 2 * Cfg<MODE>::kStageTxPerCta);
          const uint32_t fb = mapa_shared(fb_local, 0);
          const int x = ti.k0 + kb * kBK;
          tma_load_2d_pair(smem_u32(s.a[stage]), &tmA, x, ti.a_row, fb);
          tma_load_2d_pair(smem_u32(s.b[stage]), &tmB, x, ti.b_row + rank * half, fb);
          tma_load_2d_pair(smem_u32(s.sfa[stage]), &tmSFA, 0, ti.sfa0 + kb, fb);
          tma_load_2d_pair(smem_u32(s.sfb[stage]), &tmSFB, 0, 2 * (ti.sfb0 + kb), fb);
        }
        __syncwarp();
        armed |= 1u << stage;
        armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && rank == 0 && lane == 0) {  // unwinding: let the copies already counted here land
      for (int i = 0; i < kStages; ++i)
        if (armed & (1u << i)) mbar_drain(smem_u32(&s.full[i]), (armed_par >> i) & 1u, 20000000ull);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    // The whole warp runs the loop so descriptors and TMEM addresses are
    // warp-uniform; one elected lane issues the tcgen05 instructions (issuing
    // from a lone active lane costs about as much per MMA as the MMA itself).
    if (rank == 0) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0, sf_buf = 0;
      bool ok = true, issued = false;
      if (g.stall_test) ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.never), 0, wc));
      TileWalker<MODE> walk;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        const TileInfo ti = walk.at_warp(s, g, t, 0);
        if (ti.kb_count == 0) continue;
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&s.acc_empty[acc]), acc_phase ^ 1u, wc))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccStride;
        const uint32_t n_mma = uint32_t(ti.nlen + 15) & ~15u;
        const uint32_t idesc0 = make_idesc_mxf8(2 * kBM, n_mma);
        // k-steps go in pairs: both stages' scale factors are copied to TMEM
        // before the pair's MMAs, so the tensor pipe switches between copies
        // and MMAs once per two k-steps (a copy issued between MMAs costs
        // far more than its own duration; one pair group measured ~4% fewer
        // cycles than a copy group per k-step)
        for (int kb = 0; kb < ti.kb_count; kb += 2) {
          const bool two = kb + 1 < ti.kb_count;
          const uint32_t stage2 = stage + 1 == kStages ? 0u : stage + 1;
          const uint32_t phase2 = stage + 1 == kStages ? phase ^ 1u : phase;
          bool ready = mbar_wait(smem_u32(&s.full[stage]), phase, wc);
          if (ready && two) ready = mbar_wait(smem_u32(&s.full[stage2]), phase2, wc);
          if (!__all_sync(0xffffffffu, ready)) {
            ok = false;
            break;
          }
          tc_fence_after();
          auto step = [&](uint32_t stg, uint32_t buf, int kbi) {
            const uint32_t sfa_t = tmem_base + (buf ? kSfCol1 : kSfCol0);
            const uint32_t sfb_t = sfa_t + kSfbOff;
            const int rem = ti.klen - kbi * kBK;
            const int nk = rem >= kBK ? 4 : rem / 32;
            const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(s.a[stg]));
            const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(s.b[stg]));
            for (int kk = 0; kk < nk; ++kk) {
              tc_mma_mxf8_pair(d_tmem, adesc + uint64_t(2 * kk), bdesc + uint64_t(2 * kk),
                               idesc_with_sf_id(idesc0, kk, kk), sfa_t | (uint32_t(kk) << 30),
                               sfb_t | (uint32_t(kk) << 30), (kbi | kk) != 0 ? 1u : 0u);
            }
            tc_commit_pair_mc(smem_u32(&s.empty[stg]), 0x3);
          };
          auto copy_sf = [&](uint32_t stg, uint32_t buf) {
            const uint32_t sfa_t = tmem_base + (buf ? kSfCol1 : kSfCol0);
            const uint32_t sfb_t = sfa_t + kSfbOff;
            const uint32_t sfa_s = smem_u32(s.sfa[stg]), sfb_s = smem_u32(s.sfb[stg]);
            tc_cp_32x128b_warpx4_pair(sfa_t, sdesc_sf_chunk(sfa_s));
            tc_cp_32x128b_warpx4_pair(sfb_t, sdesc_sf_chunk(sfb_s));
            tc_cp_32x128b_warpx4_pair(sfb_t + 4, sdesc_sf_chunk(sfb_s + 512));
          };
          if (elect_one_sync()) {
            copy_sf(stage, sf_buf);
            if (two) copy_sf(stage2, sf_buf ^ 1u);
            step(stage, sf_buf, kb);
            if (two) step(stage2, sf_buf ^ 1u, kb + 1);
          }
          __syncwarp();
          issued = true;
          if (!two) sf_buf ^= 1u;
          const int adv = two ? 2 : 1;
          for (int i = 0; i < adv; ++i) {
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        if (!ok) break;
        if (elect_one_sync()) tc_commit_pair_mc(smem_u32(&s.acc_full[acc]), 0x3);
        __syncwarp();
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (issued) {  // every MMA done before TMEM is released
        if (elect_one_sync()) tc_commit_pair(smem_u32(&s.drain));
        __syncwarp();
        mbar_drain(smem_u32(&s.drain), 0, 50000000ull);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // TMEM loads are software-pipelined one 32-column chunk ahead; staged
    // chunks leave through TMA stores from two 2 KiB slots per warp, so the
    // next chunk is written while the previous store still reads its slot.
    // A warp reads TMEM lane quarter warp % 4 (the hardware's rule); with
    // eight epilogue warps, warps 0-3 take the first half of a tile's
    // 32-column chunks and warps 6-9 the second.
    const int qw = warp & 3;                       // TMEM lane quarter = rows qw*32 .. qw*32+31
    const int ew = warp < 4 ? warp : warp - 2;     // epilogue warp index (staging buffer)
    const int grp = warp < 4 ? 0 : 1;              // column half (eight epilogue warps)
    const int row = qw * 32 + lane;
    uint32_t acc = 0, acc_phase = 0;
    uint32_t slot = 0;         // staging slot (2 KiB half of s.epi[ew]) the next store uses
    bool epi_pending = false;  // a TMA store of this warp may still read its staging buffer
    uint8_t* const epi = s.epi[ew];
    // this warp's 32-column chunks [cb, ce) of a tile with nchunks chunks
    // (an even split point keeps the bf16 chunk pairs within one warp)
    auto chunk_range = [&](int nchunks, int& cb, int& ce) {
      cb = 0;
      ce = nchunks;
      if (kEpiWarps == 8) {
        const int h = min(nchunks, (((nchunks + 1) >> 1) + 1) & ~1);
        cb = grp ? h : 0;
        ce = grp ? nchunks : h;
      }
    };
    const bool f32 = g.out_dtype == MXG_DTYPE_F32;
    // free the slot about to be written: at most the other slot's store may still read
    auto slot_ready = [&]() {
      if (epi_pending) {
        if (lane == 0) bulk_wait_group_read1();
        __syncwarp();
      }
    };
    auto issue_store = [&](const CUtensorMap* tm, uint32_t src, int x, int y, int z, bool three_d) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (three_d) tma_store_3d(tm, src, x, y, z);
        else tma_store_2d(tm, src, x, y);
        bulk_commit_group();
      }
      epi_pending = true;
    };
    TileWalker<MODE> walk;
    for (int t = pair; t < num_tiles; t += npairs) {
      const TileInfo ti = walk.at(s, g, t, rank);
      if (ti.kb_count == 0) {  // empty group (wgrad): dW[e] = 0
        uint32_t z[32];
        int cb, ce;
        chunk_range((ti.nlen + 31) >> 5, cb, ce);
        for (int ci = cb; ci < ce; ++ci) store_chunk<MODE>(g, ti, row, 32 * ci, z, true);
        continue;
      }
      bool ok = mbar_wait(smem_u32(&s.acc_full[acc]), acc_phase, wc);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (uint32_t(qw * 32) << 16) + acc * kAccStride;
      const uint32_t acc_empty_leader = mapa_shared(smem_u32(&s.acc_empty[acc]), 0);
      auto release_acc = [&]() {  // accumulator fully read: let the next tile's MMAs start
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
      };
      auto emit = [&](int c0, const uint32_t (&v)[32]) {
        const int cols_here = min(32, ti.nlen - c0);
        if (MODE == MODE_FWD && g.scatter_bufs != nullptr) {
          // the [token][feature] staging of the bf16 path below, then every
          // lane reads one 16-byte piece (8 features) of a token row and
          // stores it straight into the row's home buffer: four lanes write
          // one token's 64 bytes, eight tokens per instruction.  The reads
          // are synchronous, so one 2 KiB slot suffices.
          const int f0 = ti.mb * kBM + qw * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            *reinterpret_cast<__nv_bfloat16*>(epi + j * 64 + (((lane >> 3) ^ ((j >> 1) & 3)) * 16) +
                                              (lane & 7) * 2) = __float2bfloat16_rn(__uint_as_float(v[j]));
          __syncwarp();
          const int p = lane & 3;
          const int f = f0 + 8 * p;
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int j = it * 8 + (lane >> 2);
            if (j < cols_here && f < g.n_out) {
              const int64_t q = int64_t(ti.b_row) + c0 + j;
              const int r = __ldg(g.back_rank + q);
              if (r >= 0) {
                const int64_t dr = __ldg(g.back_row + q);
                const uint4 piece = *reinterpret_cast<const uint4*>(epi + j * 64 + ((p ^ ((j >> 1) & 3)) * 16));
                if (r < g.scatter_nbufs && dr >= 0 && dr < g.scatter_rows)
                  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(g.scatter_bufs[r]) + dr * g.ldo + f) =
                      piece;
                else
                  atomicCAS(g.err, 0, MXG_ERR_WORKSPACE_TOO_SMALL);
              }
            }
          }
          __syncwarp();  // the slot is rewritten by the next chunk
        } else if (MODE == MODE_FWD && g.fwd_tma_store && (cols_here == 32 || cols_here == 16)) {
          // this warp holds 32 features (lanes) x 32 tokens (columns): stage it
          // transposed as [token][feature] and store whole token rows
          const int f0 = ti.mb * kBM + qw * 32;
          if (f32) {  // 32 tokens x 128 B, 128-byte swizzle: the whole 4 KiB buffer
            if (epi_pending) {
              if (lane == 0) bulk_wait_group_read0();
              __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < 32; ++j)
              *reinterpret_cast<uint32_t*>(epi + j * 128 + (((lane >> 2) ^ (j & 7)) * 16) +
                                           (lane & 3) * 4) = v[j];
            issue_store(cols_here == 32 ? &tmOut : &tmOut16, smem_u32(epi), f0, ti.b_row + c0, 0, false);
            slot = 0;
          } else {    // 32 tokens x 64 B, 64-byte swizzle: one 2 KiB slot
            slot_ready();
            uint8_t* buf = epi + slot * 2048;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              *reinterpret_cast<__nv_bfloat16*>(buf + j * 64 + (((lane >> 3) ^ ((j >> 1) & 3)) * 16) +
                                                (lane & 7) * 2) =
                  __float2bfloat16_rn(__uint_as_float(v[j]));
            issue_store(cols_here == 32 ? &tmOut : &tmOut16, smem_u32(buf), f0, ti.b_row + c0, 0, false);
            slot ^= 1u;
          }
        } else if (MODE == MODE_WGRAD && g.wgrad_tma_store && f32) {
          // row = lane; 32 fp32 columns (128 B rows, 128-byte swizzle) per
          // store from the warp's whole 4 KiB buffer, or 16 (64 B rows,
          // 64-byte swizzle) for the remainder of a 240-column tile; the
          // store clips at the tensor edge.  Half as many store requests as
          // 64-byte rows through two 2 KiB slots, which measured slower.
          const int r0 = ti.mb * kBM + qw * 32;
          if constexpr (Cfg<MODE>::kEpiBytes < 4096) {  // 2 KiB slot: 16 columns (64-byte rows) per store
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              if (16 * hh < cols_here) {
                if (epi_pending) {
                  if (lane == 0) bulk_wait_group_read0();
                  __syncwarp();
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
                  *reinterpret_cast<uint4*>(epi + lane * 64 + ((u ^ ((lane >> 1) & 3)) * 16)) =
                      make_uint4(v[16 * hh + 4 * u], v[16 * hh + 4 * u + 1], v[16 * hh + 4 * u + 2],
                                 v[16 * hh + 4 * u + 3]);
                issue_store(&tmOut16, smem_u32(epi), ti.n0 + c0 + 16 * hh, r0, ti.e, true);
              }
            }
            return;
          }
          if (epi_pending) {
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
          }
          if (cols_here == 32) {
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *reinterpret_cast<uint4*>(epi + lane * 128 + ((u ^ (lane & 7)) * 16)) =
                  make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
            issue_store(&tmOut, smem_u32(epi), ti.n0 + c0, r0, ti.e, true);
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<uint4*>(epi + lane * 64 + ((u ^ ((lane >> 1) & 3)) * 16)) =
                  make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
            issue_store(&tmOut16, smem_u32(epi), ti.n0 + c0, r0, ti.e, true);
          }
        } else if (MODE == MODE_WGRAD && g.wgrad_tma_store) {
          // bf16: row = lane.  Chunks pair up (columns [64j, 64j + 64) of the
          // tile) into 128-byte rows, 128-byte swizzle, one store from the
          // warp's whole 4 KiB buffer -- half the store requests of 64-byte
          // rows.  A chunk without a full partner (the tile's last 32 or 16
          // columns) leaves alone: 64-byte rows (64-byte swizzle) or 32-byte
          // rows (unswizzled); the tensor edge clips every store.
          const int r0 = ti.mb * kBM + qw * 32;
          const int pair0 = c0 & ~63;
          const bool paired = Cfg<MODE>::kEpiBytes >= 4096 && pair0 + 64 <= ti.nlen;
          auto pack8 = [&](int u) {
            return make_uint4(pack_bf16x2(__uint_as_float(v[8 * u]), __uint_as_float(v[8 * u + 1])),
                              pack_bf16x2(__uint_as_float(v[8 * u + 2]), __uint_as_float(v[8 * u + 3])),
                              pack_bf16x2(__uint_as_float(v[8 * u + 4]), __uint_as_float(v[8 * u + 5])),
                              pack_bf16x2(__uint_as_float(v[8 * u + 6]), __uint_as_float(v[8 * u + 7])));
          };
          if (paired) {
            const int hc = (c0 - pair0) >> 3;  // 16-byte chunk offset of this half (8 bf16 each): 0 or 4
            if (hc == 0 && epi_pending) {      // the previous store has read the buffer
              if (lane == 0) bulk_wait_group_read0();
              __syncwarp();
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<uint4*>(epi + lane * 128 + (((hc + u) ^ (lane & 7)) * 16)) = pack8(u);
            if (hc != 0) issue_store(&tmOut, smem_u32(epi), ti.n0 + pair0, r0, ti.e, true);
          } else {
            if (epi_pending) {
              if (lane == 0) bulk_wait_group_read0();
              __syncwarp();
            }
            if (cols_here == 32) {
#pragma unroll
              for (int u = 0; u < 4; ++u)
                *reinterpret_cast<uint4*>(epi + lane * 64 + ((u ^ ((lane >> 1) & 3)) * 16)) = pack8(u);
              issue_store(&tmOut16, smem_u32(epi), ti.n0 + c0, r0, ti.e, true);
            } else {
#pragma unroll
              for (int u = 0; u < 2; ++u) *reinterpret_cast<uint4*>(epi + lane * 32 + u * 16) = pack8(u);
              issue_store(&tmOutAux, smem_u32(epi), ti.n0 + c0, r0, ti.e, true);
            }
          }
        } else {
          store_chunk<MODE>(g, ti, row, c0, v, false);
        }
      };
      int cb, ce;
      chunk_range((ti.nlen + 31) >> 5, cb, ce);
      uint32_t va[32], vb[32];
      if (cb < ce) tmem_ld_32x32b_x32(tb + uint32_t(32 * cb), va);
      else release_acc();  // no columns for this warp in this tile
      for (int ci = cb; ci < ce; ci += 2) {
        tmem_ld_wait_regs(va);
        if (ci + 1 < ce) tmem_ld_32x32b_x32(tb + uint32_t(32 * (ci + 1)), vb);
        else release_acc();
        emit(32 * ci, va);
        if (ci + 1 < ce) {
          tmem_ld_wait_regs(vb);
          if (ci + 2 < ce) tmem_ld_32x32b_x32(tb + uint32_t(32 * (ci + 2)), va);
          else release_acc();
          emit(32 * (ci + 1), vb);
        }
      }
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (epi_pending && lane == 0) bulk_wait_group0();
    __syncwarp();
    if (MODE == MODE_FWD && g.scatter_bufs != nullptr) __threadfence_system();  // rows to peers
  }

  if (s.abort_flag) {  // unwinding: give copies issued by either CTA time to land
    const uint64_t until = globaltimer_ns() + 2000000ull;
    while (globaltimer_ns() < until) {
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer no longer touches this CTA's barriers or TMEM
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  cluster_sync_all();
}

// Forward: rows [meta[3], M) belong to no group -> write zeros.
__global__ void zero_tail_kernel(const int* meta, uint8_t* out, int64_t M, int64_t row_bytes) {
  const int64_t first = meta[3];
  if (first >= M) return;
  const int64_t beg = first * row_bytes, end = M * row_bytes;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = beg + (int64_t(blockIdx.x) * blockDim.x + threadIdx.x); i < end; i += stride)
    out[i] = 0;
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D uint8 operand [rows, cols] (cols contiguous), box {128 bytes, box_rows},
// 128-byte swizzle; out-of-range elements read as zero.
static int make_tmap(CUtensorMap* tm, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXG_ERR_CUDA;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols)};
  cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MXG_OK : MXG_ERR_CUDA;
}

// Packed scale chunks viewed as rows of 128 uint32 (512 bytes), box of
// `box_rows` rows, no swizzle.
// Forward output y [M, N] (bf16 or fp32), box {32 features, box_rows tokens};
// swizzle matches the staging layout (64-byte rows for bf16, 128 for fp32).
static int make_out_tmap_fwd(CUtensorMap* tm, void* base, int64_t M, int64_t N, int out_dtype,
                             int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXG_ERR_CUDA;
  const bool f32 = out_dtype == MXG_DTYPE_F32;
  const cuuint64_t esz = f32 ? 4 : 2;
  cuuint64_t dims[2] = {cuuint64_t(N), cuuint64_t(M)};
  cuuint64_t strides[1] = {cuuint64_t(N) * esz};
  cuuint32_t box[2] = {32, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MXG_OK : MXG_ERR_CUDA;
}

// dW [E, rows, cols] output, box {row_bytes of columns (64: 16 fp32 or 32
// bf16; 128: 32 fp32 or 64 bf16), 32 rows, 1}, swizzle of the same width
// (the epilogue's staging layout).
static int make_out_tmap_wgrad(CUtensorMap* tm, void* base, int64_t E, int64_t rows, int64_t cols,
                               int out_dtype, int row_bytes) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXG_ERR_CUDA;
  const bool f32 = out_dtype == MXG_DTYPE_F32;
  const cuuint64_t esz = f32 ? 4 : 2;
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(E)};
  cuuint64_t strides[2] = {cuuint64_t(cols) * esz, cuuint64_t(cols) * esz * cuuint64_t(rows)};
  cuuint32_t box[3] = {cuuint32_t(row_bytes / int(esz)), 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                   base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MXG_OK : MXG_ERR_CUDA;
}

// dW [E, rows, cols] bf16, box {16 cols (32 B), 32 rows, 1}, no swizzle.
static int make_out_tmap_wgrad16(CUtensorMap* tm, void* base, int64_t E, int64_t rows, int64_t cols) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXG_ERR_CUDA;
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(E)};
  cuuint64_t strides[2] = {cuuint64_t(cols) * 2, cuuint64_t(cols) * 2 * cuuint64_t(rows)};
  cuuint32_t box[3] = {16, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MXG_OK : MXG_ERR_CUDA;
}

static int make_sf_tmap(CUtensorMap* tm, const void* base, int64_t rows, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXG_ERR_CUDA;
  cuuint64_t dims[2] = {128, cuuint64_t(rows)};
  cuuint64_t strides[1] = {512};
  cuuint32_t box[2] = {128, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MXG_OK : MXG_ERR_CUDA;
}

struct WsLayout {
  size_t meta_off, sfa_off, sfb_off, total;
  int64_t sfa_chunks, sfb_chunks;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static WsLayout ws_layout(int mode, int E, int64_t M, int64_t n_out, int64_t n_ext, int64_t K) {
  const int64_t mb2 = 2 * ((n_out + 2 * kBM - 1) / (2 * kBM));  // A blocks, rounded to pairs
  int64_t asf, bsf;
  if (mode == MODE_FWD) {
    const int64_t kb = (K + kBK - 1) / kBK;
    asf = int64_t(E) * mb2 * kb;
    const int64_t bn = bn_max(MODE_FWD);
    bsf = kb * ((M + (bn - 1) * E) / bn + 1);
  } else {
    const int64_t kbs = (M + int64_t(kBK - 1) * E) / kBK + 1;
    const int64_t nt = (n_ext + bn_max(MODE_WGRAD) - 1) / bn_max(MODE_WGRAD);
    asf = mb2 * kbs;
    bsf = nt * kbs;
  }
  WsLayout w;
  w.sfa_chunks = asf;
  w.sfb_chunks = bsf;
  w.meta_off = 0;
  w.sfa_off = align_up(MetaView::words(E) * 4, 1024);
  w.sfb_off = align_up(w.sfa_off + size_t(asf) * kSfaBytes, 1024);
  w.total = align_up(w.sfb_off + size_t(bsf) * kSfbBytes, 1024);
  return w;
}

// Kernel attributes of one mode and the number of its CTA pairs that fit at once.
template <int MODE>
static int configure_mode(int* pairs) {
  const size_t smem = smem_bytes<MODE>();
  if (cudaFuncSetAttribute(grouped_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(smem)) != cudaSuccess)
    return MXG_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * 74, 1, 1);
  cfg.blockDim = dim3(Cfg<MODE>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, grouped_gemm_kernel<MODE>, &cfg) != cudaSuccess || n < 1)
    return MXG_ERR_CUDA;
  *pairs = n;
  return MXG_OK;
}

// Per device and mode: the CTA pairs of a persistent launch (set up once).
static int configure_kernels(int mode, int* pairs) {
  static std::mutex mu;
  static int cached_pairs[64][2] = {{0}};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MXG_ERR_CUDA;
  std::lock_guard<std::mutex> lk(mu);
  if (cached_pairs[dev][0] == 0) {
    int st = configure_mode<MODE_FWD>(&cached_pairs[dev][0]);
    if (st == MXG_OK) st = configure_mode<MODE_WGRAD>(&cached_pairs[dev][1]);
    if (st != MXG_OK) {
      cached_pairs[dev][0] = 0;
      return st;
    }
  }
  *pairs = cached_pairs[dev][mode == MODE_WGRAD ? 1 : 0];
  return MXG_OK;
}


// Host launch is split in two halves that share the workspace:
//   prepare: group scheduler + scale-factor packing (reads offs and scales)
//   run:     the tcgen05 GEMM kernel (reads the e4m3 operands)
// A operand: rows of [a_rows, kc] e4m3; B operand: rows of [b_rows, kc] e4m3.
struct Problem {
  int mode;
  int E;
  int64_t M;      // rows covered by offs (forward: tokens; wgrad: tokens)
  int64_t n_out;  // A rows per group
  int64_t n_ext;  // wgrad: B rows
  int64_t kc;     // contraction length (forward K; wgrad M)
};

static int prepare_grouped(const Problem& P, const void* a_sc, const void* b_sc,
                           const int32_t* offs, int offs_len, int offs_kind, void* ws,
                           size_t ws_bytes, cudaStream_t stream) {
  const WsLayout L = ws_layout(P.mode, P.E, P.M, P.n_out, P.n_ext, P.kc);
  if (ws_bytes < L.total) return MXG_ERR_WORKSPACE_TOO_SMALL;
  int st = check_device();
  if (st) return st;
  uint8_t* wsb = reinterpret_cast<uint8_t*>(ws);
  int* meta = reinterpret_cast<int*>(wsb + L.meta_off);
  int* err = device_error_word();
  if (!err) return MXG_ERR_CUDA;
  SchedArgs sa{offs, offs_len, offs_kind, P.E, int(P.M), P.mode, int(P.n_out), int(P.n_ext),
               int(P.kc), meta, err};
  schedule_kernel<<<1, MXG_MAX_GROUPS, 0, stream>>>(sa);
  const int sms = num_sms();
  PackArgs pa{meta, P.E, P.mode, 0, reinterpret_cast<const uint8_t*>(a_sc), P.kc / 32,
              wsb + L.sfa_off, int(P.n_out), int(P.n_ext), int(P.kc)};
  // A side: E * 2 * mbp units of 128 rows; B side: one unit per N tile (the
  // count is only known on the device: grid-stride over a generous grid)
  const int mbp = int((P.n_out + 2 * kBM - 1) / (2 * kBM));
  const int a_units = P.E * 2 * mbp;
  PackArgs pb = pa;
  pb.side = 1;
  pb.src = reinterpret_cast<const uint8_t*>(b_sc);
  pb.dst = wsb + L.sfb_off;
  if (P.mode == MODE_FWD) {  // K/32-byte scale rows: word-aligned row walks
    // 256 threads per unit: 8 k-split groups of a 128-row A unit, 4 of a
    // 256-row B unit
    const int ga = std::max(1, std::min(a_units, sms * 16));
    pack_scales_kernel<<<ga + sms * 8, 256, 0, stream>>>(PackPair{{pa, pb}, ga});
  } else {
    // about one chunk half per warp (the chunk counts are bounded by the
    // workspace layout), so each warp's loads go out in one round
    const int64_t cap = int64_t(sms) * 64;
    const int ga = int(std::max<int64_t>(1, std::min(cap, (L.sfa_chunks + 7) / 8)));
    const int gb = int(std::max<int64_t>(1, std::min(cap, (2 * L.sfb_chunks + 7) / 8)));
    pack_scales_chunk_kernel<<<ga + gb, 256, 0, stream>>>(PackPair{{pa, pb}, ga});
  }
  return cuda_status(cudaGetLastError());
}

// Destinations of a forward in scatter mode (see GemmArgs); null: write `out`.
struct Scatter {
  const uint64_t* bufs;
  int nbufs;
  const int32_t* back_rank;
  const int32_t* back_row;
  int64_t rows;
};

static int run_grouped(const Problem& P, const void* a_ptr, int64_t a_rows, const void* b_ptr,
                       int64_t b_rows, void* out, int out_dtype, int64_t ldo, void* ws,
                       size_t ws_bytes, cudaStream_t stream, const Scatter* scatter = nullptr) {
  const WsLayout L = ws_layout(P.mode, P.E, P.M, P.n_out, P.n_ext, P.kc);
  if (ws_bytes < L.total) return MXG_ERR_WORKSPACE_TOO_SMALL;
  int st = check_device();
  if (st) return st;
  int pairs = 0;
  st = configure_kernels(P.mode, &pairs);
  if (st) return st;
  const int limit = gemm_sm_limit();  // leave SMs to concurrent kernels (peer exchanges)
  if (limit > 0) pairs = std::max(1, std::min(pairs, limit / 2));
  uint8_t* wsb = reinterpret_cast<uint8_t*>(ws);
  int* meta = reinterpret_cast<int*>(wsb + L.meta_off);
  int* err = device_error_word();
  if (!err) return MXG_ERR_CUDA;
  CUtensorMap tmA, tmB, tmSFA, tmSFB;
  st = make_tmap(&tmA, a_ptr, a_rows, P.kc, kBM);
  if (st) return st;
  st = make_tmap(&tmB, b_ptr, b_rows, P.kc,
                 P.mode == MODE_FWD ? Cfg<MODE_FWD>::kBHalf : Cfg<MODE_WGRAD>::kBHalf);
  if (st) return st;
  st = make_sf_tmap(&tmSFA, wsb + L.sfa_off, std::max<int64_t>(L.sfa_chunks, 1), 1);
  if (st) return st;
  st = make_sf_tmap(&tmSFB, wsb + L.sfb_off, std::max<int64_t>(2 * L.sfb_chunks, 2), 2);
  if (st) return st;
  CUtensorMap tmOut = tmA, tmOut16 = tmA, tmOutAux = tmA;  // epilogue store maps (unused: dummies)
  const int64_t out_esz = out_dtype == MXG_DTYPE_F32 ? 4 : 2;
  // TMA stores need the output row stride to be a multiple of 16 bytes
  const bool wgrad_tma = P.mode == MODE_WGRAD && (P.n_ext * out_esz) % 16 == 0;
  if (wgrad_tma) {
    if (out_dtype == MXG_DTYPE_F32) {  // 32-column stores, 16-column remainders
      st = make_out_tmap_wgrad(&tmOut, out, P.E, P.n_out, P.n_ext, out_dtype, 128);
      if (st) return st;
      st = make_out_tmap_wgrad(&tmOut16, out, P.E, P.n_out, P.n_ext, out_dtype, 64);
      if (st) return st;
    } else {  // 64-column stores, 32- and 16-column remainders of bf16 tiles
      st = make_out_tmap_wgrad(&tmOut, out, P.E, P.n_out, P.n_ext, out_dtype, 128);
      if (st) return st;
      st = make_out_tmap_wgrad(&tmOut16, out, P.E, P.n_out, P.n_ext, out_dtype, 64);
      if (st) return st;
      st = make_out_tmap_wgrad16(&tmOutAux, out, P.E, P.n_out, P.n_ext);
      if (st) return st;
    }
  }
  // TMA stores need the output row stride (N elements) to be a multiple of 16 bytes
  const bool fwd_tma = P.mode == MODE_FWD && scatter == nullptr &&
                       (P.n_out * (out_dtype == MXG_DTYPE_F32 ? 4 : 2)) % 16 == 0;
  if (fwd_tma) {
    st = make_out_tmap_fwd(&tmOut, out, P.M, P.n_out, out_dtype, 32);
    if (st) return st;
    st = make_out_tmap_fwd(&tmOut16, out, P.M, P.n_out, out_dtype, 16);
    if (st) return st;
  }
  GemmArgs ga;
  ga.meta = meta;
  ga.out = out;
  ga.out_dtype = out_dtype;
  ga.E = P.E;
  ga.n_out = int(P.n_out);
  ga.n_ext = int(P.n_ext);
  ga.k_fwd = int(P.kc);
  ga.ldo = ldo;
  ga.err = err;
  const int64_t stall = take_injected_stall();
  ga.timeout_ns = stall > 0 ? uint64_t(stall) : kWaitLimitNs;
  ga.stall_test = stall > 0 ? 1 : 0;
  ga.fwd_tma_store = fwd_tma ? 1 : 0;
  ga.wgrad_tma_store = wgrad_tma ? 1 : 0;
  ga.scatter_bufs = scatter ? scatter->bufs : nullptr;
  ga.back_rank = scatter ? scatter->back_rank : nullptr;
  ga.back_row = scatter ? scatter->back_row : nullptr;
  ga.scatter_nbufs = scatter ? scatter->nbufs : 0;
  ga.scatter_rows = scatter ? scatter->rows : 0;

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(unsigned(2 * pairs), 1, 1);
  cfg.blockDim = dim3(unsigned(P.mode == MODE_FWD ? Cfg<MODE_FWD>::kThreads : Cfg<MODE_WGRAD>::kThreads), 1, 1);
  cfg.dynamicSmemBytes = P.mode == MODE_FWD ? smem_bytes<MODE_FWD>() : smem_bytes<MODE_WGRAD>();
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (P.mode == MODE_FWD) {
    e = cudaLaunchKernelEx(&cfg, grouped_gemm_kernel<MODE_FWD>, tmA, tmB, tmSFA, tmSFB, tmOut, tmOut16, tmOutAux, ga);
    if (e == cudaSuccess && scatter == nullptr) {
      const int64_t row_bytes = P.n_out * (out_dtype == MXG_DTYPE_F32 ? 4 : 2);
      zero_tail_kernel<<<num_sms(), 256, 0, stream>>>(meta, reinterpret_cast<uint8_t*>(out), P.M,
                                                      row_bytes);
      e = cudaGetLastError();
    }
  } else {
    e = cudaLaunchKernelEx(&cfg, grouped_gemm_kernel<MODE_WGRAD>, tmA, tmB, tmSFA, tmSFB, tmOut, tmOut16, tmOutAux, ga);
  }
  return cuda_status(e);
}

}  // namespace mxg

using namespace mxg;

extern "C" size_t mxg_grouped_fwd_workspace_size(int num_groups, int64_t m, int64_t n, int64_t k) {
  if (num_groups < 1 || m < 0 || n < 0 || k < 0) return 0;
  return ws_layout(MODE_FWD, num_groups, m, n, 0, k).total;
}

extern "C" size_t mxg_grouped_wgrad_workspace_size(int num_groups, int64_t m, int64_t n,
                                                   int64_t k) {
  if (num_groups < 1 || m < 0 || n < 0 || k < 0) return 0;
  return ws_layout(MODE_WGRAD, num_groups, m, n, k, m).total;
}

// Stand-in offs pointer for validating run() arguments; never dereferenced.
static const int32_t* const kOffsGivenToPrepare = reinterpret_cast<const int32_t*>(uintptr_t(16));

static int check_common(int num_groups, int64_t m, int64_t n, int64_t k, int out_dtype,
                        const int32_t* offs, int offs_len, int offs_kind) {
  if (num_groups < 1) return MXG_ERR_INVALID_ARGUMENT;
  if (num_groups > MXG_MAX_GROUPS) return MXG_ERR_TOO_MANY_GROUPS;
  if (m < 0 || n < 1 || k < 1) return MXG_ERR_BAD_SHAPE;
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return MXG_ERR_BAD_SHAPE;
  if (out_dtype != MXG_DTYPE_BF16 && out_dtype != MXG_DTYPE_F32) return MXG_ERR_INVALID_ARGUMENT;
  if (offs == nullptr) {
    if (num_groups != 1) return MXG_ERR_INVALID_ARGUMENT;
  } else {
    if (offs_kind < MXG_OFFS_LEADING_ZERO || offs_kind > MXG_OFFS_AUTO) return MXG_ERR_INVALID_ARGUMENT;
    const int need = offs_kind == MXG_OFFS_LEADING_ZERO ? num_groups + 1 : num_groups;
    if (offs_kind == MXG_OFFS_AUTO) {
      if (offs_len != num_groups && offs_len != num_groups + 1) return MXG_ERR_INVALID_ARGUMENT;
    } else if (offs_len != need) {
      return MXG_ERR_INVALID_ARGUMENT;
    }
  }
  return MXG_OK;
}

extern "C" int mxg_grouped_fwd(const void* a, const void* a_scales, const void* w,
                               const void* w_scales, const int32_t* offs, int offs_len,
                               int offs_kind, int num_groups, int64_t m, int64_t n, int64_t k,
                               void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                               void* stream) {
  int st = check_common(num_groups, m, n, k, out_dtype, offs, offs_len, offs_kind);
  if (st) return st;
  if (k % 32 != 0) return MXG_ERR_BAD_SHAPE;
  if (m == 0) return MXG_OK;
  if (!a || !w || !out || !workspace) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(a) || !aligned16(w) || !aligned16(out) || !aligned16(workspace))
    return MXG_ERR_MISALIGNED;
  if (int64_t(num_groups) * n > INT32_MAX) return MXG_ERR_BAD_SHAPE;
  const Problem P{MODE_FWD, num_groups, m, n, 0, k};
  st = prepare_grouped(P, w_scales, a_scales, offs, offs_len, offs_kind, workspace,
                       workspace_bytes, (cudaStream_t)stream);
  if (st) return st;
  return run_grouped(P, w, int64_t(num_groups) * n, a, m, out, out_dtype, n, workspace,
                     workspace_bytes, (cudaStream_t)stream);
}

extern "C" int mxg_grouped_fwd_prepare(const void* a_scales, const void* w_scales,
                                       const int32_t* offs, int offs_len, int offs_kind,
                                       int num_groups, int64_t m, int64_t n, int64_t k,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_common(num_groups, m, n, k, MXG_DTYPE_BF16, offs, offs_len, offs_kind);
  if (st) return st;
  if (k % 32 != 0) return MXG_ERR_BAD_SHAPE;
  if (!workspace) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(workspace)) return MXG_ERR_MISALIGNED;
  if (m == 0) return MXG_OK;
  if (int64_t(num_groups) * n > INT32_MAX) return MXG_ERR_BAD_SHAPE;
  const Problem P{MODE_FWD, num_groups, m, n, 0, k};
  return prepare_grouped(P, w_scales, a_scales, offs, offs_len, offs_kind, workspace,
                         workspace_bytes, (cudaStream_t)stream);
}

extern "C" int mxg_grouped_fwd_run(const void* a, const void* w, int num_groups, int64_t m,
                                   int64_t n, int64_t k, void* out, int out_dtype,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  // offs were captured by prepare; validate the rest as if they were present
  int st = check_common(num_groups, m, n, k, out_dtype, kOffsGivenToPrepare, num_groups,
                        MXG_OFFS_SIZES);
  if (st) return st;
  if (k % 32 != 0) return MXG_ERR_BAD_SHAPE;
  if (m == 0) return MXG_OK;
  if (!a || !w || !out || !workspace) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(a) || !aligned16(w) || !aligned16(out) || !aligned16(workspace))
    return MXG_ERR_MISALIGNED;
  if (int64_t(num_groups) * n > INT32_MAX) return MXG_ERR_BAD_SHAPE;
  const Problem P{MODE_FWD, num_groups, m, n, 0, k};
  return run_grouped(P, w, int64_t(num_groups) * n, a, m, out, out_dtype, n, workspace,
                     workspace_bytes, (cudaStream_t)stream);
}

extern "C" int mxg_grouped_fwd_run_scatter(const void* a, const void* w, int num_groups, int64_t m,
                                           int64_t n, int64_t k, const uint64_t* dst_bufs, int n_dst,
                                           const int32_t* back_rank, const int32_t* back_row,
                                           int64_t dst_rows, void* workspace, size_t workspace_bytes,
                                           void* stream) {
  int st = check_common(num_groups, m, n, k, MXG_DTYPE_BF16, kOffsGivenToPrepare, num_groups,
                        MXG_OFFS_SIZES);
  if (st) return st;
  if (k % 32 != 0 || n % 8 != 0) return MXG_ERR_BAD_SHAPE;
  if (n_dst < 1 || dst_rows < 0) return MXG_ERR_INVALID_ARGUMENT;
  if (m == 0) return MXG_OK;
  if (!a || !w || !workspace || !dst_bufs || !back_rank || !back_row) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(a) || !aligned16(w) || !aligned16(workspace)) return MXG_ERR_MISALIGNED;
  if (int64_t(num_groups) * n > INT32_MAX) return MXG_ERR_BAD_SHAPE;
  const Problem P{MODE_FWD, num_groups, m, n, 0, k};
  const Scatter sc{dst_bufs, n_dst, back_rank, back_row, dst_rows};
  return run_grouped(P, w, int64_t(num_groups) * n, a, m, nullptr, MXG_DTYPE_BF16, n, workspace,
                     workspace_bytes, (cudaStream_t)stream, &sc);
}

extern "C" int mxg_grouped_wgrad(const void* go, const void* go_scales, const void* ia,
                                 const void* ia_scales, const int32_t* offs, int offs_len,
                                 int offs_kind, int num_groups, int64_t m, int64_t n, int64_t k,
                                 void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  int st = check_common(num_groups, m, n, k, out_dtype, offs, offs_len, offs_kind);
  if (st) return st;
  if (m % 32 != 0 || k % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (!go || !ia || !out || !workspace) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(go) || !aligned16(ia) || !aligned16(out) || !aligned16(workspace))
    return MXG_ERR_MISALIGNED;
  if (m == 0) {  // no tokens: every dW[e] is zero
    const size_t bytes = size_t(num_groups) * n * k * (out_dtype == MXG_DTYPE_F32 ? 4 : 2);
    return cuda_status(cudaMemsetAsync(out, 0, bytes, (cudaStream_t)stream));
  }
  const Problem P{MODE_WGRAD, num_groups, m, n, k, m};
  st = prepare_grouped(P, go_scales, ia_scales, offs, offs_len, offs_kind, workspace,
                       workspace_bytes, (cudaStream_t)stream);
  if (st) return st;
  return run_grouped(P, go, n, ia, k, out, out_dtype, k, workspace, workspace_bytes,
                     (cudaStream_t)stream);
}

extern "C" int mxg_grouped_wgrad_prepare(const void* go_scales, const void* ia_scales,
                                         const int32_t* offs, int offs_len, int offs_kind,
                                         int num_groups, int64_t m, int64_t n, int64_t k,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_common(num_groups, m, n, k, MXG_DTYPE_BF16, offs, offs_len, offs_kind);
  if (st) return st;
  if (m % 32 != 0 || k % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (!workspace) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(workspace)) return MXG_ERR_MISALIGNED;
  if (m == 0) return MXG_OK;
  const Problem P{MODE_WGRAD, num_groups, m, n, k, m};
  return prepare_grouped(P, go_scales, ia_scales, offs, offs_len, offs_kind, workspace,
                         workspace_bytes, (cudaStream_t)stream);
}

extern "C" int mxg_grouped_wgrad_run(const void* go, const void* ia, int num_groups, int64_t m,
                                     int64_t n, int64_t k, void* out, int out_dtype,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  // offs were captured by prepare; validate the rest as if they were present
  int st = check_common(num_groups, m, n, k, out_dtype, kOffsGivenToPrepare, num_groups,
                        MXG_OFFS_SIZES);
  if (st) return st;
  if (m % 32 != 0 || k % 16 != 0) return MXG_ERR_BAD_SHAPE;
  if (!go || !ia || !out || !workspace) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(go) || !aligned16(ia) || !aligned16(out) || !aligned16(workspace))
    return MXG_ERR_MISALIGNED;
  if (m == 0) {
    const size_t bytes = size_t(num_groups) * n * k * (out_dtype == MXG_DTYPE_F32 ? 4 : 2);
    return cuda_status(cudaMemsetAsync(out, 0, bytes, (cudaStream_t)stream));
  }
  const Problem P{MODE_WGRAD, num_groups, m, n, k, m};
  return run_grouped(P, go, n, ia, k, out, out_dtype, k, workspace, workspace_bytes,
                     (cudaStream_t)stream);
}

extern "C" size_t mxg_dense_fwd_kn_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0) return 0;
  return align_up(size_t(n) * size_t(k), 1024) + ws_layout(MODE_FWD, 1, m, n, 0, k).total;
}

extern "C" int mxg_dense_fwd_kn(const void* x, const void* w_kn, int64_t m, int64_t n, int64_t k,
                                void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                                void* stream) {
  int st = check_common(1, m, n, k, out_dtype, nullptr, 0, 0);
  if (st) return st;
  if (k % 32 != 0) return MXG_ERR_BAD_SHAPE;
  if (m == 0) return MXG_OK;
  if (!x || !w_kn || !out || !workspace) return MXG_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(out) || !aligned16(workspace)) return MXG_ERR_MISALIGNED;
  if (workspace_bytes < mxg_dense_fwd_kn_workspace_size(m, n, k))
    return MXG_ERR_WORKSPACE_TOO_SMALL;
  // W [k, n] -> W^T [n, k] (K-contiguous rows for the MMA), then one group.
  uint8_t* wt = reinterpret_cast<uint8_t*>(workspace);
  const size_t wt_bytes = align_up(size_t(n) * size_t(k), 1024);
  st = mxg_transpose_u8(w_kn, k, n, wt, stream);
  if (st) return st;
  const Problem P{MODE_FWD, 1, m, n, 0, k};
  st = prepare_grouped(P, nullptr, nullptr, nullptr, 0, 0, wt + wt_bytes,
                       workspace_bytes - wt_bytes, (cudaStream_t)stream);
  if (st) return st;
  return run_grouped(P, wt, n, x, m, out, out_dtype, n, wt + wt_bytes, workspace_bytes - wt_bytes,
                     (cudaStream_t)stream);
}

// ---------------------------------------------------------------- no-allocation variant
// Some callers cannot allocate device memory themselves: plugins hosted by a
// framework that owns the whole device memory pool, or host code that must
// not call cudaMalloc (it may synchronise the device).  For them the grouped
// forward can run on a scratch area built into this library: a fixed device
// array in this file, one copy on every GPU that loads the library, held
// until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(MXG_NOALLOC_SCRATCH_BYTES);
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a stand-in, so the address is looked up once per
// device (with that device current) and cached.
static void* noalloc_scratch(int* status) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = MXG_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = MXG_ERR_CUDA;
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

extern "C" int mxg_grouped_fwd_noalloc(const void* a, const void* a_scales, const void* w,
                                       const void* w_scales, const int32_t* offs, int offs_len,
                                       int offs_kind, int num_groups, int64_t m, int64_t n,
                                       int64_t k, void* out, int out_dtype, void* stream) {
  const size_t need = mxg_grouped_fwd_workspace_size(num_groups, m, n, k);
  if (need > kNoAllocScratchBytes) return MXG_ERR_WORKSPACE_TOO_SMALL;
  int st = MXG_OK;
  void* scratch = noalloc_scratch(&st);
  if (scratch == nullptr) return st;
  return mxg_grouped_fwd(a, a_scales, w, w_scales, offs, offs_len, offs_kind, num_groups, m, n, k,
                         out, out_dtype, scratch, kNoAllocScratchBytes, stream);
}
