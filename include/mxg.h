/*
 * mxg — B200-native (sm_100a) MXFP8 grouped GEMM: C ABI.
 *
 * Plain pointers, sizes and a CUDA stream (passed as void*) only; no torch
 * types.  Every entry point is asynchronous on the given stream, returns 0 on
 * success and a non-zero MXG_ERR_* code on a host-side validation or CUDA
 * launch error.  Errors found on the device (inconsistent group offsets, a
 * bounded wait that gave up) are recorded in a per-device error word read by
 * mxg_get_device_error().  No entry point allocates memory: the caller passes
 * a workspace whose size the *_workspace_size() functions return.
 *
 * Operand conventions (bytes are raw OCP MX formats):
 *   e4m3  = float8_e4m3fn codes (uint8), e8m0 = biased power-of-two scale
 *   (uint8, value 2^(b-127)); one scale per 32 consecutive elements along the
 *   contraction dimension, stored row-major [rows, cols/32].  A null scale
 *   pointer means unit scales (byte 0x7F).
 *
 * Reference interfaces replaced (indianspeedster/mxfp8-grouped-gemm):
 *   mxg_grouped_fwd    <- fused_fwd.py:172-230   fused_grouped_fwd()
 *   mxg_dense_fwd_kn   <- fwd_final.py:121-131   fwd_ge()
 *   mxg_grouped_wgrad  <- wgrad_fused.py:34-112  wgrad_fused()/wgrad_kernel()
 *   mxg_quantize_*     <- torchao triton_to_mxfp8_dim0/dim1 (mxfp8_rceil recipe),
 *                         called by the reference's MoE path (port_mxfp8.py:43-49,207-212)
 */
#ifndef MXG_H_
#define MXG_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MXG_API __attribute__((visibility("default")))
#else
#define MXG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define MXG_OK 0
#define MXG_ERR_INVALID_ARGUMENT 1    /* null pointer, negative size, bad enum */
#define MXG_ERR_BAD_SHAPE 2           /* dims not multiples of 32, too large    */
#define MXG_ERR_MISALIGNED 3          /* base pointer not 16-byte aligned       */
#define MXG_ERR_WORKSPACE_TOO_SMALL 4
#define MXG_ERR_CUDA 5                /* a CUDA runtime/driver call failed      */
#define MXG_ERR_DEVICE_TIMEOUT 6      /* a device-side bounded wait gave up     */
#define MXG_ERR_BAD_OFFSETS 7         /* group offsets inconsistent (device)    */
#define MXG_ERR_UNSUPPORTED_DEVICE 8  /* not an sm_100 (B200-class) GPU          */
#define MXG_ERR_TOO_MANY_GROUPS 9

/* ---- group-offset conventions (the reference uses all three) ------------ */
#define MXG_OFFS_LEADING_ZERO 0 /* [E+1], offs[0]==0, group e = [offs[e], offs[e+1])   fused_fwd.py:7 */
#define MXG_OFFS_CUMULATIVE 1   /* [E],   group e = [offs[e-1], offs[e])                fwd_final.py:170 */
#define MXG_OFFS_SIZES 2        /* [E],   group e has offs[e] rows                      wgrad_fused.py:37 */
#define MXG_OFFS_AUTO 3         /* [E+1] -> leading zero; [E] -> cumulative when
                                   non-decreasing with last == M, sizes when they
                                   sum to M, else MXG_ERR_BAD_OFFSETS (device)       */

#define MXG_DTYPE_BF16 0
#define MXG_DTYPE_F32 1

#define MXG_MAX_GROUPS 256

/* Human-readable text for a status code (static storage). */
MXG_API const char* mxg_error_string(int code);

/* Library version, major*10000 + minor*100 + patch. */
MXG_API int mxg_version(void);

/* Read (and optionally clear) the current device's error word.  Synchronises
 * the device.  *code receives 0 or the first MXG_ERR_* a kernel recorded.
 * The library looks up each device's error word once and keeps the address
 * for the life of the process, so cudaDeviceReset() on a device it has used
 * is not supported. */
MXG_API int mxg_get_device_error(int* code, int clear);

/* ---- MXFP8 quantisers (RCEIL E8M0 scales, RNE e4m3, saturating) ------------
 * Row-wise 1x32: x [rows, cols] bf16 -> q [rows, cols] e4m3, scales [rows, cols/32].
 * cols % 32 == 0.  Replaces torchao triton_to_mxfp8_dim0 (reference MoE forward
 * operands, memory/2026-06-09.md:10,20). */
MXG_API int mxg_quantize_rowwise(const void* x_bf16, int64_t rows, int64_t cols, void* q_e4m3,
                         void* scales_e8m0, void* stream);

/* Column-wise 32x1 with transposed output: x [rows, cols] bf16 ->
 * qt [cols, rows] e4m3, scales_t [cols, rows/32].  rows % 32 == 0, cols even.
 * Produces the token-contiguous wgrad operands go (N, M) / ia (K, M) of
 * wgrad_fused.py:35-39; replaces torchao triton_to_mxfp8_dim1. */
MXG_API int mxg_quantize_colwise(const void* x_bf16, int64_t rows, int64_t cols, void* qt_e4m3,
                         void* scales_t_e8m0, void* stream);

/* ---- grouped forward: y[rows of e] = x[rows of e] . W[e]^T -----------------
 * a [m, k] e4m3, a_scales [m, k/32]; w [num_groups, n, k] e4m3,
 * w_scales [num_groups, n, k/32]; offs int32 device array (see MXG_OFFS_*; may
 * be null when num_groups == 1, meaning one group of all m rows); out [m, n]
 * bf16 or f32.  Rows of out outside every group are written as zero.
 * k % 32 == 0, num_groups <= MXG_MAX_GROUPS.
 * Replaces fused_fwd.py:172-230 fused_grouped_fwd (which assumed equal
 * groups, fused_fwd.py:48; here groups may be any size, including empty). */
MXG_API size_t mxg_grouped_fwd_workspace_size(int num_groups, int64_t m, int64_t n, int64_t k);
MXG_API int mxg_grouped_fwd(const void* a, const void* a_scales, const void* w, const void* w_scales,
                    const int32_t* offs, int offs_len, int offs_kind, int num_groups, int64_t m,
                    int64_t n, int64_t k, void* out, int out_dtype, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Two-phase form of mxg_grouped_fwd (same workspace, same stream order):
 * prepare reads offs and the scales (group scheduler + scale-factor packing
 * into the workspace), run launches the tensor-core kernel on the e4m3
 * operands with the groups and scales captured by the last prepare on that
 * workspace.  prepare + run == mxg_grouped_fwd. */
MXG_API int mxg_grouped_fwd_prepare(const void* a_scales, const void* w_scales, const int32_t* offs,
                                    int offs_len, int offs_kind, int num_groups, int64_t m,
                                    int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                                    void* stream);
MXG_API int mxg_grouped_fwd_run(const void* a, const void* w, int num_groups, int64_t m, int64_t n,
                                int64_t k, void* out, int out_dtype, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Run half of the grouped forward (after mxg_grouped_fwd_prepare) whose bf16
 * output rows leave for other buffers instead of `out`: row q goes to row
 * back_row[q] of dst_bufs[back_rank[q]] (dst_bufs: device array of n_dst
 * buffer addresses, this GPU's or peers' -- mxg_peer_open; back_rank[q] < 0
 * drops the row), row stride n elements.  This is the expert-parallel
 * combine's return written from the epilogue of the GEMM that produces the
 * rows, by plain stores, so the exchange overlaps the tensor-core work (the
 * reference returns rows with a separate all-to-all after the GEMM,
 * port_mxfp8.py:74,240).  n % 8 == 0; buffers 16-byte aligned; a
 * destination row outside [0, dst_rows) is skipped and sets the device error
 * word.  The caller orders the ranks around it as around mxg_ep_return_p2p. */
MXG_API int mxg_grouped_fwd_run_scatter(const void* a, const void* w, int num_groups, int64_t m,
                                        int64_t n, int64_t k, const uint64_t* dst_bufs, int n_dst,
                                        const int32_t* back_rank, const int32_t* back_row,
                                        int64_t dst_rows, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* Grouped forward for callers that cannot allocate device memory (a plugin
 * inside a framework that owns the device memory pool, or host code that must
 * not call cudaMalloc): same arguments and result as mxg_grouped_fwd, minus
 * the workspace.  No counterpart in the reference.  Its scratch is a fixed
 * array of MXG_NOALLOC_SCRATCH_BYTES inside this library, present on every GPU
 * that loads the library until the process exits; problems whose
 * mxg_grouped_fwd_workspace_size() exceeds it return
 * MXG_ERR_WORKSPACE_TOO_SMALL.  The first call on a device looks up that
 * array's device address (make it before any stream capture).  All calls on
 * a device share the one array: calls that overlap on the GPU (different
 * streams, or different host threads) race; run them in order on one stream.
 * Nothing in the array needs to start zeroed: each call rewrites what it reads.
 * It calls no cudaMalloc/cudaFree.  The looked-up address (like the error
 * word's) is kept for the life of the process: cudaDeviceReset() on a device
 * this library has used is not supported. */
#define MXG_NOALLOC_SCRATCH_BYTES (64u << 20)
MXG_API int mxg_grouped_fwd_noalloc(const void* a, const void* a_scales, const void* w,
                                    const void* w_scales, const int32_t* offs, int offs_len,
                                    int offs_kind, int num_groups, int64_t m, int64_t n, int64_t k,
                                    void* out, int out_dtype, void* stream);

/* ---- dense forward with a K x N weight: out[m, n] = x[m, k] . w[k, n] -------
 * Unit scales (the reference's fwd_ge passes none, fwd_final.py:101-106).
 * Replaces fwd_final.py:121-131 fwd_ge. */
MXG_API size_t mxg_dense_fwd_kn_workspace_size(int64_t m, int64_t n, int64_t k);
MXG_API int mxg_dense_fwd_kn(const void* x, const void* w_kn, int64_t m, int64_t n, int64_t k, void* out,
                     int out_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ---- grouped weight gradient: dW[e] = go[:, tokens of e] . ia[:, tokens of e]^T
 * go [n, m] e4m3 (token-contiguous), go_scales [n, m/32]; ia [k, m] e4m3,
 * ia_scales [k, m/32]; out [num_groups, n, k] bf16 or f32 (empty groups -> 0).
 * Group boundaries must be multiples of 32 tokens (one scale block never
 * straddles two experts); m % 32 == 0, k % 16 == 0.
 * Replaces wgrad_fused.py:34-112 (which stacked per-expert copies and assumed
 * equal groups, wgrad_fused.py:46-62; here the contraction reads each
 * expert's token range in place). */
MXG_API size_t mxg_grouped_wgrad_workspace_size(int num_groups, int64_t m, int64_t n, int64_t k);
MXG_API int mxg_grouped_wgrad(const void* go, const void* go_scales, const void* ia,
                      const void* ia_scales, const int32_t* offs, int offs_len, int offs_kind,
                      int num_groups, int64_t m, int64_t n, int64_t k, void* out, int out_dtype,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Two-phase form of mxg_grouped_wgrad, the counterpart of the reference's
 * wgrad_prepare()/wgrad_kernel() split (wgrad_fused.py:74-112), without its
 * operand copies: prepare reads offs and the scales, run the e4m3 operands. */
MXG_API int mxg_grouped_wgrad_prepare(const void* go_scales, const void* ia_scales,
                                      const int32_t* offs, int offs_len, int offs_kind,
                                      int num_groups, int64_t m, int64_t n, int64_t k,
                                      void* workspace, size_t workspace_bytes, void* stream);
MXG_API int mxg_grouped_wgrad_run(const void* go, const void* ia, int num_groups, int64_t m,
                                  int64_t n, int64_t k, void* out, int out_dtype, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* Both MXFP8 encodings of x [rows, cols] bf16 in one pass: row-wise (q, s as
 * mxg_quantize_rowwise) and column-wise (qt, st as mxg_quantize_colwise),
 * bit-identical to those two.  rows and cols multiples of 32; either output
 * pair may be null (not both). */
MXG_API int mxg_quantize_dual(const void* x_bf16, int64_t rows, int64_t cols, void* q_e4m3,
                              void* scales_e8m0, void* qt_e4m3, void* scales_t_e8m0, void* stream);

/* mxg_quantize_dual restricted to rows [row_begin, row_end) of x (both
 * multiples of 32): the outputs keep the layout of the whole [rows, cols]
 * tensor and only the bytes of those rows (row-wise) or of those columns of
 * qt / 32-row blocks of st (column-wise) are written, so encoding a tensor in
 * row ranges, one launch each, writes the same bytes as one whole-tensor
 * encode.  Lets the rows of some expert groups be encoded while the rest are
 * still arriving. */
MXG_API int mxg_quantize_dual_rows(const void* x_bf16, int64_t rows, int64_t cols, int64_t row_begin,
                                   int64_t row_end, void* q_e4m3, void* scales_e8m0, void* qt_e4m3,
                                   void* scales_t_e8m0, void* stream);

/* MXFP8 encodings of h = silu(g) * u for gu rows [g (inter) | u (inter)]
 * (bf16 [rows, 2*inter]) without writing h: bit-identical to mxg_swiglu
 * followed by mxg_quantize_dual on its output.  rows, inter multiples of 32. */
MXG_API int mxg_swiglu_quantize(const void* gu_bf16, int64_t rows, int64_t inter, void* q_e4m3,
                                void* scales_e8m0, void* qt_e4m3, void* scales_t_e8m0, void* stream);

/* MXFP8 encodings of dgu = mxg_swiglu_bwd(gu, dh) ([rows, 2*inter]) without
 * writing dgu; bit-identical to the unfused pair. */
MXG_API int mxg_swiglu_bwd_quantize(const void* gu_bf16, const void* dh_bf16, int64_t rows,
                                    int64_t inter, void* q_e4m3, void* scales_e8m0, void* qt_e4m3,
                                    void* scales_t_e8m0, void* stream);

/* ---- expert parallelism: token routing (experts sharded evenly over ranks) ----
 * Global expert e lives on rank e / E_local as local expert e % E_local.  The
 * reference relies on torchtitan's MoE token dispatcher for this step
 * (port_mxfp8.py:74,214-218,240: all-to-all dispatch, groups padded to 32). */
#define MXG_EP_MAX_EXPERTS 384
#define MXG_EP_MAX_RANKS 64

/* Stable counting sort of routing slots (token t, choice j at t*topk + j) by
 * expert slot = slot_of_expert[expert id] (slot_of_expert null = identity;
 * slot s lives on rank s / E_local): counts[s], send_rows[p] = token row sent
 * at position p (positions grouped by slot, tokens in order),
 * slot_pos[t*topk+j] = p.  An id outside [0, num_experts) sets the device
 * error word to MXG_ERR_INVALID_ARGUMENT and its slot_pos to -1. */
MXG_API size_t mxg_ep_route_workspace_size(int64_t n_slots, int num_experts);
MXG_API int mxg_ep_route(const int32_t* expert_ids, const int32_t* slot_of_expert, int64_t n_slots,
                         int topk, int num_experts, int32_t* counts, int32_t* send_rows,
                         int32_t* slot_pos, void* workspace, size_t workspace_bytes, void* stream);

/* dst[i] = src[idx[i]] for rows of row_bytes (multiple of 16); idx[i] < 0 or
 * >= src_rows gives a zero row. */
MXG_API int mxg_gather_rows(const void* src, int64_t src_rows, int64_t row_bytes, const int32_t* idx,
                            int64_t n, void* dst, void* stream);

/* Rows received from every rank (ordered by source rank, then local expert,
 * counts in recv_counts[world][e_local]) -> expert-major groups padded to
 * `pad` rows: idx[i] = received row of padded row i (-1 for padding),
 * back[received row] = its padded row, group_rows[le] = padded group size. */
MXG_API int mxg_ep_regroup(const int32_t* recv_counts, int world, int e_local, int pad, int32_t* idx,
                           int32_t* back, int32_t* group_rows, void* stream);

/* out[t] = sum_j w[t*topk+j] * rows[slot_pos[t*topk+j]] (bf16 rows, fp32 sum,
 * bf16 out; weights may be null = 1). */
MXG_API int mxg_ep_combine(const void* rows, const int32_t* slot_pos, const float* weights,
                           int64_t n_tokens, int topk, int64_t hidden, void* out, void* stream);

/* h = silu(g) * u for gu rows [g (inter) | u (inter)], bf16 (the gate/up ->
 * down activation of the expert FFN, e2e_bench.py:56-61). */
MXG_API int mxg_swiglu(const void* gu, int64_t rows, int64_t inter, void* h, void* stream);

/* Backward of mxg_swiglu: dgu = [dg | du] (bf16 [rows, 2*inter]) from gu and
 * dh (bf16 [rows, inter]). */
MXG_API int mxg_swiglu_bwd(const void* gu, const void* dh, int64_t rows, int64_t inter, void* dgu,
                           void* stream);

/* ---- expert parallelism over NVLink peer memory ----
 * Receive buffers are shared between the ranks of one node with CUDA IPC; a
 * dispatch writes every routed row straight into its final (expert-major,
 * padded) row of the owner's buffer, a combine writes results back to the
 * token's home rank.  The kernels only store; the caller orders the ranks
 * with a collective before and after each exchange (replaces the all-to-all
 * of torchtitan's token dispatcher, port_mxfp8.py:74,240). */
#define MXG_PEER_HANDLE_BYTES 64
MXG_API int mxg_peer_alloc(size_t bytes, void** dptr, void* handle_out);
MXG_API int mxg_peer_open(const void* handle, void** dptr);
MXG_API int mxg_peer_close(void* dptr);
MXG_API int mxg_peer_free(void* dptr);

/* From the all-gathered slot counts counts_all [world][num_slots] (slot s on
 * rank s / (num_slots / world)): this rank's send-position prefix
 * slot_start [num_slots + 1], dest_base [num_slots] (destination row of send
 * position p in slot s = dest_base[s] + p), its own padded groups
 * group_rows / group_start [e_local (+1)], for each of its m_pad padded rows
 * the rank and send position the result returns to (back_rank, back_row; -1
 * on padding rows), and ret_order: its real rows grouped by home rank in the
 * order me+1, me+2, ... (mod world). */
MXG_API size_t mxg_ep_p2p_plan_workspace_size(int world, int num_slots);
MXG_API int mxg_ep_p2p_plan(const int32_t* counts_all, int world, int num_slots, int me, int pad,
                            int64_t m_pad, int32_t* slot_start, int32_t* dest_base,
                            int32_t* group_rows, int32_t* group_start, int32_t* back_rank,
                            int32_t* back_row, int32_t* ret_order, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Row src[send_rows[p]] -> row dest_base[s] + p of peer_bufs[s / e_local]
 * (peer_bufs: device array of every rank's buffer address), starting with
 * the positions bound for rank me+1 so that the ranks write to different
 * peers at the same time.  Only the positions p < slot_start[num_slots] are
 * sent (routing slots with an out-of-range expert id are counted nowhere).
 * A destination row outside [0, capacity_rows) or a source row outside
 * [0, src_rows) is skipped and sets the device error word
 * (MXG_ERR_WORKSPACE_TOO_SMALL, MXG_ERR_INVALID_ARGUMENT).  max_blocks <= 0: the library's
 * default grid, sharing SMs with concurrent work; max_blocks > 0: that many
 * 1024-thread blocks that only run on SMs no GEMM block occupies (pair with
 * mxg_set_gemm_sm_limit to overlap an exchange with the GEMMs). */
MXG_API int mxg_ep_dispatch_p2p(const void* src, int64_t src_rows, int64_t row_bytes,
                                const int32_t* send_rows, int64_t n_send, const int32_t* slot_start,
                                const int32_t* dest_base, int num_slots, int e_local, int me,
                                const uint64_t* peer_bufs, int64_t capacity_rows, int max_blocks,
                                void* stream);

/* mxg_ep_dispatch_p2p of src with two additions, in the same pass (bound by
 * NVLink, so the local copies ride along):
 *  - src2 non-null: row send_rows[p] of src2 (same row size and row count as
 *    src) is copied to row p of gather_out (this GPU's memory, n_send rows):
 *    a second tensor put in send order for a later exchange on the copy
 *    engines (mxg_copy_runs);
 *  - split_h in (0, e_local]: positions of slots whose local expert index
 *    (slot % e_local) is >= split_h are not stored to their owner; their src
 *    row goes to row p of src_later (this GPU's memory, n_send rows) instead,
 *    so that part of the dispatch can follow on the copy engines while the
 *    owners already work on the experts below split_h.  0: no split.
 * Default grid. */
MXG_API int mxg_ep_dispatch_p2p_gather(const void* src, int64_t src_rows, int64_t row_bytes,
                                       const int32_t* send_rows, int64_t n_send,
                                       const int32_t* slot_start, const int32_t* dest_base,
                                       int num_slots, int e_local, int me, const uint64_t* peer_bufs,
                                       int64_t capacity_rows, const void* src2, void* gather_out,
                                       int split_h, void* src_later, void* stream);

/* Padded local rows q = ret_order[i] (i < n_rows) -> row back_row[q] of
 * peer_bufs[back_rank[q]] (skipped where back_rank < 0). */
MXG_API int mxg_ep_return_p2p(const void* src, int64_t row_bytes, const int32_t* ret_order,
                              int64_t n_rows, const int32_t* back_rank, const int32_t* back_row,
                              const uint64_t* peer_bufs, int world, int64_t capacity_rows,
                              int max_blocks, void* stream);

/* Contiguous runs of rows moved by the GPU's copy engines instead of SMs, so
 * an exchange can run beside tensor-core kernels without taking their SMs:
 * run i copies rows [src_row[i], src_row[i] + rows[i]) of src to rows
 * [dst_row[i], dst_row[i] + rows[i]) of dst_bufs[dst_buf[i]], one
 * cudaMemcpyAsync per run on the given stream.  The run tables and dst_bufs
 * are HOST arrays; dst_bufs may hold peer addresses (mxg_peer_open).  Every
 * run is checked against src_rows and dst_rows before any copy is issued
 * (MXG_ERR_INVALID_ARGUMENT).  The copies only write; the caller orders the
 * ranks around them as around mxg_ep_dispatch_p2p. */
MXG_API int mxg_copy_runs(const void* src, int64_t src_rows, int64_t row_bytes, const int64_t* src_row,
                          const int64_t* dst_row, const int64_t* rows, const int32_t* dst_buf,
                          int64_t n_runs, const uint64_t* dst_bufs, int n_dst, int64_t dst_rows,
                          void* stream);

/* Zero the rows q < m_pad of buf with back_rank[q] < 0. */
MXG_API int mxg_ep_zero_pad_rows(void* buf, int64_t row_bytes, const int32_t* back_rank,
                                 int64_t m_pad, void* stream);

/* Cap on the SMs the grouped GEMMs' persistent grids use (0: all SMs);
 * process-wide, read at each GEMM launch.  Leaves SMs to kernels that run
 * concurrently on another stream, such as the peer exchanges above. */
MXG_API int mxg_set_gemm_sm_limit(int sms);
MXG_API int mxg_get_gemm_sm_limit(void);

/* ---- byte transpose: dst [cols, rows] = src [rows, cols]^T (uint8) ----------- */
MXG_API int mxg_transpose_u8(const void* src, int64_t rows, int64_t cols, void* dst, void* stream);

/* Test hook: the next grouped GEMM launch on this device waits on a barrier
 * nothing arrives on, with the given limit in nanoseconds, so the bounded
 * wait runs out and records MXG_ERR_DEVICE_TIMEOUT.  0 disables. */
MXG_API int mxg_debug_inject_stall(int64_t timeout_ns);

#ifdef __cplusplus
}
#endif

#endif /* MXG_H_ */
