/*
 * mlxturbo_b200.h -- C ABI of the B200 quantized-matmul library
 * (libmlxturbo_b200.so).
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to
 * contiguous row-major memory, every `stream` is a cudaStream_t passed as
 * void* (NULL = legacy default stream).  Calls are stream ordered and
 * asynchronous; nothing here synchronises the device or the host.
 *
 * Quantised weights use the MLX affine layout (mx.quantize, mode="affine"):
 *   w       uint32 [N, K*bits/32]   value k of a row at bit offset k*bits of the
 *                                   row's little-endian bit stream (low bits first)
 *   scales  T [N, K/group_size]     biases T [N, K/group_size]
 *   dequant(w)[n,k] = scales[n,k/gs] * q[n,k] + biases[n,k/gs]
 * with T = bf16 or fp16 (the activation dtype), bits in {4, 8}, group_size in
 * {32, 64, 128}.  Expert banks add a leading E dimension.
 *
 * Error model: the reference never raises on an ineligible shape -- it falls
 * back to stock MLX (mlxturbo/kernels/dispatch.py:329-330, fast_qmm.py:356-362).
 * This library has no fallback, so every entry point returns a status instead;
 * the Python layer turns QMM_EUNSUPPORTED into NotImplementedError and
 * QMM_EINVAL into ValueError.
 */
#ifndef MLXTURBO_B200_H
#define MLXTURBO_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QMM_API __attribute__((visibility("default")))
#else
#define QMM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    QMM_OK = 0,
    QMM_EUNSUPPORTED = 1, /* valid request outside what the kernels implement */
    QMM_EINVAL = 2,       /* inconsistent shapes, null or misaligned pointers */
    QMM_ECUDA = 3,        /* a CUDA runtime call or kernel launch failed */
    QMM_ENCCL = 4,        /* reserved for collective errors */
    QMM_ETIMEOUT = 5      /* a bounded device-side wait gave up */
} qmm_status;

typedef enum { QMM_BF16 = 0, QMM_F16 = 1 } qmm_dtype;

/* Human-readable text of a status, and of the last error recorded on the
 * calling thread (empty string when none). */
QMM_API const char* qmm_status_string(int status);
QMM_API const char* qmm_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
QMM_API int qmm_version(void);

/*
 * y[M,N] = x[M,K] @ dequant(w)^T.
 * Replaces mx.quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size, bits, mode="affine") as routed by
 * mlxturbo/kernels/dispatch.py:302-382 quantized_matmul and
 * mlxturbo/fast_qmm.py:334-374 fast_qmm.
 *   M <= 16 : decode / speculative-verify kernel (weights streamed once,
 *             in-register unpack, warp MMA, fixed-order split-K).
 *   M >  16 : prefill kernel (tensor cores).
 * Each output row depends only on its own input row: an M-row call returns,
 * row for row, the bits of M single-row calls (the property the reference
 * pins in bench/test_qmm_smallm.py:68-84).
 * x, scales, biases, y must be 16-byte aligned; w 16-byte aligned.
 * workspace (M <= 16 only; may be NULL): see qmm_quantized_matmul_workspace_size.
 */
QMM_API int qmm_quantized_matmul(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                         int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype, void* workspace,
                         size_t workspace_bytes, void* stream);
/*
 * Device scratch for qmm_quantized_matmul with M <= 16 (0 for M > 16).  The
 * whole buffer must be zero before the first call (cudaMemset once).  The
 * first 256 KiB hold the stream-K kernel's tile counters, which every call
 * leaves zero; from 8 MiB on, the integer-MMA kernel keeps an epoch word and
 * partial sums tagged with it, so a slot from an earlier call never reads as
 * this call's.  One buffer serves calls of any shape.  Calls sharing a
 * workspace must not overlap on the GPU.
 * With workspace == NULL the decode kernel runs without the stream-K schedule.
 */
QMM_API size_t qmm_quantized_matmul_workspace_size(int64_t M, int64_t N, int64_t K, int group_size, int bits);

/*
 * Greedy sampling fused with the lm_head matmul: y = x @ dequant(w)^T as
 * qmm_quantized_matmul computes it (y is stored), and per row m
 *   keys[m] = max over n of key(y[m, n], index_offset + n),
 *   key(v, i) = (order-preserving bits of the f32 value of v) << 32 | (0xFFFFFFFF - i),
 * so the token id is 0xFFFFFFFF - (keys[m] & 0xFFFFFFFF): the largest logit,
 * the smallest index among equal ones (a single-device argmax).  Keys of
 * column shards (index_offset = the shard's first row) combine with a max,
 * so a sharded lm_head exchanges M words instead of M*N logits.  For M <= 8 on
 * matrices the integer-MMA kernel takes, the keys come from that kernel's
 * output epilogue (one atomic max per warp and row, no second pass); other
 * shapes read y once more in a second launch.  Replaces the logits-then-argmax
 * of the reference's verify head (mlxturbo/spec.py:388-408 SpecEngine._head).
 * keys: uint64 [M], 8-byte aligned; cleared by the call.  workspace: as for
 * qmm_quantized_matmul.
 */
QMM_API int qmm_quantized_matmul_argmax(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                        void* y, int64_t M, int64_t N, int64_t K, int group_size, int bits,
                                        int dtype, int64_t index_offset, uint64_t* keys, void* workspace,
                                        size_t workspace_bytes, void* stream);

/*
 * The decode matmul (1 <= M <= 16) without a workspace argument, for callers
 * that cannot allocate device memory once they run: runtimes with a fixed
 * memory arena planned up front, FFI hosts without an allocator binding, and
 * serving loops that may not allocate on the first call of a new shape.  No
 * counterpart in the reference (MLX allocates inside its own runtime).
 * Scratch comes from a 16 MiB array inside the library (held by every GPU
 * that loads it until exit).  The kernel choice is qmm_quantized_matmul's
 * with a 16 MiB workspace: the integer-MMA kernel's share of the array covers
 * K up to about 200k, the stream-K kernel's every shape up to N = 2^20; a
 * larger integer-MMA problem runs on another decode kernel (results within the
 * bf16/fp16 tolerance of qmm_quantized_matmul's, not bit for bit), and a
 * shape that fits no kernel returns QMM_EUNSUPPORTED.
 * The first call on a device, with that device current, looks the array up
 * and clears it on the caller's stream -- make that call before any stream
 * capture.  All calls on a device share the array: calls that overlap on the
 * GPU race.  M = 0 returns QMM_OK; argument checks are qmm_quantized_matmul's.
 */
QMM_API int qmm_quantized_matmul_noalloc(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                         void* y, int64_t M, int64_t N, int64_t K, int group_size, int bits,
                                         int dtype, void* stream);

/*
 * gather_qmm: y[r] = x[lhs[r]] @ dequant(w[rhs[r]])^T for r in [0, rows).
 * Replaces mx.gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices,
 * transpose=True, group_size, bits, sorted_indices) as called from
 * mlxturbo/fused.py:3105-3116 and mlx-lm's QuantizedSwitchLinear.
 *   w [E, N, K*bits/32], scales/biases [E, N, K/gs], x [x_rows, K],
 *   lhs_indices int32 [rows] or NULL (identity), rhs_indices int32 [rows].
 *   sorted_indices != 0 promises rhs_indices is non-decreasing (the only form
 *   the reference uses); 0 sorts rows by expert on the device first.
 * workspace: device scratch of at least qmm_gather_workspace_size(rows, E)
 * bytes: the stream-K kernel's tile counters (the first 256 KiB: zero
 * before the first call, left zero by every call, and the same block the
 * decode workspace of qmm_quantized_matmul uses, so one buffer can serve
 * both), partial sums, segment tables and the sort permutation.
 */
QMM_API int qmm_gather_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases,
                   const int32_t* lhs_indices, const int32_t* rhs_indices, void* y, int64_t rows, int64_t x_rows,
                   int64_t E, int64_t N, int64_t K, int group_size, int bits, int dtype, int sorted_indices,
                   void* workspace, size_t workspace_bytes, void* stream);
QMM_API size_t qmm_gather_workspace_size(int64_t rows, int64_t E);

/*
 * Expert-segmented grouped matmul over rows already sorted by expert:
 * y[s] = x[row_src ? row_src[s] : s] @ dequant(w[e(s)])^T, written to row
 * row_dst ? row_dst[s] : s and scaled by row_scale[s] when given.
 * Replaces mlxturbo/kernels/moe_grouped_gemm.py:913-1065 qmm_segmented
 * (row_src gather fold, row_dst/row_scale epilogue).
 *   row_start int32 [E+1] (first row of each expert), M = row_start[E] rows.
 * workspace: at least qmm_segmented_workspace_size(M, E) bytes, laid out and
 * initialised like the qmm_gather_qmm workspace (zero tile counters first).
 */
QMM_API int qmm_segmented(const void* x, const uint32_t* w, const void* scales, const void* biases,
                  const int32_t* row_start, const uint32_t* row_src, const uint32_t* row_dst, const float* row_scale,
                  void* y, int64_t M, int64_t x_rows, int64_t E, int64_t N, int64_t K, int group_size, int bits,
                  int dtype, void* workspace, size_t workspace_bytes, void* stream);
QMM_API size_t qmm_segmented_workspace_size(int64_t M, int64_t E);

/*
 * The gathered matmul in two steps, for a caller that runs several
 * projections over the same expert-sorted rows (an MoE block: gate, up,
 * down): qmm_gather_tables builds the segment tables once from the sorted
 * expert ids (int32 [rows], non-decreasing) into the workspace, and each
 * qmm_gather_run launches only the matmul on them (same rows and E).
 * Workspace: qmm_segmented_workspace_size(rows, E) bytes, initialised like
 * the qmm_gather_qmm workspace.
 * qmm_gather_run: y[s] = x[row_src[s]] @ dequant(w[expert(s)])^T, stored to
 * row_dst[s] (or s) and scaled by row_scale[s] (or 1).  x rows are x_stride
 * elements apart (0: K; else a multiple of 8 that is >= K, e.g. the rows of
 * a qmm_ep_pack buffer, whose ids follow each row).  glu != 0: w holds
 * fused gate/up banks, rows interleaved per 16-row block (rows 16b..16b+7 =
 * gate rows 8b..8b+7, rows 16b+8..16b+15 = the matching up rows; N a multiple
 * of 16) and y[s] has N/2 columns, silu(gate) * up: the reference's
 * gate_proj / up_proj / SwitchGLU activation (mlx-lm SwitchGLU as called from
 * mlxturbo/_vendor/qwen4_exp.py:1796-1800) in one launch.
 * Returns QMM_EUNSUPPORTED when the problem exceeds the kernel's tile
 * counters (then use qmm_segmented).
 */
QMM_API int qmm_gather_tables(const int32_t* ids_sorted, int64_t rows, int64_t E, void* workspace,
                              size_t workspace_bytes, void* stream);
/*
 * The counting sort and the segment tables of qmm_gather_tables in one launch
 * (one CTA), for decode / verify batches: rows <= 16384 and E <= 1024, else
 * QMM_EUNSUPPORTED (use qmm_sort_rows + qmm_gather_tables).  Replaces
 * mlxturbo/kernels/moe_counting_sort.py:41-80 sort_rows (hist -> scan ->
 * in-order scatter) followed by moe_grouped_gemm.py:818-867 segment_tables.
 *   ids int32 [rows] expert ids in token-major order (ids outside [0, E) are
 *   padding rows: they sort last, in input order, with idx_s = E);
 *   order / idx_s / row_src / inv: uint32 [rows] exactly as qmm_sort_rows
 *   writes them (stable, so identical on every run);
 *   workspace: the qmm_gather_tables workspace, which then holds the tables
 *   qmm_gather_run reads (its counter block zero, as there).
 */
QMM_API int qmm_moe_route(const int32_t* ids, int64_t rows, int64_t E, int top_k, uint32_t* order, uint32_t* idx_s,
                          uint32_t* row_src, uint32_t* inv, void* workspace, size_t workspace_bytes, void* stream);
/*
 * Expert-parallel dispatch, the send side of the fixed-capacity exchange: for
 * each of a rank's n (token, expert) rows i = t * top_k + k with global
 * expert id ids[i] in [0, world * e_local), the owner d = ids[i] / e_local,
 * the slot s = d * n + (earlier rows with owner d), slot_of[i] = s.  send
 * holds world * n rows of row_stride elements (row_stride >= hidden + 8, a
 * multiple of 8): row s carries x row t in its first hidden bf16/fp16 values
 * and the local expert id ids[i] - d * e_local as an int32 right after them,
 * so rows and ids travel in one all-to-all.  Slots no row claims get the
 * padding id e_local (which the sort and the gathered kernels skip); their x
 * values are left as they were.  world <= 256, n <= 65536 (each row's CTA
 * scans all n ids).  Deterministic (stable by row).  No counterpart in the reference, whose MoE runs on one device: one
 * launch in place of the argsort / bincount / scatter glue of this library's
 * expert-parallel exchange.
 */
QMM_API int qmm_ep_pack(const int32_t* ids, int64_t n, int64_t e_local, int64_t world, int top_k, const void* x,
                        int64_t hidden, void* send, int64_t row_stride, int32_t* slot_of, void* stream);
QMM_API int qmm_gather_run(const void* x, const uint32_t* w, const void* scales, const void* biases,
                           const uint32_t* row_src, const uint32_t* row_dst, const float* row_scale, void* y,
                           int64_t rows, int64_t x_rows, int64_t x_stride, int64_t E, int64_t N, int64_t K,
                           int group_size, int bits, int dtype, int glu, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Per-expert row counts and segment tables from expert ids, no host sync.
 * Replaces moe_grouped_gemm.py:818-855 counts_from_sorted_ids + segment_tables:
 *   counts[e] = #{i : ids[i] == e}; row_start[0]=0, row_start[e+1]=row_start[e]+counts[e];
 *   tile_prefix[e+1] = tile_prefix[e] + ceil(counts[e]/b_e), b_e = bm, or
 *   16 / 32 by counts[e] < mix_threshold when mix_threshold > 0.
 * counts / row_start / tile_prefix may be NULL when not wanted.
 */
QMM_API int qmm_segment_tables(const int32_t* ids, int64_t M, int64_t E, int bm, int mix_threshold, int32_t* counts,
                       int32_t* row_start, int32_t* tile_prefix, void* stream);
/* The same tables from per-expert counts [E] (moe_grouped_gemm.py:829-855 segment_tables). */
QMM_API int qmm_segment_tables_from_counts(const int32_t* counts, int64_t E, int bm, int mix_threshold,
                                   int32_t* row_start, int32_t* tile_prefix, void* stream);

/*
 * Deterministic stable counting sort of expert ids (no atomics in the output
 * order): order = stable argsort(ids), idx_s = ids[order],
 * row_src = order / top_k, inv = argsort(order).
 * Replaces mlxturbo/kernels/moe_counting_sort.py sort_rows and the argsort
 * chain of _vendor/qwen4_exp.py:1775-1778 + fused._inv_perm.
 * workspace >= qmm_sort_workspace_size(M, E) bytes.
 */
QMM_API int qmm_sort_rows(const uint32_t* ids, int64_t M, int64_t E, int top_k, uint32_t* order, uint32_t* idx_s,
                  uint32_t* row_src, uint32_t* inv, void* workspace, size_t workspace_bytes, void* stream);
QMM_API size_t qmm_sort_workspace_size(int64_t M, int64_t E);

/*
 * MoE combine: y[t,n] = sum_k w[t*top_k+k] * out_sorted[inv[t*top_k+k], n]
 * with fp32 accumulation in k order and one rounding at the store.
 * Replaces mlxturbo/kernels/moe_combine.py combine.
 */
QMM_API int qmm_moe_combine(const void* out_sorted, const uint32_t* inv, const float* weights, void* y, int64_t rows,
                    int top_k, int64_t N, int dtype, void* stream);
/*
 * The same combine over a source of src_rows rows (inv entries >= src_rows are
 * skipped): for outputs that sit in a larger buffer, such as the
 * fixed-capacity slots of the expert-parallel exchange.
 */
QMM_API int qmm_moe_combine_rows(const void* out_src, int64_t src_rows, const uint32_t* inv, const float* weights,
                                 void* y, int64_t rows, int top_k, int64_t N, int dtype, void* stream);
/*
 * qmm_moe_combine_rows launched with programmatic dependent launch, for a
 * caller whose previous operation on the stream is this library's gathered
 * matmul (the down projection of qmm_gather_run): the combine's launch then
 * overlaps that kernel's tail.  After anything else on the stream (a
 * collective's join, another library's kernel) use qmm_moe_combine_rows.
 * Replaces the same moe_combine.py combine.
 */
QMM_API int qmm_moe_combine_chained(const void* out_src, int64_t src_rows, const uint32_t* inv, const float* weights,
                                    void* y, int64_t rows, int top_k, int64_t N, int dtype, void* stream);

/*
 * The whole MoE block at decode widths in one launch (replaces the
 * SparseMoeBlock call chain of mlxturbo/_vendor/qwen4_exp.py:1763-1806:
 * gather_qmv over gate_proj and up_proj, the SwiGLU activation, gather_qmv
 * over down_proj, the top_k sum weighted by the router; and the fused
 * gate/up variant of mlxturbo/kernels/moe_glu.py:145-168):
 *
 *   y[t] = sum_k weights[t, k] * down_e(silu(gate_e x[t]) * up_e x[t]),  e = ids[t, k]
 *
 * x [T, hidden] (dtype), ids int32 [T, top_k], weights fp32 [T, top_k]
 * (token-major), y [T, hidden].  gate_up_* is the gate and up banks
 * interleaved per 16-row block ([E, 2 * inter, hidden]: gate rows of
 * channels 8b..8b+7, then the up rows of the same channels), down_* the down
 * bank [E, hidden, inter]; MLX affine layout, one group size and code width
 * for all three.  An id outside [0, E) contributes nothing.
 *
 * Every (token, k) pair is computed on its own (no grouping by expert), so
 * a result does not depend on the other tokens' routing.  Shapes outside
 * the kernel (hidden and inter multiples of 1024 / bits with a multiple of
 * 8 quantisation groups per row; inter <= 2048; T * hidden <= 16384;
 * T * top_k <= 1024) return QMM_EUNSUPPORTED: the caller then runs the block
 * as separate launches (qmm_moe_route, qmm_gather_run, qmm_moe_combine_*).
 * The kernel needs every CTA of its grid resident at once (one per SM; a
 * bounded grid barrier sets the qmm_device_error flag if not).
 *
 * workspace: qmm_moe_glu_decode_workspace_size(T, top_k, inter) bytes,
 * 16-byte aligned, zero before the first call and used by one stream at a
 * time; the kernel leaves it ready for the next call.
 */
QMM_API size_t qmm_moe_glu_decode_workspace_size(int64_t T, int64_t top_k, int64_t inter);
QMM_API int qmm_moe_glu_decode(const void* x, const int32_t* ids, const float* weights, const uint32_t* gate_up_w,
                               const void* gate_up_scales, const void* gate_up_biases, const uint32_t* down_w,
                               const void* down_scales, const void* down_biases, void* y, int64_t T, int64_t top_k,
                               int64_t E, int64_t hidden, int64_t inter, int group_size, int bits, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream);

/* dequant(w) as T [N, K] (testing and weight conversion). */
QMM_API int qmm_dequantize(const uint32_t* w, const void* scales, const void* biases, void* out, int64_t N, int64_t K,
                   int group_size, int bits, int dtype, void* stream);

/*
 * MLX affine quantisation of fp32 weights w [N, K] into the layout above
 * (mx.quantize(w, group_size, bits, mode="affine"); the reference converts
 * checkpoints with it in mlxturbo/rebit.py:103-121).  bits in {2,3,4,5,6,8}.
 */
QMM_API int qmm_quantize(const float* w, uint32_t* wq, void* scales, void* biases, int64_t N, int64_t K, int group_size,
                 int bits, int dtype, void* stream);

/*
 * Kernel fire counters (mirrors mlxturbo/kernels/_fire.py:1-32): how many
 * times each kernel family was launched by this process.
 * qmm_fire_count(name) returns the count for one name (-1 if unknown);
 * qmm_fire_names() returns a comma-separated list of names.
 */
QMM_API long long qmm_fire_count(const char* name);
QMM_API const char* qmm_fire_names(void);
QMM_API void qmm_fire_reset(void);

/*
 * Decode-kernel tuning/test hook: run the M <= 16 kernel with an explicit
 * rows-per-warp (1 or 2) and K-split warp count (1..16).  Results depend
 * only on k_warps; rows_per_warp never changes a bit.
 */
QMM_API int qmm_qmv_explicit(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                     int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype, int rows_per_warp,
                     int k_warps, void* stream);

/*
 * The integer-MMA decode kernel for M <= 8 (mma.sync m16n8k32, u8 codes x
 * exact int8 activation planes built per call by a prep kernel), called
 * directly.  qmm_quantized_matmul dispatches to it for matrices of at least
 * 12 MiB of codes (the measured crossover; the same kernel for every M <= 8
 * on one matrix, so each row keeps the bits of a single-row call).
 * Requirements: M <= 8, K a multiple of 256 (4-bit) / 128 (8-bit),
 * (K / group_size) % 8 == 0, 16-byte aligned x, w, scales, biases, y and
 * workspace (qmm_quantized_matmul_workspace_size bytes, its counter block
 * zero).  QMM_EUNSUPPORTED outside those shapes.
 */
QMM_API int qmm_qmv_i8(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int64_t M,
                       int64_t N, int64_t K, int group_size, int bits, int dtype, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * Prefill-kernel test hook: run the tensor-core kernel (any M >= 1) with an
 * explicit token tile of 128 or 256 per CTA.  The tile never changes a bit.
 */
QMM_API int qmm_prefill_explicit(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                                 int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype,
                                 int tokens_per_cta, void* stream);

/*
 * Device-side error flag of the tensor-core kernels: nonzero after a bounded
 * wait inside a kernel gave up (the kernel then finished without a valid
 * result).  Synchronises the device; reset != 0 clears the flag.
 */
QMM_API int qmm_device_error(int reset);

/*
 * Measurement hook (no reference counterpart): one plain streaming read of
 * `bytes` (a multiple of 16) from the 16-byte aligned device buffer `p` on
 * `blocks` CTAs of 256 threads, launched like the decode kernel (programmatic
 * stream serialization).  `sink` is a device buffer of at least 1 KiB that the
 * kernel may write.  A chain of these with a decode layer's projection sizes
 * is the HBM floor the benchmark reports the decode kernel against.
 */
QMM_API int qmm_stream_read(const void* p, size_t bytes, int blocks, void* sink, void* stream);

/*
 * Copy `bytes` (a multiple of 16, both pointers 16-byte aligned) from src to
 * dst with one kernel on `stream`, where either side may be pinned host
 * memory (device-addressable under unified addressing) and the other device
 * memory: the few hundred KB a decode step moves in and out without a
 * copy-engine transfer's setup on the critical path.  Host memory is read
 * uncached and written through, so the host sees the data after a stream
 * synchronisation.  QMM_EINVAL for pageable host memory (use cudaMemcpyAsync).
 * No counterpart in the reference (MLX on Apple silicon shares one memory).
 */
QMM_API int qmm_copy_kernel(void* dst, const void* src, size_t bytes, void* stream);

/* The K-split warp count the decode kernel uses for (N, K) (never depends on M). */
QMM_API int qmm_qmv_k_warps(int64_t N, int64_t K, int group_size);

#ifdef __cplusplus
}
#endif

#endif /* MLXTURBO_B200_H */
