/*
 * mrun-b200 C ABI: the drop-in boundary for mrun's quantized decode hot path.
 *
 * Every function is `extern "C"`, takes plain device pointers, element counts and a
 * `void *stream` (a cudaStream_t, or NULL for the legacy default stream), enqueues its
 * kernels on that stream without synchronising, and returns an int status:
 *
 *   MRB_OK (0)            success
 *   MRB_ERR_ARG (1)       an argument failed validation (the Python mirror raises ValueError)
 *   MRB_ERR_CUDA (2)      a CUDA launch or runtime call failed (RuntimeError)
 *   MRB_ERR_UNSUPPORTED (3) a valid request outside this build's kernels (RuntimeError)
 *   MRB_ERR_IO (4)        an operating-system file call failed (OSError)
 *
 * mrb_last_error() returns the message of the last failing call on the calling thread.
 * Layouts follow the reference QStore: a "qrow" matrix is int8 codes [rows, cols] row-major
 * with one fp32 scale per row (weight = code * scale), exactly as written by
 * `_quant_row_int8` (mrun engine/kernels/qstore_build.py:496-501).
 *
 * The reference is pure Python; a maintainer binds these entry points on its side with
 * ctypes. Each entry point names the reference function it replaces.
 */
#ifndef MRUN_B200_H
#define MRUN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MRB_OK = 0,
  MRB_ERR_ARG = 1,
  MRB_ERR_CUDA = 2,
  MRB_ERR_UNSUPPORTED = 3,
  MRB_ERR_IO = 4,
};

/* Element types of activation/output buffers. */
enum {
  MRB_F32 = 0,
  MRB_BF16 = 1,
  MRB_F16 = 2,
};

/* ---------------------------------------------------------------- library */

/* ABI revision of this header; bumps on any signature change. */
int mrb_abi_version(void);

/* Message for the last non-zero status returned on this host thread ("" if none). */
const char *mrb_last_error(void);

/* ---------------------------------------------------------------- (a) QStore int8 linear */

/* Per-output-channel symmetric int8 quantisation of an fp32 [rows, cols] matrix:
 * scale = max|w_row| / 127 (1 for an all-zero row), code = round_half_even(w / scale)
 * clipped to [-127, 127].
 * Replaces `_quant_row_int8` (engine/kernels/qstore_build.py:496-501). */
int mrb_quant_row_int8(const float *weight, int64_t rows, int64_t cols, int8_t *codes,
                       float *scales, void *stream);

/* Dequantised row gather: out[i, :] = codes[ids[i], :] * scales[ids[i]] in fp32, stored
 * as out_dtype. ids outside [0, rows) produce a zero row and set *bad_ids (device int32,
 * may be NULL) to 1.
 * Replaces `QStore.embed_rows` (engine/kernels/qstore.py:1099-1128). */
int mrb_qrow_embed_rows(const int8_t *codes, const float *scales, int64_t rows, int64_t cols,
                        const int64_t *ids, int64_t n_ids, void *out, int out_dtype,
                        int32_t *bad_ids, void *stream);

/* y[m, n] = sum_k x[m, k] * codes[n, k] * scales[n] (+ bias[n]), fp32 accumulation.
 * x_dtype in {F32, BF16, F16}; y_dtype = x_dtype (the reference returns x's dtype).
 * bias (fp32 [n], may be NULL) is added after rounding to y's dtype, as the reference adds
 * a compute-dtype bias to the projection output.
 * Requires k % 16 == 0 and 16-byte aligned codes.
 * workspace (may be NULL): zero-initialised device memory of mrb_qrow_workspace(n) bytes,
 * 256-byte aligned. With it, decode-size calls (m <= 16) whose 16-row tiles do not spread
 * evenly over the SMs split tiles along k (stream-K) so every CTA streams the same number
 * of weight bytes; a split tile is finished by its last CTA, adding partial sums in a fixed
 * order. Its counters reset themselves, so one workspace serves any number of calls that
 * are ordered on one stream; calls that may run concurrently need separate workspaces.
 * With NULL every CTA owns whole tiles.
 * Replaces `fused_qrow_matmul` (engine/kernels/dense_qstore_cuda.py:1105-1152) for
 * bf16/fp16 rows and `QStore.matmul` (engine/kernels/qstore.py:1082-1092) for fp32 rows. */
int mrb_qrow_matmul(const void *x, int x_dtype, int64_t m, int64_t k, const int8_t *codes,
                    const float *scales, int64_t n, const float *bias, void *y, int y_dtype,
                    void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of the optional mrb_qrow_matmul / mrb_qrow_swiglu workspace for n output rows on
 * the current device (any m, k and dtype). */
size_t mrb_qrow_workspace(int64_t n);

/* Paired gate/up W8A16 projection with the reference's BF16 SwiGLU boundaries:
 * g = bf16(x.Wg), u = bf16(x.Wu), s = bf16(g * sigmoid(g)), y = bf16(s * u).
 * workspace: as for mrb_qrow_matmul.
 * Replaces `fused_qrow_swiglu` (engine/kernels/dense_qstore_cuda.py:1052-1102). */
int mrb_qrow_swiglu(const void *x_bf16, int64_t m, int64_t k, const int8_t *gate_codes,
                    const float *gate_scales, const int8_t *up_codes, const float *up_scales,
                    int64_t n, void *y_bf16, void *workspace, size_t workspace_bytes,
                    void *stream);

/* Greedy language head: logits[m, v] = x[m].W[v] * scale[v] in fp32 over the first
 * `semantic_rows` rows, then the first maximal index per row (lowest index on ties), fused
 * into the head GEMV (order-preserving 64-bit keys, atomic max). out_index: int64 [m];
 * out_value: fp32 [m] (may be NULL); logits: fp32 [m, n] (may be NULL: not stored).
 * Replaces the streamed exact head `_head` (engine/dense_qstore_cuda.py:800-896). */
int mrb_qrow_argmax(const void *x, int x_dtype, int64_t m, int64_t k, const int8_t *codes,
                    const float *scales, int64_t n, int64_t semantic_rows, float *logits,
                    int64_t *out_index, float *out_value, void *stream);

/* Row RMSNorm in fp32: y = x * rsqrt(mean(x^2) + eps) * w, stored in x's dtype.
 * Replaces `stable_rms_norm` (engine/kernels/dense_qstore_cuda.py:1473-1511). */
int mrb_rms_norm(const void *x, int dtype, int64_t rows, int64_t width, const float *weight,
                 float eps, void *y, void *stream);

/* r = bf16(residual + update); normed = bf16(RMSNorm(r) * w).
 * Replaces `fused_residual_rms_norm` (engine/kernels/dense_qstore_cuda.py:1411-1459). */
int mrb_residual_rms_norm(const void *residual_bf16, const void *update_bf16, int64_t rows,
                          int64_t width, const float *weight, float eps, void *residual_out,
                          void *normed_out, void *stream);


/* ---------------------------------------------------------------- (a) W8A8 */

/* Number of bounded waits of the tensor-core (tcgen05) GEMMs that timed out since the last
 * call, then reset; 0 in normal operation (non-zero: those launches' outputs are invalid).
 * Synchronises the current device. No counterpart in the reference. */
int mrb_tc_status(unsigned *timeouts);

/* Per-token dynamic int8 activations exactly as the reference quantises them:
 * act_scale[r] = max|x[r] * keep| / 127 (fp32 division, 0 -> 1),
 * qx = clamp(round_half_even(x * keep / act_scale), -127, 127). keep (fp32 [k]) may be NULL.
 * Replaces the activation step of `w8a8_matmul` (engine/kernels/w8a8.py:117-121). */
int mrb_w8a8_quantize(const void *x, int x_dtype, int64_t m, int64_t k, const float *keep,
                      int8_t *qx, float *act_scale, void *stream);

/* acc[m, n] = sum_k qx[m, k] * qw[n, k] in int32, exact (k % 16 == 0, k <= 133000).
 * Replaces `_int8_gemm` (engine/kernels/w8a8.py:33-64). */
int mrb_int8_gemm(const int8_t *qx, const int8_t *qw, int64_t m, int64_t n, int64_t k,
                  int32_t *acc, void *stream);

/* Outlier columns: the `topk` columns with the largest max|x| over all rows (ties -> lower
 * column), written to idx_out, with keep[col] = 0 for them and 1 elsewhere.
 * Replaces the protect_k selection of `w8a8_matmul` (engine/kernels/w8a8.py:98-105). */
int mrb_w8a8_protect_topk(const void *x, int x_dtype, int64_t m, int64_t k, int topk,
                          int64_t *idx_out, float *keep, void *stream);

/* y[m, n] = side + (float(acc) * act_scale[m]) * w_scale[n] with acc the exact int32 dot of
 * the quantised activations and codes; side is the fp32 path of the `nprotect` protected
 * columns (0 when nprotect == 0, making y bit-identical to the reference). keep: the mask
 * from mrb_w8a8_protect_topk (or any 0/1 mask matching protect_idx). acc_out (int32 [m, n])
 * may be NULL. Workspaces: qx_ws int8 [m, k] and scale_ws fp32 [m] (needed unless the
 * decode GEMV takes the call: m <= 16 and the int8 row block fits one CTA; scale_ws also
 * receives the activation scales there when given), side_ws fp32 [m, n]
 * (needed when nprotect > 0).
 * Replaces `w8a8_matmul` (engine/kernels/w8a8.py:67-125). */
int mrb_w8a8_matmul(const void *x, int x_dtype, int64_t m, int64_t k, const int8_t *qw,
                    const float *w_scale, int64_t n, const int64_t *protect_idx, int nprotect,
                    const float *keep, float *y, int32_t *acc_out, int8_t *qx_ws, float *scale_ws,
                    float *side_ws, void *stream);

/* W8A8 projection of a bf16 decoder: per-token int8 activations (the mrb_w8a8_quantize
 * arithmetic, into qx_ws int8 [m, k] and scale_ws fp32 [m]), exact int32 accumulation on the
 * tensor cores, then y = bf16((float(acc) * act_scale) * w_scale + bias) (bias fp32 [n] or
 * NULL). With up_codes/up_scales (paired gate/up pages, each [n, k]) y is the SwiGLU
 * bf16(bf16(silu(bf16 g)) * bf16 u) of the two rescaled projections and bias must be NULL.
 * Skinny row blocks (decode batches) split k over the CTAs of a thread-block cluster and
 * reduce the exact int32 partials through distributed shared memory, so y does not depend
 * on the split and no workspace is needed.
 * Replaces `store.matmul` under `enable_w8a8` (engine/kernels/w8a8.py:145-177) for the
 * dense engine's projections and its paired gate/up (engine/dense_qstore_cuda.py:661-687). */
int mrb_w8a8_linear_bf16(const void *x_bf16, int64_t m, int64_t k, const int8_t *codes,
                         const float *scales, const int8_t *up_codes, const float *up_scales,
                         const float *bias, int64_t n, void *y_bf16, int8_t *qx_ws, float *scale_ws,
                         void *stream);

/* ---------------------------------------------------------------- (b) routed MoE */

/* Router: probabilities = softmax(fp32(logits)) per token (max-subtracted, divided by the
 * sum), the k largest (ties -> lower expert) in descending order, optionally renormalised
 * by their fp32 sum; weights also rounded to bf16 (top_w_f32 / top_w_bf16 may be NULL).
 * logits_dtype in {F32, BF16}; experts <= 256; k <= 16.
 * Replaces the router of `Qwen3MoeDecodeRuntime.forward` (engine/qwen3_moe_cuda.py:3700-3707). */
int mrb_router_topk(const void *logits, int logits_dtype, int64_t tokens, int64_t experts, int64_t k,
                    int renorm, int64_t *top_idx, float *top_w_f32, void *top_w_bf16, void *stream);

/* The whole router of one MoE layer: logits[t, e] = bf16(scale[e] * sum_k x[t, k] * code[e, k])
 * (bf16 activations [tokens, hidden], int8 router codes [experts, hidden] with fp32 row
 * scales: the W8A16 projection's boundary, exact products, fp32 sums in a fixed order), then
 * the selection of mrb_router_topk on them -- two launches on `stream`, the second waiting on
 * the first's grid. logits_bf16 [tokens, experts] receives the logits and is required.
 * Outputs: top_idx, top_w_f32 (before bf16 rounding; may be NULL), top_w_bf16 (may be NULL)
 * and top_w_coef = float(bf16 weight) (the route compiler's coefficients; may be NULL).
 * hidden % 8 == 0; experts <= 256; k <= 16. Replaces the router linear and selection of
 * `Qwen3MoeDecodeRuntime.forward` (engine/qwen3_moe_cuda.py:3700-3707, 3927-3933). */
int mrb_router_qrow_topk(const void *x_bf16, int64_t tokens, int64_t hidden, const int8_t *codes,
                         const float *scales, int64_t experts, int64_t k, int renorm, void *logits_bf16,
                         int64_t *top_idx, float *top_w_f32, void *top_w_bf16, float *top_w_coef,
                         void *stream);

/* Route plan: counts/starts per expert (exclusive scan), expert-major token_ids and
 * coefficients in the stable order of the reference's CPU branch (argsort by expert,
 * stable: flat (token, rank) order inside each expert), and inverse[token*k + rank] = the
 * assignment's expert-major position. Deterministic: no atomic decides a position.
 * Expert ids outside [0, experts) set *error_flag (may be NULL) and are skipped.
 * experts <= 512. Replaces `grouped_route_tensors_with_inverse` (engine/olmoe_cuda.py:989-1135). */
int mrb_route_compile(const int64_t *top_idx, const float *top_w, int64_t tokens, int64_t k,
                      int64_t experts, int32_t *counts, int32_t *starts, int64_t *token_ids,
                      float *coef, int64_t *inverse, int32_t *error_flag, void *stream);

/* Grouped W8A16 expert projection over ragged per-expert row groups: for expert e, rows
 * [starts[e], starts[e] + counts[e]) of the output are x[row_ids[a]] (row_ids NULL: a) times
 * the expert's int8 codes (slot slot_of[e], NULL: e, at codes + slot * codes_stride bytes;
 * fp32 row scales at scales + slot * scales_stride floats), fp32 accumulation, bf16 output
 * [A, n]. swiglu: the page's rows [0, n) are gate rows and [up_rows, up_rows + n) up rows,
 * and the output is bf16(bf16(silu(bf16 g)) * bf16 u) as the reference forms it.
 * rows_hint: the total row count A (0 if unknown); with 8 or more rows per expert on
 * average the kernel stages 16 rows per pass instead of 8 (results are the same either way).
 * Replaces the grouped expert GEMMs of `PagedFP8ExpertBackend.moe`
 * (engine/qwen3_moe_cuda.py:2740-2761), with the int8 qrow codec. */
int mrb_grouped_qrow(const void *x_bf16, const int64_t *row_ids, const int32_t *starts,
                     const int32_t *counts, int64_t experts, const int8_t *codes,
                     int64_t codes_stride, const float *scales, int64_t scales_stride,
                     const int32_t *slot_of, int64_t n, int64_t k, int64_t up_rows, int swiglu,
                     int64_t rows_hint, void *y_bf16, void *stream);

/* The expert MLP of one MoE layer: the gate/up projection with the fused SwiGLU into act_bf16
 * [A, ffn], then the down projection into y_bf16 [A, hidden], over expert pages laid out as
 * `ExpertPageLayout` (codes and scales of each part at the given byte offsets inside a page of
 * page_stride bytes; expert e's page at slot slot_of[e], identity when NULL). Rows as for
 * mrb_grouped_qrow (row_ids: activation row of each expert-major assignment, NULL = identity).
 * The down launch starts on an expert as soon as the gate/up launch has stored that expert's
 * rows: sync is uint32 [2 * experts + 1], zeroed before the first call and left zeroed by each
 * call (per-expert counters); its last word is set to 1 when a down wait ran out (bounded),
 * after which the outputs are not to be trusted. Calls that may overlap need their own sync.
 * Replaces the expert loop of `PagedFP8ExpertBackend.moe` (engine/qwen3_moe_cuda.py:2740-2761). */
int mrb_grouped_expert_mlp(const void *x_bf16, const int64_t *row_ids, const int32_t *starts,
                           const int32_t *counts, int64_t experts, const void *pages, int64_t page_stride,
                           int64_t gate_up_codes_offset, int64_t gate_up_scales_offset,
                           int64_t down_codes_offset, int64_t down_scales_offset, const int32_t *slot_of,
                           int64_t hidden, int64_t ffn, int64_t rows_hint, void *act_bf16, void *y_bf16,
                           uint32_t *sync, void *stream);

/* Fixed-capacity expert-parallel dispatch plan (no reference counterpart: the reference
 * runs every expert on one device). Expert e lives on rank e / experts_per_rank. Each
 * (source, destination) block has `capacity` >= tokens * k slots, so the plan never
 * overflows and every exchange has a size known on the host (CUDA-graph friendly).
 * Assignment a = t * k + r goes to slot dst * capacity + pos (pos: its rank among the
 * assignments to dst, in route order). Outputs (device): send_expert int32 [world *
 * capacity] (destination-local expert id; unused slots: experts_per_rank), coef_slot fp32
 * (top_w of the slot's assignment, 0 if unused), slot_of_assign int64 [tokens * k],
 * slot_src int32 (source token, -1 if unused). An expert id outside [0, world *
 * experts_per_rank) sets *error_flag (device int32, may be NULL). */
int mrb_ep_pack(const int64_t *top_idx, const float *top_w, int64_t tokens, int64_t k,
                int64_t experts_per_rank, int64_t world, int64_t capacity, int32_t *send_expert,
                float *coef_slot, int64_t *slot_of_assign, int32_t *slot_src, int32_t *error_flag,
                void *stream);

/* send_rows[s] = source[slot_src[s]] (bf16 rows of `hidden`) for every used slot of a
 * dispatch plan; unused slots are left as they are. No reference counterpart. */
int mrb_ep_gather_rows(const void *source_bf16, int64_t hidden, const int32_t *slot_src, int64_t slots,
                       void *send_rows_bf16, void *stream);

/* Weighted combine in route-rank order: out[t] = sum_r coef[p] * expert_out[p] with
 * p = inverse[t*k + r], fp32 products summed left to right; fp32 and/or bf16 outputs.
 * Replaces `stable_route_reduce` (engine/qwen3_moe_cuda.py:2561-2664). */
int mrb_stable_route_reduce(const void *expert_out_bf16, const float *coef, const int64_t *inverse,
                            int64_t tokens, int64_t k, int64_t hidden, float *out_f32,
                            void *out_bf16, void *stream);

/* Expert-parallel exchange over NVLink peer memory (no counterpart in the reference, which
 * runs every expert on one device; an alternative to the NCCL all-to-all of the same
 * fixed-capacity plan). Each rank owns one mailbox of mrb_ep_mailbox_bytes(world,
 * capacity, hidden) bytes; mrb_ep_mailbox_create allocates and zeroes it and returns its
 * 64-byte CUDA IPC handle, mrb_ep_mailbox_open maps a peer's handle (another process on the
 * same node), mrb_ep_mailbox_close unmaps (owned = 0) or frees (owned = 1).
 * mrb_ep_mailbox_offsets gives the byte offsets of its six sections: dispatch flags,
 * return flags, counts, ids (int32 [world, capacity]), rows and back rows (bf16
 * [world * capacity, hidden]). `mailboxes` is a device array of the world mailbox pointers
 * (this rank's own at index rank); `state` is int32[4] of zeros owned by the caller per
 * exchange site ([3] becomes 1 if a bounded wait timed out: outputs are then invalid).
 * Per use: mrb_ep_pack (the plan) -> mrb_ep_p2p_dispatch (real rows into each destination's
 * mailbox, then release flags) -> mrb_ep_p2p_wait_dispatch (acquire every source's flag;
 * ids64 = received local expert ids, unused slots = dummy_expert) -> route + grouped MLP on
 * the mailbox rows -> mrb_ep_p2p_return (outputs into each source's back rows, then flags)
 * -> mrb_ep_p2p_wait_return -> mrb_stable_route_reduce on the back rows. Every rank must run
 * the same sequence (one process per GPU); waits are bounded. */
size_t mrb_ep_mailbox_bytes(int64_t world, int64_t capacity, int64_t hidden);
int mrb_ep_mailbox_offsets(int64_t world, int64_t capacity, int64_t hidden, int64_t *out6);
int mrb_ep_mailbox_create(size_t bytes, void **ptr, void *ipc_handle);
int mrb_ep_mailbox_open(const void *ipc_handle, void **ptr);
int mrb_ep_mailbox_close(void *ptr, int owned);
int mrb_ep_p2p_dispatch(const void *x_bf16, int64_t hidden, const int32_t *slot_src,
                        const int32_t *send_expert, int64_t world, int64_t rank, int64_t capacity,
                        void *const *mailboxes, int32_t *state, void *stream);
int mrb_ep_p2p_wait_dispatch(void *mailbox, int64_t world, int64_t capacity, int64_t hidden,
                             int32_t dummy_expert, int64_t *ids64, int32_t *state, void *stream);
int mrb_ep_p2p_return(const void *eo_bf16, const int64_t *inverse, int64_t hidden, int64_t world,
                      int64_t rank, int64_t capacity, void *const *mailboxes, int32_t *state,
                      void *stream);
int mrb_ep_p2p_wait_return(void *mailbox, int64_t world, int64_t capacity, int64_t hidden,
                           int32_t *state, void *stream);
/* The receive side of a dispatch and the route compile in one launch (one CTA): waits as
 * mrb_ep_p2p_wait_dispatch does, writes each slot's local expert id into ids64 [world *
 * capacity] (-1 for padding, so only the rows that arrived are ranked), then compiles their
 * routes as mrb_route_compile(ids64, coef_in, world * capacity, 1, experts_local, ...) does:
 * counts/starts [experts_local], token_ids/coef/inverse [world * capacity] (entries of padding
 * slots unused). experts_local <= 512. */
int mrb_ep_p2p_wait_route(void *mailbox, int64_t world, int64_t capacity, int64_t hidden, int64_t experts_local,
                          int64_t *ids64, const float *coef_in, int32_t *counts, int32_t *starts, int64_t *token_ids,
                          float *coef, int64_t *inverse, int32_t *state, void *stream);
/* Waits for every owner's return flag (as mrb_ep_p2p_wait_return) and combines the back rows
 * in the same launch, as mrb_stable_route_reduce(back, coef, slot_of_assign, tokens, k, hidden,
 * NULL, out_bf16) does (bit-identical). */
int mrb_ep_p2p_combine(void *mailbox, int64_t world, int64_t capacity, int64_t hidden, const float *coef,
                       const int64_t *slot_of_assign, int64_t tokens, int64_t k, void *out_bf16, int32_t *state,
                       void *stream);
/* Bound (in polls, each followed by a ~64 ns sleep) of the flag waits launched from now on by
 * mrb_ep_p2p_wait_dispatch / mrb_ep_p2p_wait_return in this process; 2^22 by default, [1, 2^30].
 * A graph captured earlier keeps the bound it was captured with. mrb_ep_wait_limit reads it. */
int mrb_ep_set_wait_limit(int64_t polls);
int64_t mrb_ep_wait_limit(void);

/* ---------------------------------------------------------------- on-disk stores */

/* Open a store file (a QStore's weights.i8 / scales.f32 / extras.f32, an expert page file)
 * for reading: *handle receives the reader, *size the file's length in bytes. Host only.
 * Replaces the numpy memory maps of `QStore.__init__` (engine/kernels/qstore.py:700-714). */
int mrb_store_file_open(const char *path, void **handle, uint64_t *size);
/* Close a reader from mrb_store_file_open (NULL: no-op). */
int mrb_store_file_close(void *handle);
/* Copy bytes [offset, offset + bytes) of the file into host memory dst (normally a pinned
 * staging buffer), split over up to `threads` parallel pread calls of 4 MiB pieces (the
 * calling thread is one of them; small ranges use it alone). drop_after != 0 then asks the
 * kernel to drop the range's cached pages (POSIX_FADV_DONTNEED). A range past the end of the
 * file is MRB_ERR_ARG; a failed or short read is MRB_ERR_IO. Safe to call from several
 * threads at once (pread does not move a shared offset). Replaces the mmap-to-pinned copy of
 * `_RingPrefetch._stage` (engine/kernels/qstore.py:622-660, with `_drop_mmap_pages`
 * :402-426) and the pread warm-up of `HostPageTier.warm` (engine/qwen3_moe_cuda.py:925-951). */
int mrb_store_file_read(void *handle, uint64_t offset, uint64_t bytes, void *dst, int threads,
                        int drop_after);
/* Read-ahead hint for a range the caller expects to read next (will_need != 0:
 * POSIX_FADV_WILLNEED) or no longer needs (0: POSIX_FADV_DONTNEED); clipped to the file. */
int mrb_store_file_advise(void *handle, uint64_t offset, uint64_t bytes, int will_need);

/* ---------------------------------------------------------------- (c) paged-KV decode attention */

/* RoPE (rotate-half, fp32 products rounded separately, then bf16) for the queries and keys of
 * `tokens` new positions, and the K/V append into a paged cache.
 * Token t reads q/k/v rows at q_in/k_in/v_in + t * in_row_stride (bf16 elements), sits at
 * absolute position positions[t] of block-table row token_rows[t] (NULL: row 0), and is
 * written to page block_table[row * block_table_stride + pos / page_size], slot
 * pos % page_size, of K/V caches addressed as page*stride_page + head*stride_head +
 * slot*stride_tok + d. rope_cos/rope_sin: fp32 [rope_len, head_dim/2] tables (NULL: no
 * rotation, a plain scatter). q_out: bf16 [tokens, hq, head_dim] rotated queries (may be
 * NULL). Invalid positions/pages are skipped and set *error_flag (device int32, may be NULL).
 * q_norm / k_norm (bf16 [head_dim], may be NULL): per-head RMSNorm applied to each query /
 * key head before the rotation, as the reference's Qwen3 q/k norm (fp32 mean of squares +
 * norm_eps, normalised value rounded to bf16, times the weight rounded to bf16;
 * engine/qwen3_moe_cuda.py:3282-3285, 3903-3904).
 * Replaces `_rope` (engine/dense_qstore_cuda.py:689-704) and `scatter_segmented_decode_kv`
 * (engine/kernels/segmented_gqa_decode.py:458-524). */
int mrb_rope_kv_append(const void *q_in, const void *k_in, const void *v_in, int64_t in_row_stride,
                       int64_t tokens, int64_t hq, int64_t hkv, int64_t head_dim,
                       const int32_t *positions, const int32_t *token_rows, const float *rope_cos,
                       const float *rope_sin, int64_t rope_len, void *q_out, void *k_cache,
                       void *v_cache, int64_t stride_page, int64_t stride_head, int64_t stride_tok,
                       int64_t page_size, const int32_t *block_table, int64_t block_table_stride,
                       int64_t num_pages, int32_t *error_flag, const void *q_norm,
                       const void *k_norm, float norm_eps, void *stream);

/* Causal prefill attention for n tokens of one sequence at positions start .. start + n - 1,
 * already appended to the paged cache (mrb_rope_kv_append): token i attends to positions
 * [0, start + i] of the sequence whose page-table row is block_table. q/out: bf16
 * [n, hq, 128]. Flash attention on the tensor pipe: one CTA per (16-token query block, KV
 * head), the K/V prefix read once per block instead of once per token. An unmapped page sets
 * *error_flag (may be NULL) and reads as zeros. head_dim 128, hq / hkv <= 16, page_size a
 * multiple of 16. Replaces the prefill attention of the dense engine
 * (`_stable_attention_kernel` / SDPA, engine/kernels/dense_qstore_cuda.py:747-829). */
int mrb_paged_prefill_attention(const void *q, int64_t n, int64_t hq, int64_t hkv, int64_t head_dim,
                                int64_t start, const void *k_cache, const void *v_cache,
                                int64_t stride_page, int64_t stride_head, int64_t stride_tok,
                                int64_t page_size, const int32_t *block_table, int64_t num_pages,
                                int32_t *error_flag, float scale, void *out, void *stream);

/* One decode token per query row in one launch: mrb_rope_kv_append's RoPE (and optional
 * q/k norm) of the row's query heads and key, its K/V append at position positions[r] of
 * block-table row row_seq[r] (NULL: r), and mrb_paged_attention over tokens
 * [0, positions[r]] -- the cached ones plus the new one -- written to out (bf16
 * [rows, hq, head_dim]). Every row continues a different sequence.
 * - Same rounding as the two separate calls for the rotation and the append (bit-exact
 *   cache contents).
 * - The attention splits each row over a cluster of up to 16 CTAs per KV head and merges in
 *   rank order through distributed shared memory (deterministic; no workspace): on the
 *   tensor pipe (mma.sync, query heads as the rows) for head_dim 128 with pages of a
 *   multiple of 16 tokens, else one warp per query head. max_total_tokens bounds
 *   positions[r] + 1 and fixes the cluster size.
 * - state_ready = 1: positions, row_seq, the block table and the cached K/V below
 *   positions[r] are not written by any kernel that may still run when this one starts (a
 *   decode step whose bookkeeping runs after its layers); the kernel reads them before
 *   waiting on the preceding kernel (programmatic dependent launch). 0: every read waits.
 * - An invalid position or new-token page sets *error_flag and writes zeros for that row; an
 *   unmapped page among the cached tokens sets *error_flag and reads as zeros.
 * - head_dim in {64, 128}; hq / hkv <= 16; rows * hkv <= 65535; K/V rows 16-byte aligned.
 * Replaces the `_rope` + `scatter_segmented_decode_kv` + `segmented_gqa_decode` sequence of
 * one decode layer (engine/dense_qstore_cuda.py:689-704,
 * engine/kernels/segmented_gqa_decode.py:458-607). */
int mrb_rope_append_attention(const void *q_in, const void *k_in, const void *v_in,
                              int64_t in_row_stride, int64_t rows, int64_t hq, int64_t hkv,
                              int64_t head_dim, const int32_t *positions, const int32_t *row_seq,
                              const float *rope_cos, const float *rope_sin, int64_t rope_len,
                              const void *q_norm, const void *k_norm, float norm_eps,
                              void *k_cache, void *v_cache, int64_t stride_page,
                              int64_t stride_head, int64_t stride_tok, int64_t page_size,
                              const int32_t *block_table, int64_t block_table_stride,
                              int64_t num_pages, int32_t *error_flag, float scale,
                              int64_t max_total_tokens, int state_ready, void *out, void *stream);
/* CTAs per (row, KV head) cluster mrb_rope_append_attention uses for these sizes (0 for an
 * unsupported shape). Needs the current device. */
int mrb_rope_append_attention_cluster(int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                      int64_t max_total_tokens);

/* Waits of the TMA decode attention (canonical paged pools) that ran out on the current
 * device since the library loaded: each stage wait is bounded, and a wait that gives up counts
 * here and lets the kernel finish (its output is then not to be trusted). Negative on a CUDA
 * error. */
int64_t mrb_paged_attention_timeouts(void);

/* Workspace bytes mrb_paged_attention needs for these sizes (0 when no split is used). */
size_t mrb_paged_attention_workspace(int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                     int64_t max_total_tokens);

/* One-token grouped-query attention per query row over a paged KV cache, split-K over
 * 16-token tiles with a deterministic merge. q/out: bf16 [rows, hq, head_dim]; row r attends
 * to tokens [0, row_len[r]) of block-table row row_seq[r] (NULL: r), plus, when k_new/v_new
 * (bf16 [rows, hkv, head_dim]) are given, one provisional token at position row_len[r].
 * max_total_tokens bounds row_len (+1 with k_new) and fixes the split plan. The workspace
 * (mrb_paged_attention_workspace bytes) must be zero-filled before its first use; calls
 * leave it ready for the next call. head_dim in {64, 128}; hq / hkv <= 16.
 * Replaces `segmented_decode_attention` (engine/kernels/dense_qstore_cuda.py:1763-1854) and
 * `segmented_gqa_decode` (engine/kernels/segmented_gqa_decode.py:526-607). */
int mrb_paged_attention(const void *q, int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                        const void *k_cache, const void *v_cache, int64_t stride_page,
                        int64_t stride_head, int64_t stride_tok, int64_t page_size,
                        const int32_t *block_table, int64_t block_table_stride,
                        const int32_t *row_seq, const int32_t *row_len, const void *k_new,
                        const void *v_new, float scale, int64_t max_total_tokens, void *out,
                        void *workspace, size_t workspace_size, void *stream);

/* Allocation-free variant of mrb_paged_attention (no counterpart in the reference, which
 * always lets torch allocate). For callers that cannot allocate device memory -- a host that
 * has already reserved all GPU memory for its own pool, a latency-critical path where
 * cudaMalloc/cudaFree could synchronise the device, or a thin binding that only receives raw
 * pointers -- the split-K scratch lives in one static device array of
 * MRB_ATTN_STATIC_SCRATCH_BYTES per GPU (held by every GPU that loads the library until the
 * process exits), and nothing is allocated per call.
 * - Arguments and results as mrb_paged_attention, without the workspace.
 * - Sizes whose split plan needs more scratch than the array holds are rejected with
 *   MRB_ERR_UNSUPPORTED (mrb_paged_attention_workspace gives the need; use the
 *   workspace entry point for those).
 * - The first call on a device looks up the array's device address with that device
 *   current; make that first call before any stream capture. The address is kept per device
 *   and context: after cudaDeviceReset the next call looks it up again (a call made while
 *   capturing would then fail), so repeat a first call outside capture after a reset.
 * - Every call on a device shares the array: calls that can overlap on the GPU (different
 *   streams without ordering) race and must not be issued. Each call returns the array's
 *   merge counters to zero, so consecutive calls need no clearing. */
#define MRB_ATTN_STATIC_SCRATCH_BYTES (2 << 20)
size_t mrb_paged_attention_static_capacity(void);
int mrb_paged_attention_static(const void *q, int64_t rows, int64_t hq, int64_t hkv,
                               int64_t head_dim, const void *k_cache, const void *v_cache,
                               int64_t stride_page, int64_t stride_head, int64_t stride_tok,
                               int64_t page_size, const int32_t *block_table,
                               int64_t block_table_stride, const int32_t *row_seq,
                               const int32_t *row_len, const void *k_new, const void *v_new,
                               float scale, int64_t max_total_tokens, void *out, void *stream);

/* Greedy decode bookkeeping: input_ids[i] = next_ids[i]; positions[i] += 1; row_len[i] += 1
 * for i < rows. Lets a captured decode step feed itself (the reference's engine does this on
 * the host after `token.cpu()`, engine/dense_qstore_cuda.py:2389-2416). */
int mrb_decode_advance(const int64_t *next_ids, int64_t *input_ids, int32_t *positions,
                       int32_t *row_len, int64_t rows, void *stream);

/* ---------------------------------------------------------------- (d) weight-page streaming */

/* Host->device page copies on `stream`: page src_pages[i] (at src_base + page * src_stride,
 * pinned host memory for asynchronous copies) to slot dst_slots[i] (dst_base + slot *
 * dst_stride), one cudaMemcpyAsync per page, then records `done` (a cudaEvent_t, may be
 * NULL) on the stream. dst_slots/src_pages are host arrays of `count` entries.
 * Replaces the side-stream page staging of `_RingPrefetch` (engine/kernels/qstore.py:622-660)
 * and of the expert page cache (engine/qwen3_moe_cuda.py:1533-1546). */
int mrb_copy_pages(void *dst_base, int64_t dst_stride, const void *src_base, int64_t src_stride,
                   const int32_t *dst_slots, const int32_t *src_pages, int64_t count,
                   int64_t page_bytes, void *stream, void *done);

#ifdef __cplusplus
}
#endif

#endif /* MRUN_B200_H */
