/*
 * helm_b200 — C ABI of the B200-native paged-KV decode path.
 *
 * This library replaces the eager-PyTorch KV-cache / attention path of HELM
 * (helm/runtime/kv_cache.py, kv_allocator.py, kv_offload.py).  Every entry
 * point takes plain device pointers, element strides and sizes, runs on the
 * CUDA stream it is given (a cudaStream_t passed as void*), never allocates
 * or frees caller memory, and returns an int status (HELM_OK on success).
 *
 * KV page pool layout (one contiguous allocation per device or host tier):
 *     pool[slot][kv][head][token][dim]      kv = 0 for K, 1 for V
 * i.e. a page slot holds K then V for all KV heads, each head's page_size x
 * head_dim block contiguous.  One (page, head) block is therefore a dense
 * page_size*head_dim*elt byte run (4 KiB for 16 bf16 tokens at head_dim 128).
 *
 * Data types: HELM_DTYPE_BF16 / HELM_DTYPE_FP16 for K, V, Q and outputs;
 * masks may also be HELM_DTYPE_FP32.  Softmax state is always fp32.
 */
#ifndef HELM_B200_H_
#define HELM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host return values) ---------------------------------- */
#define HELM_OK 0
#define HELM_ERR_INVALID_ARGUMENT 1
#define HELM_ERR_UNSUPPORTED 2
#define HELM_ERR_CUDA 3
#define HELM_ERR_WORKSPACE 4
#define HELM_ERR_ALIGNMENT 5

/* ---- device status bits (read with helm_get_device_status) --------------- */
#define HELM_DEV_TIMEOUT 1u   /* a bounded wait inside a kernel gave up      */
#define HELM_DEV_BAD_PAGE 2u  /* a page-table entry or page count was out of */
                              /* range; the access was skipped / clamped     */

/* ---- data types ------------------------------------------------------------ */
#define HELM_DTYPE_FP32 0
#define HELM_DTYPE_FP16 1
#define HELM_DTYPE_BF16 2

/* Library version (major*10000 + minor*100 + patch). */
int helm_version(void);

/* Human-readable text for a status code. */
const char* helm_status_string(int status);

/* Text of the last CUDA error seen by this thread inside the library. */
const char* helm_last_cuda_error(void);

/*
 * Reads the device status word of the current device into *out (after
 * synchronising `stream`), and clears it when `reset` is non-zero.
 * No reference counterpart: the reference raises Python exceptions
 * synchronously (kv_allocator.py:128-140, kv_cache.py:208); kernels here
 * record errors instead of trapping.
 */
int helm_get_device_status(unsigned int* out, int reset, void* stream);

/*
 * Bytes of fp32 scratch that helm_paged_decode_attention needs for the given
 * shape on the current device (split-KV partial softmax states).
 */
int64_t helm_paged_decode_workspace_bytes(int batch, int num_q_heads, int num_kv_heads,
                                          int head_dim);

/*
 * Paged decode attention for one query position per sequence:
 *     O[b,h,:] = softmax(scale * q[b,h,:] . K[b,kvh(h),t,:]^T  (+softcap) (+mask[b,t])) V
 * over the tokens t of sequence b, GQA mapping kvh(h) = h / (Hq/Hkv), fp32
 * accumulation, O in the query dtype, LSE = logsumexp of the same scores (fp32,
 * natural log; -inf for an empty sequence, whose O is zero).
 *
 * Replaces perform_streaming_attention (helm/runtime/kv_cache.py:405-662) and
 * the paged branches of _decode_batched (helm/runtime/kv_offload.py:144-186).
 *
 *  q            [B, Hq, D] with element strides q_stride_b, q_stride_h (dim stride 1)
 *  kv_pool      page pool (layout above), pool_pages slots
 *  page_table   int32 [B, max_pages] (row stride pt_stride_b): pool slot of page i
 *  kv_lens      int32 [B]: tokens of sequence b
 *  num_pages,   optional (all NULL or all set): ragged page lists.  When NULL,
 *  page_used,   page i of sequence b holds min(page_size, kv_len - i*page_size)
 *  page_start   tokens.  When set, sequence b has num_pages[b] pages, page i
 *               holds page_used[b*pt_stride_b+i] tokens whose first logical
 *               position is page_start[b*pt_stride_b+i].
 *  mask         optional additive key mask [B, T] (row stride mask_stride_b),
 *               indexed by logical token position, dtype mask_dtype
 *  softcap      tanh soft-capping of the scaled scores when > 0
 *  out          [B, Hq, D] strides out_stride_b, out_stride_h, in out_dtype: the
 *               query dtype, or HELM_DTYPE_FP32 (partial states that another
 *               device's results are merged with, see helm_merge_attention_states)
 *  lse          optional fp32 [B, Hq]
 *  workspace    >= helm_paged_decode_workspace_bytes(...) bytes, 256-byte aligned,
 *               holding the split-KV partial states; no initialisation needed
 *               (its first roundup(4*batch*num_kv_heads, 256) bytes are reserved).
 *               The call launches two kernels on `stream`: the decode kernel and,
 *               as its programmatic dependent, the merge of split pairs.
 *  max_kv_len_hint  upper bound on kv_lens (0 = unknown); sizes the grid
 */
int helm_paged_decode_attention(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                const void* kv_pool, int64_t pool_pages,
                                const int32_t* page_table, int64_t pt_stride_b, int max_pages,
                                const int32_t* kv_lens, const int32_t* num_pages,
                                const int32_t* page_used, const int32_t* page_start,
                                const void* mask, int mask_dtype, int64_t mask_stride_b,
                                void* out, int64_t out_stride_b, int64_t out_stride_h, float* lse,
                                void* workspace, int64_t workspace_bytes, int batch,
                                int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                int dtype, int out_dtype, float scale, float softcap,
                                int max_kv_len_hint, void* stream);

/*
 * Decode overlap, a setting of the calling host thread (default off; returns
 * the previous setting).  When on, helm_paged_decode_attention and
 * helm_paged_decode_attention_noalloc launch the decode kernel as a
 * programmatic dependent of the kernel before it on the stream (PDL): the
 * kernel is placed while that one still runs, reads kv_lens, num_pages and
 * page_table and starts loading K/V tiles outside each sequence's last page
 * early, but waits for it to finish before it reads q, the mask or a last
 * page, and before it writes anything.  Turn it on only where the kernel
 * immediately before each call does not write kv_lens, num_pages, page_used,
 * page_start or page_table, and writes no K/V page other than the sequences'
 * last pages (for example the fused append of the new token in a captured
 * decode step).  No counterpart in the reference.
 */
int helm_set_decode_overlap(int enable);

/*
 * Same computation and arguments as helm_paged_decode_attention (output in the
 * query dtype), without the workspace: for callers that cannot allocate device memory, such as a server
 * that gives all of HBM to its own pool at start-up (a later cudaMalloc would
 * fail or fragment it) or a decode loop that must not stall on the device-wide
 * synchronisation of cudaFree.  It has no counterpart in the reference (HELM
 * allocates freely through PyTorch).
 *
 * Scratch comes from a fixed 8 MiB array inside the library, held by every GPU
 * that loads it until exit; shapes needing more (see
 * helm_paged_decode_workspace_bytes) return HELM_ERR_WORKSPACE.  The first call
 * on a device sets up that device's scratch address: make it before any stream
 * capture.  All calls share the array, so calls that overlap on the GPU race;
 * keep them ordered on one stream.  Nothing in the array needs to start at
 * zero, and a call allocates nothing.
 */
int helm_paged_decode_attention_noalloc(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                        const void* kv_pool, int64_t pool_pages,
                                        const int32_t* page_table, int64_t pt_stride_b,
                                        int max_pages, const int32_t* kv_lens,
                                        const int32_t* num_pages, const int32_t* page_used,
                                        const int32_t* page_start, const void* mask,
                                        int mask_dtype, int64_t mask_stride_b, void* out,
                                        int64_t out_stride_b, int64_t out_stride_h, float* lse,
                                        int batch, int num_q_heads, int num_kv_heads,
                                        int head_dim, int page_size, int dtype, float scale,
                                        float softcap, int max_kv_len_hint, void* stream);

/*
 * Fused KV append: optional per-head RMSNorm of q and k (fp32 variance,
 * eps, weight * normed.to(dtype)), optional rotary embedding with the
 * caller's cos/sin tables (HF rotate_half convention), then the K and V rows
 * of every token are written into the page pool at row slot_rows[token] =
 * slot*page_size + row_in_page (a negative entry skips the token).  The
 * processed q is written to q_out.
 *
 * Replaces the q_norm/k_norm + apply_rotary_pos_emb of the patched attention
 * forwards (helm/runtime/kv_offload.py:368-373) and the page writes of
 * KVCacheManager.append_decode / append_prefill (helm/runtime/kv_cache.py:
 * 113-171).
 *
 *  q, k, v      [N tokens, H, D] with token strides q_stride_t, k_stride_t,
 *               v_stride_t and head strides q_stride_h, k_stride_h, v_stride_h
 *  q_norm_w,    [D] RMSNorm weights (NULL: no norm)
 *  k_norm_w
 *  cos, sin     [N, D] rotary tables in the model dtype (NULL: no rotation),
 *               token stride rope_stride_t
 *  q_out        [N, Hq, D], strides q_out_stride_t, q_out_stride_h (may be NULL)
 *  k_out, v_out optional copies of the processed K/V rows ([N, Hkv, D] dense)
 * Norm, RoPE and q/k/v outputs need bf16/fp16 and head_dim 64, 128 or 256; a
 * plain page write (all of them NULL) also takes fp32 and any head_dim.
 */
int helm_kv_append(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                   int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                   int64_t v_stride_h, const void* q_norm_w, const void* k_norm_w, float eps,
                   const void* cos, const void* sin, int64_t rope_stride_t, void* q_out,
                   int64_t q_out_stride_t, int64_t q_out_stride_h, void* k_out, void* v_out,
                   void* kv_pool, int64_t pool_pages, const int64_t* slot_rows, int num_tokens,
                   int num_q_heads, int num_kv_heads, int head_dim, int page_size, int dtype,
                   void* stream);

/*
 * Copies whole page slots between two pools (device <-> pinned host, or
 * device <-> device): dst_pool[dst_slots[i]] = src_pool[src_slots[i]] for
 * i < n.  Slot lists are HOST int64 arrays; runs of consecutive slots are
 * merged into one cudaMemcpyAsync each.  Both pools must be reachable from
 * the copy engine (device memory or page-locked host memory).
 *
 * Replaces KVAllocator.move_page (helm/runtime/kv_allocator.py:95-144) and the
 * per-page CPU->GPU stream copies of perform_streaming_attention
 * (helm/runtime/kv_cache.py:482-530, :624-659).
 */
int helm_copy_pages(void* dst_pool, const void* src_pool, int64_t page_bytes,
                    const int64_t* dst_slots, const int64_t* src_slots, int64_t n, void* stream);

/*
 * Gathers paged K/V into dense tensors K_out, V_out [B, Hkv, T_max, D]
 * (token positions >= kv_lens[b] are zero-filled).  Used where a dense
 * library attention is called on paged data (chunked prefill).
 *
 * Replaces the torch.cat page concatenation of perform_streaming_attention
 * (helm/runtime/kv_cache.py:563-564) and _decode_batched
 * (helm/runtime/kv_offload.py:160-171).
 */
int helm_gather_kv(const void* kv_pool, int64_t pool_pages, const int32_t* page_table,
                   int64_t pt_stride_b, int max_pages, const int32_t* kv_lens, void* k_out,
                   void* v_out, int batch, int num_kv_heads, int head_dim, int page_size,
                   int t_max, int dtype, void* stream);

/*
 * Chunk-prefill attention straight over the page pool: for every sequence b,
 * the q_len queries of the chunk (already appended: query i sits at position
 * kv_lens[b] - q_len + i) attend over keys 0 .. kv_lens[b]-1 of the pages in
 * page_table row b:
 *     out = softmax(softcap(scale * q K^T) + mask [+ causal limit]) V
 * fp32 accumulation and softmax state, output in the query dtype.
 *
 * Replaces the q_len > 1 branch of perform_streaming_attention
 * (helm/runtime/kv_cache.py:469-555) as called by _stream_prefill_batched
 * (helm/runtime/kv_offload.py:206-227).
 *
 *  q           [B, Hq, q_len, D] with strides q_stride_b/_h/_s (elements; even)
 *  kv_pool     [pool_pages, 2, Hkv, page_size, D]; page_size a multiple of 16
 *  page_table  int32 [B, >= max_pages] (row stride pt_stride_b), kv_lens int32 [B]
 *  kv_starts   optional int32 [B]: key j is visible to sequence b's rows only if
 *              j >= kv_starts[b].  HELM's key-padding mask of a left-padded
 *              prompt (helm/runtime/pipeline_runtime.py:107-111) passed as a
 *              key range: the padded keys' tiles are skipped and no mask is
 *              read.  NULL: every key from 0.
 *  mask        optional additive mask [B or 1, 1, q_len, >= max kv_lens] with
 *              strides mask_stride_b (0 to broadcast) and mask_stride_q, last
 *              stride 1; fp32, bf16 or fp16
 *  causal      1: key j is visible to query i only if j <= kv_lens[b]-q_len+i
 *  softcap     > 0: scores become softcap * tanh(scores / softcap) before the mask
 *  out         [B, Hq, q_len, D] with strides out_stride_b/_h/_s (multiples of
 *              4 elements; 8-byte aligned base)
 *  workspace   helm_paged_prefill_workspace_bytes(...) bytes, 256-byte aligned,
 *              any contents (may be NULL when that size is 0)
 *  max_kv_len  the largest kv_lens entry: it sizes the split of the key range
 *              (results do not depend on it)
 * A row that sees no key gets zeros.  dtype: HELM_DTYPE_BF16 or FP16;
 * head_dim 64 or 128.  Launches the prefill kernel and, when the key range is
 * split, its merge kernel as a programmatic dependent.
 */
int64_t helm_paged_prefill_workspace_bytes(int batch, int q_len, int num_q_heads,
                                           int num_kv_heads, int head_dim, int dtype,
                                           int max_kv_len);
int helm_paged_prefill_attention(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                 int64_t q_stride_s, const void* kv_pool, int64_t pool_pages,
                                 const int32_t* page_table, int64_t pt_stride_b, int max_pages,
                                 const int32_t* kv_lens, const int32_t* kv_starts,
                                 const void* mask, int mask_dtype, int64_t mask_stride_b,
                                 int64_t mask_stride_q, void* out, int64_t out_stride_b,
                                 int64_t out_stride_h, int64_t out_stride_s, void* workspace,
                                 int64_t workspace_bytes, int batch, int q_len,
                                 int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                 int dtype, int causal, float scale, float softcap, int max_kv_len,
                                 void* stream);

/*
 * Merges R partial attention states over disjoint key ranges:
 *     M = max_r lse[r];  w_r = exp(lse[r] - M)
 *     out = sum_r w_r * o[r] / sum_r w_r,   lse_out = M + log(sum_r w_r)
 * Part r's O is [rows, D] at o_parts + r*o_part_stride elements (dtype o_dtype:
 * fp32, bf16 or fp16) and its LSE [rows] at lse_parts + r*lse_part_stride
 * (fp32), so one buffer gathered from R devices can be merged in place.  out
 * [rows, D] in out_dtype; lse_out optional fp32 [rows].  rows = batch *
 * num_q_heads.  A part with lse = -inf contributes nothing.
 *
 * No single-device counterpart in the reference (it is single-GPU); this is
 * the cross-rank form of its running-max rescale (helm/runtime/kv_cache.py:
 * 523-529) used by the sequence-split path.
 */
int helm_merge_attention_states(const void* o_parts, int o_dtype, int64_t o_part_stride,
                                const float* lse_parts, int64_t lse_part_stride, int num_parts,
                                int64_t rows, int head_dim, void* out, int out_dtype,
                                float* lse_out, void* stream);

/*
 * Sequence-split exchange over peer memory (one process per GPU, one node).
 *
 * helm_ipc_alloc      cudaMalloc + zero fill of an exchange buffer on the
 *                     current device (bytes from helm_peer_exchange_bytes).
 * helm_ipc_get_handle writes the buffer's CUDA IPC handle
 *                     (helm_ipc_handle_bytes() bytes) for the other ranks.
 * helm_ipc_open       maps another rank's buffer from its handle.
 * helm_ipc_close / helm_ipc_free   undo open / alloc.
 * helm_ipc_zero       re-zeroes a buffer (after a timeout, on every rank).
 *
 * helm_seq_exchange_merge: bufs[world] are every rank's exchange buffer as
 * mapped in this process (own buffer at bufs[rank]).  Stores this rank's
 * partial state (o_part fp32 [rows, head_dim], 8-byte aligned; lse_part fp32
 * [rows]) into slot `rank` of every buffer through NVLink, each value paired
 * with the step's epoch in one 8-byte word, polls (at most timeout_ns) its own
 * buffer until every rank's words of the step have arrived and merges:
 *     M = max_r lse_r,  out = sum_r e^(lse_r - M) o_r / sum_r e^(lse_r - M)
 * out [rows, head_dim] in out_dtype; lse_out optional fp32 [rows].  Every rank
 * must make the same sequence of calls with the same rows and head_dim.  A
 * wait that runs out sets HELM_DEV_TIMEOUT (helm_get_device_status); all
 * ranks must then helm_ipc_zero their buffers before the next call.
 * world <= 8, head_dim % 4 == 0.
 *
 * No counterpart in the reference (single GPU); this replaces an all-gather
 * of the packed states followed by helm_merge_attention_states.
 */
int64_t helm_peer_exchange_bytes(int64_t rows, int head_dim, int world);
int helm_ipc_alloc(int64_t bytes, void** ptr_out);
int helm_ipc_free(void* ptr);
int helm_ipc_zero(void* ptr, int64_t bytes, void* stream);
int helm_ipc_handle_bytes(void);
int helm_ipc_get_handle(const void* ptr, void* handle_out);
int helm_ipc_open(const void* handle, void** ptr_out);
int helm_ipc_close(void* ptr);
int helm_seq_exchange_merge(void* const* bufs, int rank, int world, const float* o_part,
                            const float* lse_part, int64_t rows, int head_dim, void* out,
                            int out_dtype, float* lse_out, uint64_t timeout_ns, void* stream);

/*
 * One matrix-vector product of a decode step with its neighbours fused in
 * (the GPU stage around the attention call; HELM runs these as the eager HF
 * modules of a stage, executor.py:420 / decode_tracer.py:274-336):
 *   y[b] = W . rmsnorm(x[b])        when norm_w != NULL (eps: the norm's eps)
 *   y[b] = silu(W x[b]) * (W2 x[b]) when w2 != NULL (SwiGLU)
 *   y[b] = residual[b] + W x[b]     when residual != NULL
 * (norm and SwiGLU/residual may be combined), rounding to `dtype` where HF's
 * eager modules do.  x [batch, k] (row stride x_stride elements), W / W2
 * [n, k] row-major 16-byte aligned, k % 16 == 0, batch <= 16, x of all batch
 * rows fits the CTA's shared memory (about batch * k * 2 bytes <= 190 KiB, less
 * for 8+ rows); y [batch, n] (row stride y_stride) in dtype, or fp32 when
 * y_fp32.  y may alias residual.  dtype: HELM_DTYPE_BF16 or HELM_DTYPE_FP16.
 */
int helm_decode_gemv(const void* x, int64_t x_stride, const void* norm_w, float eps,
                     const void* w, const void* w2, int64_t n, int64_t k, const void* residual,
                     int64_t res_stride, void* y, int64_t y_stride, int y_fp32, int batch,
                     int dtype, void* stream);

/*
 * Row-parallel projection of tensor-parallel decode with its all-reduce in
 * the same kernel: y[b] = residual[b] + sum over ranks r of W_r x_r[b], where
 * this rank holds W_r [n, k] (its slice of the input dim) and x_r [batch, k].
 * Each CTA stores its rows' fp32 partials into every rank's buffer over
 * NVLink as {value, epoch} words, polls its own buffer (at most timeout_ns)
 * for the other ranks' partials of the same rows and sums them in rank order,
 * so every rank gets the same y.  bufs[world]: every rank's exchange buffer
 * (helm_decode_gemv_allreduce_bytes(n, max batch, world) bytes, zeroed, from
 * helm_ipc_alloc / helm_ipc_open), one buffer per (n, batch) use.  All ranks
 * make the same calls in the same order.  No counterpart in the reference
 * (single GPU); replaces o_proj / down_proj + an all-reduce + the residual add.
 */
int helm_decode_gemv_allreduce(void* const* bufs, int rank, int world, const void* x,
                               int64_t x_stride, const void* w, int64_t n, int64_t k,
                               const void* residual, int64_t res_stride, void* y,
                               int64_t y_stride, int batch, int dtype, uint64_t timeout_ns,
                               void* stream);
int64_t helm_decode_gemv_allreduce_bytes(int64_t n, int batch, int world);

#ifdef __cplusplus
}
#endif

#endif /* HELM_B200_H_ */
