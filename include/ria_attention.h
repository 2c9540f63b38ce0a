/*
 * router-ia B200 attention library: C ABI.
 *
 * Drop-in device kernels for router-ia's stateful hybrid attention path
 * (v2/src/router_ia/qwen36_attention_cache.py).  Every entry point:
 *   - takes raw device pointers, element strides and sizes (no framework types);
 *   - only enqueues work on `stream` (no host synchronisation, no allocation);
 *   - returns RIA_OK (0) or a nonzero status, with a message available from
 *     ria_last_error_string() (per host thread).
 * The Python host side maps a nonzero status to RuntimeError/ValueError, the
 * exception types the reference raises for the same conditions.
 *
 * Shapes are fixed by the Qwen3.6-35B-A3B attention layers:
 *   Gated DeltaNet: 16 key heads, 32 value heads, head dim 128,
 *                   conv channels 8192 (q 2048 | k 2048 | v 4096), conv kernel 4.
 *   GQA:            16 query heads, 2 KV heads, head dim 256, RoPE on dims [0,64).
 */
#ifndef RIA_ATTENTION_H_
#define RIA_ATTENTION_H_

#include <stdint.h>

#if defined(__GNUC__)
#define RIA_API __attribute__((visibility("default")))
#else
#define RIA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define RIA_ABI_VERSION 1

#define RIA_OK 0
#define RIA_ERR_INVALID 1     /* bad argument: shape, stride, alignment, range */
#define RIA_ERR_CUDA 2        /* a CUDA runtime call or launch failed */
#define RIA_ERR_UNSUPPORTED 3 /* device or configuration not supported */

/* Opaque CUDA stream (cudaStream_t); NULL is the legacy default stream. */
typedef void* ria_stream_t;

/* Message describing the last failure on the calling host thread. */
RIA_API const char* ria_last_error_string(void);
RIA_API int ria_abi_version(void);

/* Reads (and optionally clears) the device error word that kernels set when a
 * bounded wait gives up, a block-table entry or slot is out of range, or a
 * sequence needs more KV splits than a GQA decode launch provides.
 * Synchronous.  *code_out = 0 means no device-side error was recorded;
 * otherwise the first code set: 1, 2 or 5 a bounded wait gave up (DeltaNet
 * decode, GQA decode, prefill kernels), 3 a block id outside the pool, 6 a
 * state slot outside the pool, 7 a too-small GQA split plan (that sequence was
 * left untouched: no pool, workspace or output write), 8 the MoE block's down
 * phase gave up waiting for a unit's gate/up tiles. */
RIA_API int ria_device_error(int clear, unsigned int* code_out);

/* ------------------------------------------------------------------------
 * K1: Gated DeltaNet decode step, batched over sequences.
 *
 * Replaces, per layer and per sequence, the body of
 *   _causal_conv1d_step      qwen36_attention_cache.py:176-221
 *   _linear_stateful         qwen36_attention_cache.py:232-271 (after the input
 *                            projections, before out_proj)
 *   gated_rmsnorm            qwen36_gated_norm_probe.py:19-36
 * in one pass over each head's fp32 128x128 state.
 *
 * Inputs are the projection outputs of the layer for B sequences, bf16:
 *   mixed [B, 8192] (row stride mixed_stride): in_proj_qkv output
 *   z     [B, 4096] (z_stride):  in_proj_z output
 *   b     [B, 32]   (b_stride):  in_proj_b output  (beta = sigmoid(b))
 *   a     [B, 32]   (a_stride):  in_proj_a output
 * Parameters: conv_weight [8192, 4] bf16 (the checkpoint's [8192,1,4]),
 *   a_log [32] f32, dt_bias [32] f32, norm_weight [128] f32.
 * State (updated in place): conv_state [slots, 8192, 4] bf16 (the last four
 *   conv inputs, current token last), rec_state [slots, 32, 128, 128] f32
 *   indexed [head][k][v] (16-byte aligned).  Sequence i uses slot
 *   slots[i] (slots == NULL: slot i).
 * Output: out [B, 4096] bf16 (row stride out_stride): the gated RMSNorm output
 *   that feeds out_proj.
 */
RIA_API int ria_gdn_decode_step(const void* mixed, int64_t mixed_stride, const void* z, int64_t z_stride, const void* b,
                        int64_t b_stride, const void* a, int64_t a_stride, const void* conv_weight,
                        const float* a_log, const float* dt_bias, const float* norm_weight, void* conv_state,
                        float* rec_state, const int32_t* slots, int32_t num_slots, void* out, int64_t out_stride,
                        int32_t batch, ria_stream_t stream);

/* ------------------------------------------------------------------------
 * K3: paged, ragged, split-KV GQA decode step with KV append.
 *
 * Replaces, per layer and per sequence, _full_stateful after the q/k/v
 * projections and before o_proj (qwen36_attention_cache.py:298-318):
 * per-head q/k RMSNorm (the (1+w) form, qwen36_op_probe.py:55-67), partial RoPE
 * on dims [0,64) (_apply_rope, :137-162), the KV append (_append_full_kv,
 * :334-373), softmax(q K^T / 16) V over the 8 query heads of each KV head and
 * the sigmoid output gate.
 *
 * q     [B, 16*512] bf16 (q_stride): q_proj output; head h holds q in
 *        [512h, 512h+256) and the gate in [512h+256, 512h+512).
 * k, v  [B, 2*256] bf16 (k_stride, v_stride): k_proj / v_proj outputs.
 * q_norm_weight, k_norm_weight [256] f32; inv_freq [32] f32 RoPE inverse
 *        frequencies (theta 1e7 over 64 rotary dims).
 * k_pool, v_pool [2, pool_tokens, 256] bf16: paged cache, 64-token blocks;
 *        logical block j of sequence i is physical block
 *        block_table[i*block_table_stride + j].  16-byte aligned.
 * seq_lens [B]: cached tokens before this step; the new token is written at
 *        index seq_lens[i].  positions [B]: absolute RoPE positions.  For a
 *        single sequence (batch 1) either may be NULL, and the host values
 *        seq_len0 / position0 are used instead (the reference's per-layer
 *        length and tokens_seen).
 * out   [B, 4096] bf16 (out_stride): gated attention output feeding o_proj.
 * workspace: scratch of at least ria_gqa_decode_workspace_bytes(B, max_splits)
 *        bytes (split partials), 16-byte aligned.
 * split_pages: KV blocks per split (>= 1); max_splits >= ceil(blocks / split_pages)
 *        for the longest sequence after the append.
 */
RIA_API int64_t ria_gqa_decode_workspace_bytes(int32_t batch, int32_t max_splits);
RIA_API int ria_gqa_decode_paged(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                         int64_t v_stride, const float* q_norm_weight, const float* k_norm_weight,
                         const float* inv_freq, void* k_pool, void* v_pool, int64_t pool_tokens,
                         const int32_t* block_table, int32_t block_table_stride, const int32_t* seq_lens,
                         const int32_t* positions, int32_t seq_len0, int32_t position0, void* out,
                         int64_t out_stride, void* workspace,
                         int64_t workspace_bytes, int32_t batch, int32_t split_pages, int32_t max_splits,
                         ria_stream_t stream);

/* Allocation-free variant of ria_gqa_decode_paged.  No counterpart in the
 * reference (router-ia has no device kernels); it exists for callers that
 * cannot allocate device memory where they decode: host runtimes that carve
 * all GPU memory into their own pools up front, processes held to a hard VRAM
 * budget, plugin interfaces that pass inputs and outputs but no workspace --
 * for them a cudaMalloc at decode time fails, breaks the budget or bypasses
 * the host's accounting.  Same arguments as
 * ria_gqa_decode_paged without the workspace: the split partials go to a
 * fixed RIA_GQA_STATIC_SCRATCH_BYTES array inside the library, present on
 * every GPU that loads the library until the process exits.  Calls needing
 * more (ria_gqa_decode_workspace_bytes(batch, max_splits) larger than that)
 * fail with RIA_ERR_INVALID.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make that
 * first call before any stream capture.  All calls on a device share the
 * array: calls whose kernels can overlap on the GPU race; calls ordered on one
 * stream do not.  Allocates nothing (no cudaMalloc/cudaFree). */
#define RIA_GQA_STATIC_SCRATCH_BYTES (4u << 20)
RIA_API int ria_gqa_decode_paged_static(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                                        const void* v, int64_t v_stride, const float* q_norm_weight,
                                        const float* k_norm_weight, const float* inv_freq, void* k_pool,
                                        void* v_pool, int64_t pool_tokens, const int32_t* block_table,
                                        int32_t block_table_stride, const int32_t* seq_lens,
                                        const int32_t* positions, int32_t seq_len0, int32_t position0, void* out,
                                        int64_t out_stride, int32_t batch, int32_t split_pages, int32_t max_splits,
                                        ria_stream_t stream);

/* Append one token's post-RoPE K and V rows per sequence to the paged cache:
 * the storage step of _append_full_kv (qwen36_attention_cache.py:365-373; the
 * reference's limit checks, :344-363, stay with the caller).  The GQA decode
 * and prefill kernels fuse this write into their attention pass; this entry
 * point serves callers that compute K/V themselves.
 * k_new, v_new [B, 512] (2 KV heads x 256), bf16 or, with inputs_f32, f32
 *        (rounded to bf16), rows 16-byte aligned (k_stride / v_stride in
 *        elements).
 * k_pool, v_pool, block_table, block_table_stride: as ria_gqa_decode_paged.
 * seq_lens [B]: the row index each token goes to (the cached length); NULL
 *        for batch 1 with seq_len0.
 * A block id outside the pool is recorded as device error 3 and that
 * sequence is left untouched. */
RIA_API int ria_kv_append_paged(const void* k_new, int64_t k_stride, const void* v_new, int64_t v_stride,
                                int32_t inputs_f32, void* k_pool, void* v_pool, int64_t pool_tokens,
                                const int32_t* block_table, int32_t block_table_stride, const int32_t* seq_lens,
                                int32_t seq_len0, int32_t batch, ria_stream_t stream);

/* Split size heuristic used by the Python host: KV blocks per split so that the
 * grid holds a few waves of CTAs for `total_blocks` blocks of work. */
RIA_API int32_t ria_gqa_decode_split_pages(int64_t total_blocks, int32_t num_kv_heads);

/* ------------------------------------------------------------------------
 * K2: chunked Gated DeltaNet prefill (chunk 64, WY/UT form) on tcgen05.
 *
 * Replaces gated_delta_chunk_initial (qwen36_linear_attention_hf.py:91-100,
 * transformers torch_chunk_gated_delta_rule with use_qk_l2norm_in_kernel) and
 * the token-by-token recurrence it equals (qwen36_attention_cache.py:256-266)
 * for a whole prompt: q and k are L2-normalised in-kernel, q scaled by
 * 128^-0.5, value head h reads key head h / (num_v_heads / num_k_heads).
 *
 * q, k [B, T, num_k_heads, 128] bf16 (element strides *_stride_b / *_stride_t,
 *      head dims contiguous, 16-byte aligned); v [B, T, num_v_heads, 128] bf16;
 * g    [B, T, num_v_heads] f32 log decay (-exp(A_log) softplus(a + dt_bias));
 * beta [B, T, num_v_heads] f32 (sigmoid(b)); both with strides gb_stride_*;
 * initial_state [B, num_v_heads, 128 k, 128 v] f32 or NULL (zeros);
 * final_state   same layout (may alias initial_state): the state after T tokens,
 *      in the decode kernel's layout;
 * out  [B, T, num_v_heads, 128] bf16 (o_stride_b / o_stride_t);
 * workspace: 16-byte aligned device scratch for the per-chunk matrices (W, U,
 *      the causal score tile and the chunk scalars, 41,600 bytes per sequence,
 *      value head and chunk).  ria_gdn_chunk_prefill_workspace_bytes() gives the
 *      size for the whole prompt; a smaller workspace (at least one chunk for
 *      every sequence and head) makes the call run the prompt in blocks of
 *      chunks, carrying the state through final_state. */
RIA_API int64_t ria_gdn_chunk_prefill_workspace_bytes(int32_t batch, int32_t seq_len, int32_t num_v_heads);
RIA_API int ria_gdn_chunk_prefill(const void* q, int64_t q_stride_b, int64_t q_stride_t, const void* k,
                                  int64_t k_stride_b, int64_t k_stride_t, const void* v, int64_t v_stride_b,
                                  int64_t v_stride_t, const float* g, const float* beta, int64_t gb_stride_b,
                                  int64_t gb_stride_t, const float* initial_state, float* final_state, void* out,
                                  int64_t o_stride_b, int64_t o_stride_t, void* workspace, int64_t workspace_bytes,
                                  int32_t batch, int32_t seq_len, int32_t num_k_heads, int32_t num_v_heads,
                                  ria_stream_t stream);

/* ------------------------------------------------------------------------
 * K4: GQA prefill of T new tokens per sequence (batch B, same T).
 *
 * Replaces T token-by-token _full_stateful calls (qwen36_attention_cache.py:
 * 285-324; prompt loop qwen36_chat_batch.py:255-258) for one layer: q/k RMSNorm
 * (1+w), partial RoPE at positions[b] + t, the new K/V appended to the paged
 * cache at index seq_lens[b] + t, causal softmax(q K^T / 16) V over the cached
 * prefix and the new tokens, sigmoid gate.
 *
 * q [B, T, 16*512] bf16 (q | gate per head), k, v [B, T, 2*256] bf16, with
 * element strides *_stride_b / *_stride_t (16-byte aligned); pools, block table
 * as for ria_gqa_decode_paged (blocks for all T new tokens must be mapped);
 * seq_lens [B] cached tokens before the prompt; positions [B] absolute
 * position of prompt token 0; out [B, T, 4096] bf16; workspace at least
 * ria_gqa_prefill_workspace_bytes(B, T) bytes (normalised q). */
RIA_API int64_t ria_gqa_prefill_workspace_bytes(int32_t batch, int32_t seq_len);
RIA_API int ria_gqa_prefill(const void* q, int64_t q_stride_b, int64_t q_stride_t, const void* k, int64_t k_stride_b,
                            int64_t k_stride_t, const void* v, int64_t v_stride_b, int64_t v_stride_t,
                            const float* q_norm_weight, const float* k_norm_weight, const float* inv_freq,
                            void* k_pool, void* v_pool, int64_t pool_tokens, const int32_t* block_table,
                            int32_t block_table_stride, const int32_t* seq_lens, const int32_t* positions, void* out,
                            int64_t out_stride_b, int64_t out_stride_t, void* workspace, int64_t workspace_bytes,
                            int32_t batch, int32_t seq_len, ria_stream_t stream);

/* ------------------------------------------------------------------------
 * Row kernels of the DeltaNet prompt path around K2 (the per-token arithmetic
 * of _linear_stateful, qwen36_attention_cache.py:176-271, for T tokens).
 */

/* Causal depthwise conv (kernel 4) + SiLU over T tokens in bf16, continuing
 * from conv_state [B, channels, 4] (updated to the last four inputs):
 * x, out [B, T, channels] bf16 with element strides. */
RIA_API int ria_conv1d_prefill(const void* x, int64_t x_stride_b, int64_t x_stride_t, void* conv_state,
                               const void* weight, void* out, int64_t out_stride_b, int64_t out_stride_t,
                               int32_t batch, int32_t seq_len, int32_t channels, ria_stream_t stream);

/* g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) for rows x heads:
 * a, b bf16 rows (strides), g, beta f32 [rows, heads] (qwen36_attention_cache.py:242-250). */
RIA_API int ria_gdn_gates(const void* a, int64_t a_stride, const void* b, int64_t b_stride, const float* a_log,
                          const float* dt_bias, float* g, float* beta, int32_t rows, int32_t heads,
                          ria_stream_t stream);

/* Gated RMSNorm per 128-wide head (qwen36_gated_norm_probe.py:19-36):
 * out = w * o * rsqrt(mean(o^2) + 1e-6) * silu(z); o, z, out bf16 rows. */
RIA_API int ria_gated_rmsnorm(const void* o, int64_t o_stride, const void* z, int64_t z_stride, const float* weight,
                              void* out, int64_t out_stride, int32_t rows, int32_t heads, ria_stream_t stream);

/* Diagnostic (no counterpart in the reference): one CTA computes
 * d[128 x n] = a[128 x k] * b[k x n] (row-major fp32 in/out, bf16 operands)
 * with tcgen05 MMAs whose A / B operands are staged K-major (0) or MN-major (1)
 * in 128-byte-swizzled shared memory -- the operand layouts the prefill
 * kernels use.  a_mn_major: 0 = A K-major in shared memory, 1 = MN-major,
 * 2 = A in tensor memory (16-bit pairs per 32-bit column); adding 4 makes both
 * operands fp16 instead of bf16.  n, k in {64, 128}.
 * Used by the tests to pin the descriptor encodings against a reference
 * matmul. */
RIA_API int ria_umma_selftest(int32_t a_mn_major, int32_t b_mn_major, int32_t n, int32_t k, const float* a,
                              const float* b, float* d, ria_stream_t stream);

/* ------------------------------------------------------------------------
 * Small fused row kernels used around the projections.
 */

/* out[B, n] (bf16) = rmsnorm(x[B, n] f32) * (1 + weight[n]); eps 1e-6.
 * Replaces rmsnorm (qwen36_op_probe.py:55-67) on the layer input. */
RIA_API int ria_rmsnorm_rows(const float* x, int64_t x_stride, const float* weight, void* out, int64_t out_stride, int32_t rows,
                     int32_t n, ria_stream_t stream);
/* The same norm with an fp16 output: the input of the fp16 in-projections
 * (router-ia's CUDA path runs its projections on fp16 weights,
 * qwen36_cached_loop.py:552-557). */
RIA_API int ria_rmsnorm_rows_f16(const float* x, int64_t x_stride, const float* weight, void* out,
                                 int64_t out_stride, int32_t rows, int32_t n, ria_stream_t stream);

/* Small-batch projections (batch <= 8), weight-streaming GEMVs with the
 * neighbouring row ops fused (the "projection fusion" of the layer steps):
 *
 * ria_rmsnorm_gemv: out[b, n] (bf16) = W[n, :] . fp16(rmsnorm(x[b]) * (1 + norm_w)),
 *   the layer's input RMSNorm (qwen36_op_probe.py:55-67) and its fused
 *   in-projection (qwen36_attention_cache.py:228-240 DeltaNet, :289-297 GQA);
 *   x [batch, k] f32, W [n, k] fp16 (row stride w_stride), fp32 accumulation,
 *   out bf16 -- the activations the ria_rmsnorm_rows_f16 + fp16 GEMM path
 *   produces.
 * ria_gemv_residual: out[b, n] (f32) = x0[b, n] + bf16(W[n, :] . a[b]), the
 *   out-projection and the residual add that end the layer (:272-277, :318-321);
 *   a [batch, k] bf16, x0 / out f32.
 * k a multiple of 8 with 16-byte aligned rows; batch * k * 2 <= 96 KiB. */
RIA_API int ria_rmsnorm_gemv(const float* x, int64_t x_stride, const float* norm_weight, const void* w,
                             int64_t w_stride, void* out, int64_t out_stride, int32_t batch, int32_t n, int32_t k,
                             ria_stream_t stream);
RIA_API int ria_gemv_residual(const void* a, int64_t a_stride, const void* w, int64_t w_stride, const float* x0,
                              int64_t x0_stride, float* out, int64_t out_stride, int32_t batch, int32_t n, int32_t k,
                              ria_stream_t stream);

/* Whole decode layer steps for batch <= 8 in one call: the launches a
 * DeltaNet or GQA layer makes through ria_rmsnorm_gemv, ria_gdn_decode_step /
 * ria_gqa_decode_paged and ria_gemv_residual, issued back to back from C with
 * the intermediates in `scratch` (identical results).  For callers that step
 * one layer per call from an interpreter, as router-ia's run_forward_token
 * does through step_attention (qwen36_chat_batch.py:181-207;
 * qwen36_attention_cache.py:224-324 for the layer bodies): the host work of
 * three or four separate foreign calls per layer exceeds a batch-1 layer's
 * GPU time.  x [batch, 2048] f32 is the layer input and out [batch, 2048] f32
 * its residual output (out may not alias x); weights, state and cache
 * arguments are those of the separate entry points (w_in fp16 [n_in, 2048],
 * w_out bf16 [2048, 4096]).  scratch: at least the *_scratch_bytes bytes,
 * 256-byte aligned, not shared by calls that overlap on the GPU. */
RIA_API int64_t ria_deltanet_layer_decode_scratch_bytes(int32_t batch);
RIA_API int ria_deltanet_layer_decode(const float* x, int64_t x_stride, const float* in_norm, const void* w_in,
                                      int64_t w_in_stride, const void* conv_weight, const float* a_log,
                                      const float* dt_bias, const float* norm_weight, const void* w_out,
                                      int64_t w_out_stride, void* conv_state, float* rec_state, const int32_t* slots,
                                      int32_t num_slots, float* out, int64_t out_stride, void* scratch,
                                      int64_t scratch_bytes, int32_t batch, ria_stream_t stream);
RIA_API int64_t ria_gqa_layer_decode_scratch_bytes(int32_t batch, int32_t max_splits);
RIA_API int ria_gqa_layer_decode(const float* x, int64_t x_stride, const float* in_norm, const void* w_in,
                                 int64_t w_in_stride, const float* q_norm_weight, const float* k_norm_weight,
                                 const float* inv_freq, void* k_pool, void* v_pool, int64_t pool_tokens,
                                 const int32_t* block_table, int32_t block_table_stride, const int32_t* seq_lens,
                                 const int32_t* positions, int32_t seq_len0, int32_t position0, const void* w_out,
                                 int64_t w_out_stride, float* out, int64_t out_stride, void* scratch,
                                 int64_t scratch_bytes, int32_t batch, int32_t split_pages, int32_t max_splits,
                                 ria_stream_t stream);

/* out[B, n] f32 = x0[B, n] f32 + proj[B, n] bf16: the residual add that ends
 * _linear_stateful / _full_stateful (qwen36_attention_cache.py:276-277, 320-321). */
RIA_API int ria_residual_add(const float* x0, int64_t x0_stride, const void* proj, int64_t proj_stride, float* out,
                     int64_t out_stride, int32_t rows, int32_t n, ria_stream_t stream);

/* ------------------------------------------------------------------------
 * MoE block of a decode step (hidden 2048, expert and shared-expert
 * intermediate 512), for a batch of tokens: batched_moe_step
 * (qwen36_chat_batch.py:127-178) with route (qwen36_router.py:96-133):
 *
 *   moe_in = rmsnorm(residual) * (1 + post_norm_weight)       (eps 1e-6)
 *   logits = moe_in . router_weight^T  (fp32); top_k largest; softmax over them
 *   out    = residual + sum_j w_j * down_j(silu(gate_j moe_in) * up_j moe_in)
 *                     + sigmoid(moe_in . shared_gate_weight)
 *                       * shared_down(silu(shared_gate_proj moe_in) * shared_up_proj moe_in)
 *
 * residual / out [batch, 2048] f32 (row strides in elements, multiples of 4;
 * out may alias residual); weights bf16 as in the checkpoint:
 * post_norm_weight [2048], router_weight [E, 2048], shared_gate_weight
 * [2048], experts_gate / experts_up [E, 512, 2048] and experts_down
 * [E, 2048, 512] (each expert's tensors stacked), shared_gate_proj /
 * shared_up_proj [512, 2048], shared_down_proj [2048, 512].  Also written:
 * expert_ids [batch, top_k] int32 and expert_weights [batch, top_k] f32 (the
 * routing, largest logit first; equal logits pick the lower expert id) and
 * shared_gate [batch] f32.  batch * top_k <= 2048, E <= 1024, top_k <= 16;
 * workspace (16-byte aligned, device) of ria_moe_workspace_bytes bytes,
 * zero-filled before its first use (it holds hand-off counters that every
 * call returns to zero; one workspace serves one stream at a time).
 * Experts no token chose are not read.  Deterministic: fixed-order sums. */
RIA_API int64_t ria_moe_workspace_bytes(int32_t batch, int32_t num_experts, int32_t top_k);
RIA_API int ria_moe_decode(const float* residual, int64_t residual_stride, const void* post_norm_weight,
                           const void* router_weight, const void* shared_gate_weight, const void* experts_gate,
                           const void* experts_up, const void* experts_down, const void* shared_gate_proj,
                           const void* shared_up_proj, const void* shared_down_proj, float* out, int64_t out_stride,
                           int32_t* expert_ids, float* expert_weights, float* shared_gate, void* workspace,
                           int64_t workspace_bytes, int32_t batch, int32_t num_experts, int32_t top_k,
                           ria_stream_t stream);

/* Element kernels of the prompt-prefill MoE path, whose expert projections
 * run as grouped library GEMMs over the (token, slot) pairs sorted by expert
 * (batched_moe_step, qwen36_chat_batch.py:127-178, for many tokens at once):
 * ria_moe_prompt_norm: h [rows, 2048] f32 and h_bf16 = x rsqrt(mean(x^2) +
 *   1e-6) (1 + post_norm_weight) (bf16 weight), x [rows, 2048] f32.
 * ria_silu_mul_bf16: out[i] = bf16(silu(gate[i]) * up[i]), n bf16 elements
 *   (a multiple of 8, 16-byte aligned buffers).
 * ria_moe_prompt_combine: out[t] = x[t] + (sum_{j < top_k} weights[t, j] *
 *   expert_out[sorted_position[t, j]] + shared_gate[t] * shared_out[t]), the
 *   slots summed in order; expert_out [pairs, 2048] and shared_out [rows,
 *   2048] bf16, weights [rows, top_k] f32, sorted_position [rows, top_k]
 *   int32 (where pair (t, j) sits in the expert-sorted order). */
RIA_API int ria_moe_prompt_norm(const float* x, int64_t x_stride, const void* post_norm_weight, float* h, void* h_bf16,
                                int32_t rows, ria_stream_t stream);
RIA_API int ria_silu_mul_bf16(const void* gate, const void* up, void* out, int64_t n, ria_stream_t stream);
RIA_API int ria_moe_prompt_combine(const float* x, int64_t x_stride, const void* expert_out,
                                   const int32_t* sorted_position, const float* weights, const void* shared_out,
                                   const float* shared_gate, float* out, int64_t out_stride, int32_t rows,
                                   int32_t top_k, ria_stream_t stream);

/* ------------------------------------------------------------------------
 * Greedy head of a decode step: the end of run_forward_token
 * (qwen36_chat_batch.py:194-199) and sample_next with temperature <= 0
 * (qwen36_mini_chat.py:75-78):
 *   h = fp16(rmsnorm(x) * (1 + norm_weight))   (fp32 norm, eps 1e-6, then the
 *                                               fp16 autocast rounding)
 *   logits = fp16(h . lm_head^T)               (fp32 accumulation)
 *   next_id = argmax(logits)                   (first index among equal maxima)
 *
 * ria_lm_head_greedy: batch <= 8; x [batch, 2048] f32, norm_weight [2048]
 * f32, lm_head [vocab, 2048] fp16 (row stride w_stride), next_ids [batch]
 * int32; logits [batch, vocab] fp16 (row stride logits_stride) is written
 * when not NULL.  workspace: ria_lm_head_workspace_bytes(batch) bytes,
 * 16-byte aligned, zero-filled before its first use (it holds a hand-off
 * counter that every call returns to zero; one workspace serves one stream
 * at a time).
 * Larger batches: ria_final_norm_f16 (out [rows, n] fp16), a library GEMM
 * for the fp16 logits, then ria_argmax_f16_rows (one index per row). */
RIA_API int64_t ria_lm_head_workspace_bytes(int32_t batch);
RIA_API int ria_lm_head_greedy(const float* x, int64_t x_stride, const float* norm_weight, const void* lm_head,
                               int64_t w_stride, int32_t vocab, void* logits, int64_t logits_stride,
                               int32_t* next_ids, void* workspace, int64_t workspace_bytes, int32_t batch,
                               ria_stream_t stream);
RIA_API int ria_final_norm_f16(const float* x, int64_t x_stride, const float* weight, void* out, int64_t out_stride,
                               int32_t rows, int32_t n, ria_stream_t stream);
RIA_API int ria_argmax_f16_rows(const void* logits, int64_t stride, int32_t vocab, int32_t rows, int32_t* out,
                                ria_stream_t stream);

/* One-token causal depthwise conv (kernel 4) + SiLU for B rows of `channels`
 * channels, in bf16 like the reference's conv weight dtype:
 * _causal_conv1d_step (qwen36_attention_cache.py:176-221).
 * x [B, channels] bf16, conv_state [B, channels, 4] bf16 updated in place,
 * weight [channels, 4] bf16, out [B, channels] bf16. */
RIA_API int ria_conv1d_step(const void* x, int64_t x_stride, void* conv_state, const void* weight, void* out,
                    int64_t out_stride, int32_t rows, int32_t channels, ria_stream_t stream);

/* lens[i] += 1 and positions[i] += 1 for i < batch: advances a batch of
 * sequences by one decoded token after all layers ran (the caller-side
 * `tokens_seen += 1`, qwen36_chat_batch.py:204-206), on the device so that a
 * captured decode step needs no host data. */
RIA_API int ria_advance_positions(int32_t* seq_lens, int32_t* positions, int32_t batch, ria_stream_t stream);

/* Partial NeoX RoPE in place on rows of f32 vectors: x[rows, head_dim] with the
 * first rope_dim dims rotated (rotate-half inside that slice) at `position`.
 * _apply_rope (qwen36_attention_cache.py:154-162). */
RIA_API int ria_rope_apply(float* x, int32_t rows, int32_t head_dim, int32_t rope_dim, const float* inv_freq,
                   int64_t position, ria_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RIA_ATTENTION_H_ */
