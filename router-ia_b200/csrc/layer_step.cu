// Whole decode layer steps for small batches (batch <= 8) as one C call each:
// the launches of a DeltaNet or GQA layer (input RMSNorm fused into the
// in-projection GEMV, the attention kernel, the out-projection GEMV with the
// residual add) issued back to back from C, with the intermediates in a
// caller-provided scratch buffer.
//
// This is for callers that step one layer per call from an interpreter --
// router-ia's run_forward_token calls attention_cache.step_attention once per
// layer (qwen36_chat_batch.py:181-207).  Issued as three or four separate
// foreign calls, each with its argument checks and conversions, the host work
// of a batch-1 layer (about 50 us) exceeds its GPU time; one call per layer
// removes most of it.  The kernels, their order and their arithmetic are
// those of the separate entry points, so results are identical.
#include <cuda_bf16.h>

#include "ria_capi_internal.h"

namespace {

constexpr int kHidden = 2048;
constexpr int kDnProj = 12352;  // [qkv 8192 | z 4096 | b 32 | a 32]
constexpr int kDnValue = 4096;
constexpr int kGqaProj = 9216;  // [q_gate 8192 | k 512 | v 512]
constexpr int kGqaOut = 4096;
constexpr int kGemvMaxBatch = 8;

int64_t round256(int64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

extern "C" int64_t ria_deltanet_layer_decode_scratch_bytes(int32_t batch) {
  if (batch <= 0 || batch > kGemvMaxBatch) return 0;
  return round256(static_cast<int64_t>(batch) * kDnProj * 2) + round256(static_cast<int64_t>(batch) * kDnValue * 2);
}

extern "C" int ria_deltanet_layer_decode(const float* x, int64_t x_stride, const float* in_norm, const void* w_in,
                                         int64_t w_in_stride, const void* conv_weight, const float* a_log,
                                         const float* dt_bias, const float* norm_weight, const void* w_out,
                                         int64_t w_out_stride, void* conv_state, float* rec_state,
                                         const int32_t* slots, int32_t num_slots, float* out, int64_t out_stride,
                                         void* scratch, int64_t scratch_bytes, int32_t batch, ria_stream_t stream) {
  if (batch < 0 || batch > kGemvMaxBatch)
    return ria::fail(RIA_ERR_INVALID, "ria_deltanet_layer_decode: batch %d outside [0, %d]", batch, kGemvMaxBatch);
  if (batch == 0) return RIA_OK;
  if (!scratch || !ria::aligned(scratch, 256) || scratch_bytes < ria_deltanet_layer_decode_scratch_bytes(batch))
    return ria::fail(RIA_ERR_INVALID, "ria_deltanet_layer_decode: scratch needs %lld bytes, 256-byte aligned",
                     static_cast<long long>(ria_deltanet_layer_decode_scratch_bytes(batch)));
  unsigned char* s = static_cast<unsigned char*>(scratch);
  __nv_bfloat16* proj = reinterpret_cast<__nv_bfloat16*>(s);
  __nv_bfloat16* gated = reinterpret_cast<__nv_bfloat16*>(s + round256(static_cast<int64_t>(batch) * kDnProj * 2));
  int rc = ria_rmsnorm_gemv(x, x_stride, in_norm, w_in, w_in_stride, proj, kDnProj, batch, kDnProj, kHidden, stream);
  if (rc) return rc;
  rc = ria_gdn_decode_step(proj, kDnProj, proj + 8192, kDnProj, proj + 12288, kDnProj, proj + 12320, kDnProj,
                           conv_weight, a_log, dt_bias, norm_weight, conv_state, rec_state, slots, num_slots, gated,
                           kDnValue, batch, stream);
  if (rc) return rc;
  return ria_gemv_residual(gated, kDnValue, w_out, w_out_stride, x, x_stride, out, out_stride, batch, kHidden,
                           kDnValue, stream);
}

extern "C" int64_t ria_gqa_layer_decode_scratch_bytes(int32_t batch, int32_t max_splits) {
  if (batch <= 0 || batch > kGemvMaxBatch || max_splits <= 0) return 0;
  return round256(static_cast<int64_t>(batch) * kGqaProj * 2) + round256(static_cast<int64_t>(batch) * kGqaOut * 2) +
         round256(max_splits > 1 ? ria_gqa_decode_workspace_bytes(batch, max_splits) : 0);
}

extern "C" int ria_gqa_layer_decode(const float* x, int64_t x_stride, const float* in_norm, const void* w_in,
                                    int64_t w_in_stride, const float* q_norm_weight, const float* k_norm_weight,
                                    const float* inv_freq, void* k_pool, void* v_pool, int64_t pool_tokens,
                                    const int32_t* block_table, int32_t block_table_stride, const int32_t* seq_lens,
                                    const int32_t* positions, int32_t seq_len0, int32_t position0, const void* w_out,
                                    int64_t w_out_stride, float* out, int64_t out_stride, void* scratch,
                                    int64_t scratch_bytes, int32_t batch, int32_t split_pages, int32_t max_splits,
                                    ria_stream_t stream) {
  if (batch < 0 || batch > kGemvMaxBatch)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_layer_decode: batch %d outside [0, %d]", batch, kGemvMaxBatch);
  if (batch == 0) return RIA_OK;
  if (max_splits < 1) return ria::fail(RIA_ERR_INVALID, "ria_gqa_layer_decode: max_splits=%d", max_splits);
  if (!scratch || !ria::aligned(scratch, 256) ||
      scratch_bytes < ria_gqa_layer_decode_scratch_bytes(batch, max_splits))
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_layer_decode: scratch needs %lld bytes, 256-byte aligned",
                     static_cast<long long>(ria_gqa_layer_decode_scratch_bytes(batch, max_splits)));
  unsigned char* s = static_cast<unsigned char*>(scratch);
  const int64_t attn_off = round256(static_cast<int64_t>(batch) * kGqaProj * 2);
  const int64_t ws_off = attn_off + round256(static_cast<int64_t>(batch) * kGqaOut * 2);
  __nv_bfloat16* proj = reinterpret_cast<__nv_bfloat16*>(s);
  __nv_bfloat16* attn = reinterpret_cast<__nv_bfloat16*>(s + attn_off);
  void* ws = max_splits > 1 ? static_cast<void*>(s + ws_off) : nullptr;
  const int64_t ws_bytes = max_splits > 1 ? ria_gqa_decode_workspace_bytes(batch, max_splits) : 0;
  int rc = ria_rmsnorm_gemv(x, x_stride, in_norm, w_in, w_in_stride, proj, kGqaProj, batch, kGqaProj, kHidden, stream);
  if (rc) return rc;
  rc = ria_gqa_decode_paged(proj, kGqaProj, proj + 8192, kGqaProj, proj + 8704, kGqaProj, q_norm_weight,
                            k_norm_weight, inv_freq, k_pool, v_pool, pool_tokens, block_table, block_table_stride,
                            seq_lens, positions, seq_len0, position0, attn, kGqaOut, ws, ws_bytes, batch, split_pages,
                            max_splits, stream);
  if (rc) return rc;
  return ria_gemv_residual(attn, kGqaOut, w_out, w_out_stride, x, x_stride, out, out_stride, batch, kHidden, kGqaOut,
                           stream);
}
