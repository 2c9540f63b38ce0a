// Stand-alone append of B tokens' post-RoPE K and V rows into the paged GQA
// cache: the storage step of router-ia's _append_full_kv
// (qwen36_attention_cache.py:365-373, after the limit checks of :344-363,
// which stay on the host).  The decode and prefill kernels (K3, K4) fuse this
// write into their attention pass; this entry point serves callers that
// compute K/V themselves (the module's _append_full_kv on a paged layer,
// probes that append cached tokens, cache transfer).
//
// One CTA per sequence, 128 threads: each thread moves four consecutive
// elements of the token's 512-wide K and V rows (two KV heads of 256), with
// 8-byte stores into the heads' 512-byte pool rows.  A block id outside the
// pool or a length past the block table is recorded in the device error word
// and the sequence is skipped; nothing is written out of bounds.
#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

constexpr int kHkv = 2;
constexpr int kD = 256;
constexpr int kBlock = 64;

struct AppendParams {
  const void* k;
  int64_t k_stride;
  const void* v;
  int64_t v_stride;
  bool in_f32;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  int64_t pool_tokens;
  const int32_t* block_table;
  int32_t bt_stride;
  const int32_t* seq_lens;
  int32_t seq_len0;
  int num_blocks;
  unsigned int* err;
};

__device__ __forceinline__ float4 load4(const void* base, int64_t row_off, int i, bool f32) {
  if (f32) return *reinterpret_cast<const float4*>(static_cast<const float*>(base) + row_off + i);
  const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(base) + row_off + i);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

__global__ void __launch_bounds__(128) kv_append_kernel(const AppendParams p) {
  pdl_wait();
  const int b = blockIdx.x;
  const int L = p.seq_lens ? p.seq_lens[b] : p.seq_len0;
  const int lp = L / kBlock;
  const int phys = (L >= 0 && lp < p.bt_stride) ? p.block_table[static_cast<int64_t>(b) * p.bt_stride + lp] : -1;
  if (phys < 0 || phys >= p.num_blocks) {
    if (threadIdx.x == 0) ria_set_error(p.err, RIA_DEVERR_BAD_BLOCK);
    return;
  }
  const int64_t row = static_cast<int64_t>(phys) * kBlock + L % kBlock;
  const int e = 4 * threadIdx.x;  // 128 threads x 4 elements = the token's 512-wide row (2 heads x 256)
  const int h = e / kD, d = e % kD;
  const float4 kv = load4(p.k, static_cast<int64_t>(b) * p.k_stride, e, p.in_f32);
  const float4 vv = load4(p.v, static_cast<int64_t>(b) * p.v_stride, e, p.in_f32);
  const int64_t dst = (static_cast<int64_t>(h) * p.pool_tokens + row) * kD + d;
  *reinterpret_cast<uint2*>(p.k_pool + dst) = make_uint2(pack_bf16x2(kv.x, kv.y), pack_bf16x2(kv.z, kv.w));
  *reinterpret_cast<uint2*>(p.v_pool + dst) = make_uint2(pack_bf16x2(vv.x, vv.y), pack_bf16x2(vv.z, vv.w));
}

}  // namespace

extern "C" int ria_kv_append_paged(const void* k_new, int64_t k_stride, const void* v_new, int64_t v_stride,
                                   int32_t inputs_f32, void* k_pool, void* v_pool, int64_t pool_tokens,
                                   const int32_t* block_table, int32_t block_table_stride, const int32_t* seq_lens,
                                   int32_t seq_len0, int32_t batch, ria_stream_t stream) {
  if (batch < 0) return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: batch=%d < 0", batch);
  if (batch == 0) return RIA_OK;
  if (!k_new || !v_new || !k_pool || !v_pool || !block_table)
    return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: null pointer argument");
  if (!seq_lens && batch != 1)
    return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: seq_lens may be null only for batch 1");
  if (!seq_lens && (seq_len0 < 0 || seq_len0 / kBlock >= block_table_stride))
    return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: seq_len0=%d outside the block table (stride %d)",
                     seq_len0, block_table_stride);
  if (block_table_stride < 1)
    return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: block_table_stride must be >= 1");
  if (pool_tokens <= 0 || pool_tokens % kBlock)
    return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: pool_tokens=%lld must be a positive multiple of 64",
                     static_cast<long long>(pool_tokens));
  const int esz = inputs_f32 ? 4 : 2;
  if (k_stride < kHkv * kD || v_stride < kHkv * kD)
    return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: row stride smaller than 512 elements");
  if (!ria::aligned(k_new, 4 * esz) || !ria::aligned(v_new, 4 * esz) || (k_stride * esz) % 16 ||
      (v_stride * esz) % 16 || !ria::aligned(k_pool, 16) || !ria::aligned(v_pool, 16))
    return ria::fail(RIA_ERR_INVALID, "ria_kv_append_paged: rows and pools must be 16-byte aligned");
  AppendParams p;
  p.k = k_new;
  p.k_stride = k_stride;
  p.v = v_new;
  p.v_stride = v_stride;
  p.in_f32 = inputs_f32 != 0;
  p.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  p.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  p.pool_tokens = pool_tokens;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.seq_lens = seq_lens;
  p.seq_len0 = seq_len0;
  p.num_blocks = static_cast<int>(pool_tokens / kBlock);
  p.err = ria::device_error_word();
  const cudaError_t e =
      ria::launch_pdl(kv_append_kernel, dim3(batch), dim3(128), 0, static_cast<cudaStream_t>(stream), p);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_kv_append_paged: %s", cudaGetErrorString(e));
  return ria::check_launch("ria_kv_append_paged");
}
