// Element kernels of the prompt-prefill MoE path (engine.moe_prefill).
//
// With thousands of tokens per expert the MoE block of a prompt is a grouped
// GEMM, and those GEMMs run on a library kernel; these three kernels replace
// the framework's element-by-element glue around them, each one pass over
// its data:
//   * ria_moe_prompt_norm: the post-attention RMSNorm (x rsqrt(mean(x^2) +
//     1e-6) (1 + w), qwen36_op_probe.py:55-67) into fp32 (for the fp32 router
//     GEMM) and bf16 (the experts' input);
//   * ria_silu_mul_bf16: h = silu(gate) * up of the SwiGLU experts
//     (qwen36_chat_batch.py:127-178), fp32 arithmetic on bf16 operands;
//   * ria_moe_prompt_combine: out = x + (sum over the k slots, in slot order,
//     of weight * expert output + sigmoid-gated shared expert output), reading
//     each expert output row from its position in the expert-sorted order.
#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

constexpr int kH = 2048;

__global__ void __launch_bounds__(256) moe_prompt_norm_kernel(const float* __restrict__ x, int64_t xs,
                                                              const __nv_bfloat16* __restrict__ w, float* __restrict__ h,
                                                              __nv_bfloat16* __restrict__ hb) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const float* xr = x + row * xs;
  float4 v[kH / 1024];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kH / 1024; ++i) {
    v[i] = *reinterpret_cast<const float4*>(xr + i * 1024 + threadIdx.x * 4);
    ss = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, ss))));
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(kH) + 1e-6f);
#pragma unroll
  for (int i = 0; i < kH / 1024; ++i) {
    const int d = i * 1024 + threadIdx.x * 4;
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + d));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + d + 2));
    const float4 m = make_float4(v[i].x * r * (1.f + a.x), v[i].y * r * (1.f + a.y), v[i].z * r * (1.f + b.x),
                                 v[i].w * r * (1.f + b.y));
    *reinterpret_cast<float4*>(h + row * kH + d) = m;
    uint2 pk;
    pk.x = pack_bf16x2(m.x, m.y);
    pk.y = pack_bf16x2(m.z, m.w);
    *reinterpret_cast<uint2*>(hb + row * kH + d) = pk;
  }
}

// 8 elements per thread.
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ u,
                                __nv_bfloat16* __restrict__ out, int64_t n8) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint4 gv = reinterpret_cast<const uint4*>(g)[i];
  const uint4 uv = reinterpret_cast<const uint4*>(u)[i];
  const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
  const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
  uint4 o;
  uint32_t* o2 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 a = __bfloat1622float2(g2[e]);
    const float2 b = __bfloat1622float2(u2[e]);
    o2[e] = pack_bf16x2(a.x / (1.0f + expf(-a.x)) * b.x, a.y / (1.0f + expf(-a.y)) * b.y);
  }
  reinterpret_cast<uint4*>(out)[i] = o;
}

// Token blockIdx.x, 4 columns per thread (blockIdx.y picks a 1024-column half).
__global__ void __launch_bounds__(256) moe_prompt_combine_kernel(const float* __restrict__ x, int64_t xs,
                                                                 const __nv_bfloat16* __restrict__ y,
                                                                 const int32_t* __restrict__ inv,
                                                                 const float* __restrict__ wts,
                                                                 const __nv_bfloat16* __restrict__ shared,
                                                                 const float* __restrict__ sg, float* __restrict__ out,
                                                                 int64_t os, int top_k) {
  const int64_t t = blockIdx.x;
  const int d = blockIdx.y * 1024 + threadIdx.x * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < top_k; ++j) {
    const int64_t p = inv[t * top_k + j];
    const float wj = wts[t * top_k + j];
    const uint2 raw = *reinterpret_cast<const uint2*>(y + p * kH + d);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    acc.x += wj * a.x;
    acc.y += wj * a.y;
    acc.z += wj * b.x;
    acc.w += wj * b.y;
  }
  const uint2 sraw = *reinterpret_cast<const uint2*>(shared + t * kH + d);
  const float2 sa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sraw.x));
  const float2 sb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sraw.y));
  const float gt = sg[t];
  const float4 xv = *reinterpret_cast<const float4*>(x + t * xs + d);
  *reinterpret_cast<float4*>(out + t * os + d) =
      make_float4(xv.x + (acc.x + sa.x * gt), xv.y + (acc.y + sa.y * gt), xv.z + (acc.z + sb.x * gt),
                  xv.w + (acc.w + sb.y * gt));
}

}  // namespace

extern "C" int ria_moe_prompt_norm(const float* x, int64_t x_stride, const void* post_norm_weight, float* h,
                                   void* h_bf16, int32_t rows, ria_stream_t stream) {
  if (rows < 0) return ria::fail(RIA_ERR_INVALID, "ria_moe_prompt_norm: rows %d < 0", rows);
  if (rows == 0) return RIA_OK;
  if (!x || !post_norm_weight || !h || !h_bf16) return ria::fail(RIA_ERR_INVALID, "ria_moe_prompt_norm: null pointer");
  if (!ria::aligned(x, 16) || !ria::aligned(h, 16) || !ria::aligned(h_bf16, 16) || !ria::aligned(post_norm_weight, 4) ||
      x_stride % 4 || x_stride < kH)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_prompt_norm: misaligned rows");
  moe_prompt_norm_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_stride, static_cast<const __nv_bfloat16*>(post_norm_weight), h, static_cast<__nv_bfloat16*>(h_bf16));
  return ria::check_launch("ria_moe_prompt_norm");
}

extern "C" int ria_silu_mul_bf16(const void* gate, const void* up, void* out, int64_t n, ria_stream_t stream) {
  if (n < 0 || n % 8) return ria::fail(RIA_ERR_INVALID, "ria_silu_mul_bf16: n %lld not a multiple of 8", (long long)n);
  if (n == 0) return RIA_OK;
  if (!gate || !up || !out) return ria::fail(RIA_ERR_INVALID, "ria_silu_mul_bf16: null pointer");
  if (!ria::aligned(gate, 16) || !ria::aligned(up, 16) || !ria::aligned(out, 16))
    return ria::fail(RIA_ERR_INVALID, "ria_silu_mul_bf16: buffers must be 16-byte aligned");
  const int64_t n8 = n / 8;
  silu_mul_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up), static_cast<__nv_bfloat16*>(out),
      n8);
  return ria::check_launch("ria_silu_mul_bf16");
}

extern "C" int ria_moe_prompt_combine(const float* x, int64_t x_stride, const void* expert_out,
                                      const int32_t* sorted_position, const float* weights, const void* shared_out,
                                      const float* shared_gate, float* out, int64_t out_stride, int32_t rows,
                                      int32_t top_k, ria_stream_t stream) {
  if (rows < 0 || top_k < 1) return ria::fail(RIA_ERR_INVALID, "ria_moe_prompt_combine: rows %d, top_k %d", rows, top_k);
  if (rows == 0) return RIA_OK;
  if (!x || !expert_out || !sorted_position || !weights || !shared_out || !shared_gate || !out)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_prompt_combine: null pointer");
  if (!ria::aligned(x, 16) || !ria::aligned(out, 16) || !ria::aligned(expert_out, 8) || !ria::aligned(shared_out, 8) ||
      x_stride % 4 || out_stride % 4 || x_stride < kH || out_stride < kH)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_prompt_combine: misaligned rows");
  moe_prompt_combine_kernel<<<dim3(rows, kH / 1024), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_stride, static_cast<const __nv_bfloat16*>(expert_out), sorted_position, weights,
      static_cast<const __nv_bfloat16*>(shared_out), shared_gate, out, out_stride, top_k);
  return ria::check_launch("ria_moe_prompt_combine");
}
