// Row kernels around the projections: input RMSNorm, residual add, and the
// stand-alone conv / RoPE steps behind the module's private helpers.
#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

// One CTA per row; fp32 in, bf16 out; x * rsqrt(mean(x^2) + 1e-6) * (1 + w)
// (router-ia qwen36_op_probe.py:55-67).
template <bool F16>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x, int64_t xs,
                                                           const float* __restrict__ w, uint16_t* __restrict__ out,
                                                           int64_t os, int n) {
  __shared__ float red[8];
  pdl_wait();
  const int row = blockIdx.x;
  const float* xr = x + row * xs;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(n) + 1e-6f);
  uint16_t* o = out + row * os;
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 ww = *reinterpret_cast<const float4*>(w + i);
    uint2 pk;
    if (F16) {
      pk.x = pack_f16x2(v.x * r * (1.f + ww.x), v.y * r * (1.f + ww.y));
      pk.y = pack_f16x2(v.z * r * (1.f + ww.z), v.w * r * (1.f + ww.w));
    } else {
      pk.x = pack_bf16x2(v.x * r * (1.f + ww.x), v.y * r * (1.f + ww.y));
      pk.y = pack_bf16x2(v.z * r * (1.f + ww.z), v.w * r * (1.f + ww.w));
    }
    *reinterpret_cast<uint2*>(o + i) = pk;
  }
}

__global__ void residual_add_kernel(const float* __restrict__ x0, int64_t xs, const __nv_bfloat16* __restrict__ proj,
                                    int64_t ps, float* __restrict__ out, int64_t os, int n) {
  pdl_wait();
  const int64_t row = blockIdx.x;  // rows on x: up to 2^31 - 1 of them
  const int i = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (i >= n) return;
  const float4 a = *reinterpret_cast<const float4*>(x0 + row * xs + i);
  const uint2 raw = *reinterpret_cast<const uint2*>(proj + row * ps + i);
  const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
  const float2 p01 = __bfloat1622float2(p2[0]);
  const float2 p23 = __bfloat1622float2(p2[1]);
  *reinterpret_cast<float4*>(out + row * os + i) = make_float4(a.x + p01.x, a.y + p01.y, a.z + p23.x, a.w + p23.y);
}

// Causal depthwise conv (kernel 4) + SiLU in bf16, one token
// (router-ia qwen36_attention_cache.py:176-221).
__global__ void conv1d_step_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs, __nv_bfloat16* state,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int64_t os,
                                   int channels) {
  const int row = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= channels) return;
  __nv_bfloat16* st = state + (static_cast<int64_t>(row) * channels + c) * 4;
  const __nv_bfloat16 xv = x[row * xs + c];
  const float s1 = __bfloat162float(st[1]), s2 = __bfloat162float(st[2]), s3 = __bfloat162float(st[3]);
  const __nv_bfloat16* wc = w + static_cast<int64_t>(c) * 4;
  float acc = __bfloat162float(wc[0]) * s1;
  acc = fmaf(__bfloat162float(wc[1]), s2, acc);
  acc = fmaf(__bfloat162float(wc[2]), s3, acc);
  acc = fmaf(__bfloat162float(wc[3]), __bfloat162float(xv), acc);
  st[0] = st[1];
  st[1] = st[2];
  st[2] = st[3];
  st[3] = xv;
  const float y = bf16_round(acc);
  out[row * os + c] = __float2bfloat16_rn(y / (1.0f + expf(-y)));
}

// Partial rotate-half RoPE on rows of f32 (router-ia qwen36_attention_cache.py:137-162).
__global__ void rope_apply_kernel(float* x, int head_dim, int rope_dim, const float* __restrict__ inv_freq,
                                  float position) {
  const int row = blockIdx.x;
  const int half = rope_dim / 2;
  const int i = threadIdx.x;
  if (i >= half) return;
  float* xr = x + static_cast<int64_t>(row) * head_dim;
  float sn, cs;
  sincosf(position * inv_freq[i], &sn, &cs);
  const float a = xr[i], b = xr[i + half];
  xr[i] = a * cs - b * sn;
  xr[i + half] = b * cs + a * sn;
}

__global__ void advance_kernel(int32_t* lens, int32_t* pos, int n) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    lens[i] += 1;
    pos[i] += 1;
  }
}

}  // namespace

extern "C" int ria_advance_positions(int32_t* seq_lens, int32_t* positions, int32_t batch, ria_stream_t stream) {
  if (batch < 0) return ria::fail(RIA_ERR_INVALID, "ria_advance_positions: batch < 0");
  if (batch == 0) return RIA_OK;
  if (!seq_lens || !positions) return ria::fail(RIA_ERR_INVALID, "ria_advance_positions: null pointer");
  const cudaError_t e = ria::launch_pdl(advance_kernel, dim3((batch + 255) / 256), dim3(256), 0,
                                       static_cast<cudaStream_t>(stream), seq_lens, positions, batch);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_advance_positions: %s", cudaGetErrorString(e));
  return ria::check_launch("ria_advance_positions");
}

namespace {

template <bool F16>
int rmsnorm_rows_impl(const char* what, const float* x, int64_t x_stride, const float* weight, void* out,
                      int64_t out_stride, int32_t rows, int32_t n, ria_stream_t stream) {
  if (rows < 0 || n <= 0 || n % 4 != 0) return ria::fail(RIA_ERR_INVALID, "%s: bad rows/n", what);
  if (rows == 0) return RIA_OK;
  if (!x || !weight || !out) return ria::fail(RIA_ERR_INVALID, "%s: null pointer", what);
  if (!ria::aligned(x, 16) || !ria::aligned(weight, 16) || !ria::aligned(out, 8) || x_stride % 4 || out_stride % 4)
    return ria::fail(RIA_ERR_INVALID, "%s: misaligned rows", what);
  const cudaError_t e = ria::launch_pdl(rmsnorm_rows_kernel<F16>, dim3(rows), dim3(256), 0,
                                       static_cast<cudaStream_t>(stream), x, x_stride, weight,
                                       static_cast<uint16_t*>(out), out_stride, n);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ria::check_launch(what);
}

}  // namespace

extern "C" int ria_rmsnorm_rows(const float* x, int64_t x_stride, const float* weight, void* out, int64_t out_stride,
                                int32_t rows, int32_t n, ria_stream_t stream) {
  return rmsnorm_rows_impl<false>("ria_rmsnorm_rows", x, x_stride, weight, out, out_stride, rows, n, stream);
}

extern "C" int ria_rmsnorm_rows_f16(const float* x, int64_t x_stride, const float* weight, void* out,
                                    int64_t out_stride, int32_t rows, int32_t n, ria_stream_t stream) {
  return rmsnorm_rows_impl<true>("ria_rmsnorm_rows_f16", x, x_stride, weight, out, out_stride, rows, n, stream);
}

extern "C" int ria_residual_add(const float* x0, int64_t x0_stride, const void* proj, int64_t proj_stride, float* out,
                                int64_t out_stride, int32_t rows, int32_t n, ria_stream_t stream) {
  if (rows < 0 || n <= 0 || n % 4 != 0) return ria::fail(RIA_ERR_INVALID, "ria_residual_add: bad rows/n");
  if (rows == 0) return RIA_OK;
  if (!x0 || !proj || !out) return ria::fail(RIA_ERR_INVALID, "ria_residual_add: null pointer");
  if (!ria::aligned(x0, 16) || !ria::aligned(out, 16) || !ria::aligned(proj, 8) || x0_stride % 4 || out_stride % 4 ||
      proj_stride % 4)
    return ria::fail(RIA_ERR_INVALID, "ria_residual_add: misaligned rows");
  dim3 grid(rows, (n / 4 + 255) / 256);
  const cudaError_t e =
      ria::launch_pdl(residual_add_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream), x0, x0_stride,
                      static_cast<const __nv_bfloat16*>(proj), proj_stride, out, out_stride, n);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_residual_add: %s", cudaGetErrorString(e));
  return ria::check_launch("ria_residual_add");
}

extern "C" int ria_conv1d_step(const void* x, int64_t x_stride, void* conv_state, const void* weight, void* out,
                               int64_t out_stride, int32_t rows, int32_t channels, ria_stream_t stream) {
  if (rows < 0 || channels <= 0) return ria::fail(RIA_ERR_INVALID, "ria_conv1d_step: bad rows/channels");
  if (rows == 0) return RIA_OK;
  if (!x || !conv_state || !weight || !out) return ria::fail(RIA_ERR_INVALID, "ria_conv1d_step: null pointer");
  dim3 grid((channels + 255) / 256, rows);
  conv1d_step_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), x_stride, static_cast<__nv_bfloat16*>(conv_state),
      static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out), out_stride, channels);
  return ria::check_launch("ria_conv1d_step");
}

extern "C" int ria_rope_apply(float* x, int32_t rows, int32_t head_dim, int32_t rope_dim, const float* inv_freq,
                              int64_t position, ria_stream_t stream) {
  if (rows < 0 || head_dim <= 0 || rope_dim <= 0 || rope_dim % 2 || rope_dim > head_dim || rope_dim > 2048)
    return ria::fail(RIA_ERR_INVALID, "ria_rope_apply: bad shape (rows=%d head_dim=%d rope_dim=%d)", rows, head_dim,
                     rope_dim);
  if (rows == 0) return RIA_OK;
  if (!x || !inv_freq) return ria::fail(RIA_ERR_INVALID, "ria_rope_apply: null pointer");
  rope_apply_kernel<<<rows, rope_dim / 2, 0, static_cast<cudaStream_t>(stream)>>>(x, head_dim, rope_dim, inv_freq,
                                                                                   static_cast<float>(position));
  return ria::check_launch("ria_rope_apply");
}
