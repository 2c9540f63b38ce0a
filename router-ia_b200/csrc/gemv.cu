// Small-batch projections (B <= 8) as weight-streaming GEMVs, with the layer
// input RMSNorm fused into the in-projection and the residual add fused into
// the out-projection (router-ia qwen36_attention_cache.py:228-240 and
// :272-277 for DeltaNet, :289-297 and :318-321 for GQA).  At batch 1 the
// projections read 67 MB of bf16 weights per DeltaNet layer, so the step is
// bound by that stream; a library GEMM at M = 1 runs well below it, and the
// separate norm / add launches cost as much as a GEMV.
//
// One warp per output row at a time: every lane streams 16-byte chunks of the
// weight row (coalesced, read once), multiplies them with the B input rows
// staged in shared memory, and the warp reduces.  The in-projection CTA first
// recomputes the RMSNorm of its B input rows with the same reduction order as
// ria_rmsnorm_rows_f16, so both paths produce the same fp16 activations.
//
// Types: the in-projection runs on fp16 weights and fp16 normalised inputs
// (fp32 accumulation, bf16 output), the out-projection on bf16 weights and
// the bf16 attention output.  fp16 for the in-projection input keeps the
// layer within the attention path's per-token bars against the fp32 CPU
// path: rounding the normalised input to bf16 (2^-9) moved single tokens'
// attention contribution by up to ~1.9e-2 relative RMS, fp16 (2^-12) by
// ~6e-3.  router-ia's own CUDA path runs these projections on fp16 weights.
#include <algorithm>

#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

__device__ __forceinline__ float2 to_float2(__nv_bfloat162 v) { return __bfloat1622float2(v); }
__device__ __forceinline__ float2 to_float2(__half2 v) { return __half22float2(v); }

template <class T>
struct Vec2;
template <>
struct Vec2<__nv_bfloat16> {
  using type = __nv_bfloat162;
};
template <>
struct Vec2<__half> {
  using type = __half2;
};

constexpr int kMaxBatch = 8;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// One warp per output row at a time, rows strided over all warps of the grid.
// A lane holds KC 16-byte chunks of a row (the whole row is in flight at
// once) in a ring of D rows: rows r + warps .. r + (D-1) warps are loading
// while row r is reduced.  pro() runs once the first rows' loads are issued
// (it stages the inputs, so the two overlap); f(row, acc[B]) consumes each
// finished row (lane 0's values are the sums).
template <class T, int B, int KC, int D, class P, class F>
__device__ __forceinline__ void gemv_rows(const T* __restrict__ w, int64_t ws, const T* xs, int n, P&& pro, F&& f) {
  using T2 = typename Vec2<T>::type;
  constexpr int k = KC * 256;
  pdl_wait();  // nothing is read before the preceding kernel is complete, weights included
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * kWarps;
  const int row0 = blockIdx.x * kWarps + (threadIdx.x >> 5);
  uint4 ring[D][KC];
  auto load = [&](int slot, int row) {
    if (row < n) {
#pragma unroll
      for (int c = 0; c < KC; ++c)
        ring[slot][c] =
            __ldg(reinterpret_cast<const uint4*>(w + static_cast<int64_t>(row) * ws + c * 256 + lane * 8));
    }
  };
#pragma unroll
  for (int d = 0; d < D; ++d) load(d, row0 + d * warps);
  pro();
  for (int row = row0; row < n; row += warps) {
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
#pragma unroll
    for (int c = 0; c < KC; ++c) {
      const T2* w2 = reinterpret_cast<const T2*>(&ring[0][c]);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4 u = *reinterpret_cast<const uint4*>(xs + b * k + c * 256 + lane * 8);
        const T2* x2 = reinterpret_cast<const T2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 wf = to_float2(w2[e]);
          const float2 xf = to_float2(x2[e]);
          acc[b] = fmaf(wf.x, xf.x, acc[b]);
          acc[b] = fmaf(wf.y, xf.y, acc[b]);
        }
      }
    }
#pragma unroll
    for (int d = 0; d + 1 < D; ++d)
#pragma unroll
      for (int c = 0; c < KC; ++c) ring[d][c] = ring[d + 1][c];
    if (D > 1) load(D - 1, row + D * warps);
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = warp_sum(acc[b]);
    f(row, acc);
    if (D == 1) load(0, row + warps);
  }
}

// out[b, :] = bf16(W . fp16(rmsnorm(x[b]) * (1 + norm_w))), W fp16
template <int B, int KC, int D>
__global__ void __launch_bounds__(kThreads) rmsnorm_gemv_kernel(const float* __restrict__ x, int64_t xs,
                                                                const float* __restrict__ norm_w,
                                                                const __half* __restrict__ w, int64_t ws,
                                                                __nv_bfloat16* __restrict__ out, int64_t os, int n) {
  constexpr int k = KC * 256;
  extern __shared__ __align__(16) unsigned char smem[];
  __half* h = reinterpret_cast<__half*>(smem);  // [B][k]
  __shared__ float red[kWarps];
  auto norm = [&]() {
    for (int b = 0; b < B; ++b) {  // the reduction order of rmsnorm_rows_kernel
      const float* xr = x + b * xs;
      float ss = 0.f;
      for (int i = threadIdx.x * 4; i < k; i += kThreads * 4) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int i = 0; i < kWarps; ++i) tot += red[i];
      const float r = rsqrtf(tot / static_cast<float>(k) + 1e-6f);
      for (int i = threadIdx.x * 4; i < k; i += kThreads * 4) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        const float4 ww = *reinterpret_cast<const float4*>(norm_w + i);
        uint2 pk;
        pk.x = pack_f16x2(v.x * r * (1.f + ww.x), v.y * r * (1.f + ww.y));
        pk.y = pack_f16x2(v.z * r * (1.f + ww.z), v.w * r * (1.f + ww.w));
        *reinterpret_cast<uint2*>(h + b * k + i) = pk;
      }
      __syncthreads();  // red is reused by the next row; h is complete
    }
  };
  gemv_rows<__half, B, KC, D>(w, ws, h, n, norm, [&](int row, const float (&acc)[B]) {
    if ((threadIdx.x & 31) == 0)
#pragma unroll
      for (int b = 0; b < B; ++b) out[b * os + row] = __float2bfloat16_rn(acc[b]);
  });
}

// out[b, :] = x0[b, :] + bf16(W . a[b])  (the projection rounded to bf16 as
// the library GEMM's output would be, then added in fp32)
template <int B, int KC, int D>
__global__ void __launch_bounds__(kThreads) gemv_residual_kernel(const __nv_bfloat16* __restrict__ a, int64_t as,
                                                                 const __nv_bfloat16* __restrict__ w, int64_t ws,
                                                                 const float* __restrict__ x0, int64_t x0s,
                                                                 float* __restrict__ out, int64_t os, int n) {
  constexpr int k = KC * 256;
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);  // [B][k]
  auto stage = [&]() {
    for (int b = 0; b < B; ++b)
      for (int i = threadIdx.x * 8; i < k; i += kThreads * 8)
        *reinterpret_cast<uint4*>(xs + b * k + i) = *reinterpret_cast<const uint4*>(a + b * as + i);
    __syncthreads();
  };
  gemv_rows<__nv_bfloat16, B, KC, D>(w, ws, xs, n, stage, [&](int row, const float (&acc)[B]) {
    if ((threadIdx.x & 31) == 0)
#pragma unroll
      for (int b = 0; b < B; ++b) out[b * os + row] = x0[b * x0s + row] + bf16_round(acc[b]);
  });
}

int check_common(const char* what, const void* w, int64_t w_stride, int32_t batch, int32_t n, int32_t k) {
  if (batch < 0 || batch > kMaxBatch || n <= 0)
    return ria::fail(RIA_ERR_INVALID, "%s: batch %d (max %d), n %d", what, batch, kMaxBatch, n);
  if (k != 2048 && k != 4096)
    return ria::fail(RIA_ERR_INVALID, "%s: k %d (the layer widths 2048 and 4096 are compiled)", what, k);
  if (w_stride < k || w_stride % 8 || !ria::aligned(w, 16))
    return ria::fail(RIA_ERR_INVALID, "%s: weight rows must be 16-byte aligned", what);
  return RIA_OK;
}

// Launch shape: rows that fit one per warp at two CTAs per SM need no
// prefetch ring (D = 1); otherwise one row ahead (D = 2), two CTAs per SM for
// 2048-wide rows and one for 4096-wide rows (register budget).  A ring two
// rows deep measured slower than one for the 2048-wide rows.
struct Shape {
  int grid, depth;
};
Shape shape_for(int n, int kc) {
  const int sms = ria::num_sms();
  const int ctas_for_rows = (n + kWarps - 1) / kWarps;
  if (ctas_for_rows <= 2 * sms) return {ctas_for_rows, 1};
  return kc <= 8 ? Shape{2 * sms, 2} : Shape{sms, 2};
}

template <int B, int KC, int D>
cudaError_t launch_rg(const float* x, int64_t xs, const float* nw, const __half* w, int64_t ws,
                      __nv_bfloat16* out, int64_t os, int n, int grid, cudaStream_t st) {
  const int smem = B * KC * 256 * 2;
  cudaError_t e =
      cudaFuncSetAttribute(rmsnorm_gemv_kernel<B, KC, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = ria::launch_pdl(rmsnorm_gemv_kernel<B, KC, D>, dim3(grid), dim3(kThreads), smem, st, x, xs, nw, w, ws, out, os,
                        n);
  return e;
}

template <int B, int KC, int D>
cudaError_t launch_gr(const __nv_bfloat16* a, int64_t as, const __nv_bfloat16* w, int64_t ws, const float* x0,
                      int64_t x0s, float* out, int64_t os, int n, int grid, cudaStream_t st) {
  const int smem = B * KC * 256 * 2;
  cudaError_t e =
      cudaFuncSetAttribute(gemv_residual_kernel<B, KC, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = ria::launch_pdl(gemv_residual_kernel<B, KC, D>, dim3(grid), dim3(kThreads), smem, st, a, as, w, ws, x0, x0s,
                        out, os, n);
  return e;
}

template <int KC, class L>
cudaError_t by_batch(int batch, L&& launch) {
  switch (batch) {
    case 1: return launch(std::integral_constant<int, 1>{});
    case 2: return launch(std::integral_constant<int, 2>{});
    case 3: return launch(std::integral_constant<int, 3>{});
    case 4: return launch(std::integral_constant<int, 4>{});
    case 5: return launch(std::integral_constant<int, 5>{});
    case 6: return launch(std::integral_constant<int, 6>{});
    case 7: return launch(std::integral_constant<int, 7>{});
    default: return launch(std::integral_constant<int, 8>{});
  }
}

}  // namespace

extern "C" int ria_rmsnorm_gemv(const float* x, int64_t x_stride, const float* norm_weight, const void* w,
                                int64_t w_stride, void* out, int64_t out_stride, int32_t batch, int32_t n, int32_t k,
                                ria_stream_t stream) {
  int rc = check_common("ria_rmsnorm_gemv", w, w_stride, batch, n, k);
  if (rc) return rc;
  if (batch == 0) return RIA_OK;
  if (!x || !norm_weight || !out) return ria::fail(RIA_ERR_INVALID, "ria_rmsnorm_gemv: null pointer");
  if (x_stride % 4 || !ria::aligned(x, 16) || !ria::aligned(norm_weight, 16))
    return ria::fail(RIA_ERR_INVALID, "ria_rmsnorm_gemv: x rows must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __half* wb = static_cast<const __half*>(w);
  __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(out);
  const int kc = k / 256;
  const Shape sh = shape_for(n, kc);
  auto go = [&](auto kcc, auto dd) {
    constexpr int KC = decltype(kcc)::value, D = decltype(dd)::value;
    return by_batch<KC>(batch, [&](auto bb) {
      return launch_rg<decltype(bb)::value, KC, D>(x, x_stride, norm_weight, wb, w_stride, ob, out_stride, n,
                                                   sh.grid, st);
    });
  };
  using I8 = std::integral_constant<int, 8>;
  using I16 = std::integral_constant<int, 16>;
  using D1 = std::integral_constant<int, 1>;
  using D2 = std::integral_constant<int, 2>;
  const cudaError_t e = kc == 8 ? (sh.depth == 1 ? go(I8{}, D1{}) : go(I8{}, D2{}))
                                : (sh.depth == 1 ? go(I16{}, D1{}) : go(I16{}, D2{}));
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_rmsnorm_gemv: %s", cudaGetErrorString(e));
  return ria::check_launch("ria_rmsnorm_gemv");
}

extern "C" int ria_gemv_residual(const void* a, int64_t a_stride, const void* w, int64_t w_stride, const float* x0,
                                 int64_t x0_stride, float* out, int64_t out_stride, int32_t batch, int32_t n, int32_t k,
                                 ria_stream_t stream) {
  int rc = check_common("ria_gemv_residual", w, w_stride, batch, n, k);
  if (rc) return rc;
  if (batch == 0) return RIA_OK;
  if (!a || !x0 || !out) return ria::fail(RIA_ERR_INVALID, "ria_gemv_residual: null pointer");
  if (a_stride % 8 || !ria::aligned(a, 16))
    return ria::fail(RIA_ERR_INVALID, "ria_gemv_residual: input rows must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* ab = static_cast<const __nv_bfloat16*>(a);
  const __nv_bfloat16* wb = static_cast<const __nv_bfloat16*>(w);
  const int kc = k / 256;
  const Shape sh = shape_for(n, kc);
  auto go = [&](auto kcc, auto dd) {
    constexpr int KC = decltype(kcc)::value, D = decltype(dd)::value;
    return by_batch<KC>(batch, [&](auto bb) {
      return launch_gr<decltype(bb)::value, KC, D>(ab, a_stride, wb, w_stride, x0, x0_stride, out, out_stride, n,
                                                   sh.grid, st);
    });
  };
  using I8 = std::integral_constant<int, 8>;
  using I16 = std::integral_constant<int, 16>;
  using D1 = std::integral_constant<int, 1>;
  using D2 = std::integral_constant<int, 2>;
  const cudaError_t e = kc == 8 ? (sh.depth == 1 ? go(I8{}, D1{}) : go(I8{}, D2{}))
                                : (sh.depth == 1 ? go(I16{}, D1{}) : go(I16{}, D2{}));
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_gemv_residual: %s", cudaGetErrorString(e));
  return ria::check_launch("ria_gemv_residual");
}
