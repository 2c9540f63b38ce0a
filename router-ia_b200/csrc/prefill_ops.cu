// Row kernels of a Gated DeltaNet layer's prompt (prefill) path around K2:
// the causal depthwise conv over T tokens with the rolling conv state, the
// decay / beta gates, and the gated RMSNorm of the chunked rule's output.
// Each restates, for T tokens at once, the per-token arithmetic of
// router-ia's _linear_stateful (qwen36_attention_cache.py:176-271).
#include <climits>

#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

constexpr int kConvTile = 256;  // tokens per CTA in the conv prefill

// out[b, t, c] = silu(sum_j w[c, j] * h[t - 3 + j]) with h[-3..-1] taken from
// the conv state (its last three entries) and the bf16 rounding of the conv
// output and of the SiLU, as in the one-token step.  Reads the state only.
__global__ void conv1d_prefill_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs_b, int64_t xs_t,
                                      const __nv_bfloat16* __restrict__ state, const __nv_bfloat16* __restrict__ w,
                                      __nv_bfloat16* __restrict__ out, int64_t os_b, int64_t os_t, int T,
                                      int channels) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.z;
  if (c >= channels) return;
  const int t0 = blockIdx.y * kConvTile;
  const int t1 = min(T, t0 + kConvTile);
  const __nv_bfloat16* st = state + (static_cast<int64_t>(b) * channels + c) * 4;
  const __nv_bfloat16* xc = x + static_cast<int64_t>(b) * xs_b + c;
  auto hist = [&](int t) -> float {  // input at token t (t < 0 reads the state)
    return t >= 0 ? __bfloat162float(xc[static_cast<int64_t>(t) * xs_t]) : __bfloat162float(st[4 + t]);
  };
  const float w0 = __bfloat162float(w[c * 4 + 0]), w1 = __bfloat162float(w[c * 4 + 1]);
  const float w2 = __bfloat162float(w[c * 4 + 2]), w3 = __bfloat162float(w[c * 4 + 3]);
  float h0 = hist(t0 - 3), h1 = hist(t0 - 2), h2 = hist(t0 - 1);
  __nv_bfloat16* oc = out + static_cast<int64_t>(b) * os_b + c;
  for (int t = t0; t < t1; ++t) {
    const float h3 = __bfloat162float(xc[static_cast<int64_t>(t) * xs_t]);
    float acc = w0 * h0;
    acc = fmaf(w1, h1, acc);
    acc = fmaf(w2, h2, acc);
    acc = fmaf(w3, h3, acc);
    const float y = bf16_round(acc);
    oc[static_cast<int64_t>(t) * os_t] = __float2bfloat16_rn(y / (1.0f + expf(-y)));
    h0 = h1;
    h1 = h2;
    h2 = h3;
  }
}

// The same conv for aligned channel pairs: a thread owns two channels and
// eight consecutive tokens, loads its eleven inputs (three of history from x
// or the state, then its own eight) at once and writes eight bf16 pairs, so
// every thread has one round trip to memory in flight instead of a serial
// walk over the prompt.  Same arithmetic and order as conv1d_prefill_kernel.
constexpr int kConvGroup = 8;
__global__ void __launch_bounds__(256) conv1d_prefill_pairs_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t xs_b, int64_t xs_t, const __nv_bfloat16* __restrict__ state,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int64_t os_b, int64_t os_t, int T,
    int pairs, int groups) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (idx >= static_cast<int64_t>(pairs) * groups) return;
  const int c = 2 * static_cast<int>(idx % pairs);
  const int t0 = static_cast<int>(idx / pairs) * kConvGroup;
  const __nv_bfloat16* xc = x + static_cast<int64_t>(b) * xs_b + c;
  const __nv_bfloat16* st = state + (static_cast<int64_t>(b) * 2 * pairs + c) * 4;  // channel c, then c + 1
  float2 h[kConvGroup + 3];  // inputs at tokens t0 - 3 .. t0 + 7
#pragma unroll
  for (int i = 0; i < kConvGroup + 3; ++i) {
    const int t = t0 - 3 + i;
    if (t >= 0) {
      h[i] = t < T ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xc + static_cast<int64_t>(t) * xs_t))
                   : make_float2(0.f, 0.f);
    } else {
      h[i] = make_float2(__bfloat162float(st[4 + t]), __bfloat162float(st[8 + t]));
    }
  }
  float w0[4], w1[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    w0[j] = __bfloat162float(w[c * 4 + j]);
    w1[j] = __bfloat162float(w[c * 4 + 4 + j]);
  }
  __nv_bfloat16* oc = out + static_cast<int64_t>(b) * os_b + c;
#pragma unroll
  for (int k = 0; k < kConvGroup; ++k) {
    const int t = t0 + k;
    if (t >= T) break;
    float a0 = w0[0] * h[k].x, a1 = w1[0] * h[k].y;
    a0 = fmaf(w0[1], h[k + 1].x, a0);
    a1 = fmaf(w1[1], h[k + 1].y, a1);
    a0 = fmaf(w0[2], h[k + 2].x, a0);
    a1 = fmaf(w1[2], h[k + 2].y, a1);
    a0 = fmaf(w0[3], h[k + 3].x, a0);
    a1 = fmaf(w1[3], h[k + 3].y, a1);
    const float y0 = bf16_round(a0), y1 = bf16_round(a1);
    *reinterpret_cast<__nv_bfloat162*>(oc + static_cast<int64_t>(t) * os_t) =
        __floats2bfloat162_rn(y0 / (1.0f + expf(-y0)), y1 / (1.0f + expf(-y1)));
  }
}

// The same conv for 16-byte aligned rows: a thread owns eight channels and
// sixteen consecutive tokens, so that every load and store is a 16-byte
// vector (512 contiguous bytes of a token row per warp) and three history
// rows are re-read per sixteen tokens instead of per eight.  Same arithmetic
// and order per channel as conv1d_prefill_kernel.
constexpr int kVecCh = 8;
constexpr int kVecTok = 16;
__global__ void __launch_bounds__(256) conv1d_prefill_vec_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t xs_b, int64_t xs_t, const __nv_bfloat16* __restrict__ state,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int64_t os_b, int64_t os_t, int T,
    int octs, int groups) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (idx >= static_cast<int64_t>(octs) * groups) return;
  const int c = kVecCh * static_cast<int>(idx % octs);
  const int t0 = static_cast<int>(idx / octs) * kVecTok;
  const __nv_bfloat16* xc = x + static_cast<int64_t>(b) * xs_b + c;
  uint4 h[kVecTok + 3];  // inputs at tokens t0 - 3 .. t0 + 15, eight channels each
#pragma unroll
  for (int i = 0; i < kVecTok + 3; ++i) {
    const int t = t0 - 3 + i;
    if (t >= 0) {
      h[i] = t < T ? __ldg(reinterpret_cast<const uint4*>(xc + static_cast<int64_t>(t) * xs_t)) : make_uint4(0, 0, 0, 0);
    } else {  // from the conv state [channel][4]: entry 4 + t of channels c .. c + 7
      const __nv_bfloat16* st = state + (static_cast<int64_t>(b) * octs * kVecCh + c) * 4 + 4 + t;
      __nv_bfloat16 v[kVecCh];
#pragma unroll
      for (int e = 0; e < kVecCh; ++e) v[e] = st[4 * e];
      h[i] = *reinterpret_cast<const uint4*>(v);
    }
  }
  float wf[kVecCh][4];
#pragma unroll
  for (int q = 0; q < kVecCh * 4 / 8; ++q) {  // 32 weights as four 16-byte loads
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(w + c * 4) + q);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) wf[(8 * q + i) / 4][(8 * q + i) % 4] = __bfloat162float(e[i]);
  }
  __nv_bfloat16* oc = out + static_cast<int64_t>(b) * os_b + c;
#pragma unroll
  for (int k = 0; k < kVecTok; ++k) {
    const int t = t0 + k;
    if (t >= T) break;
    const __nv_bfloat16* a0 = reinterpret_cast<const __nv_bfloat16*>(&h[k]);
    const __nv_bfloat16* a1 = reinterpret_cast<const __nv_bfloat16*>(&h[k + 1]);
    const __nv_bfloat16* a2 = reinterpret_cast<const __nv_bfloat16*>(&h[k + 2]);
    const __nv_bfloat16* a3 = reinterpret_cast<const __nv_bfloat16*>(&h[k + 3]);
    __nv_bfloat16 r[kVecCh];
#pragma unroll
    for (int e = 0; e < kVecCh; ++e) {
      float acc = wf[e][0] * __bfloat162float(a0[e]);
      acc = fmaf(wf[e][1], __bfloat162float(a1[e]), acc);
      acc = fmaf(wf[e][2], __bfloat162float(a2[e]), acc);
      acc = fmaf(wf[e][3], __bfloat162float(a3[e]), acc);
      const float y = bf16_round(acc);
      r[e] = __float2bfloat16_rn(y / (1.0f + expf(-y)));
    }
    *reinterpret_cast<uint4*>(oc + static_cast<int64_t>(t) * os_t) = *reinterpret_cast<const uint4*>(r);
  }
}

// New conv state = the last four inputs of [state, x_0 .. x_{T-1}]; runs after
// conv1d_prefill_kernel so that every read of the old state came first.
__global__ void conv1d_state_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs_b, int64_t xs_t,
                                    __nv_bfloat16* state, int T, int channels) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= channels) return;
  __nv_bfloat16* st = state + (static_cast<int64_t>(b) * channels + c) * 4;
  const __nv_bfloat16* xc = x + static_cast<int64_t>(b) * xs_b + c;
  __nv_bfloat16 s[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = T - 4 + i;
    s[i] = t >= 0 ? xc[static_cast<int64_t>(t) * xs_t] : st[4 + t];  // t < 0: shifted old entry
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) st[i] = s[i];
}

__device__ __forceinline__ float softplus_torch(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b); rows x heads.
__global__ void gdn_gates_kernel(const __nv_bfloat16* __restrict__ a, int64_t as, const __nv_bfloat16* __restrict__ bb,
                                 int64_t bs, const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                 float* __restrict__ g, float* __restrict__ beta, int rows, int heads) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * heads) return;
  const int r = idx / heads, h = idx % heads;
  const float av = __bfloat162float(a[static_cast<int64_t>(r) * as + h]);
  const float bv = __bfloat162float(bb[static_cast<int64_t>(r) * bs + h]);
  g[idx] = -expf(a_log[h]) * softplus_torch(av + dt_bias[h]);
  beta[idx] = 1.0f / (1.0f + expf(-bv));
}

// out = w * (o * rsqrt(mean(o^2) + 1e-6)) * silu(z) per 128-wide head,
// qwen36_gated_norm_probe.py:19-36.  One warp per (row, head).
__global__ void gated_rmsnorm_kernel(const __nv_bfloat16* __restrict__ o, int64_t os, const __nv_bfloat16* __restrict__ z,
                                     int64_t zs, const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                     int64_t outs, int rows, int heads) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows * heads) return;
  const int r = gw / heads, h = gw % heads;
  const __nv_bfloat16* orow = o + static_cast<int64_t>(r) * os + h * 128 + lane * 4;
  const __nv_bfloat16* zrow = z + static_cast<int64_t>(r) * zs + h * 128 + lane * 4;
  float v[4], zz[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __bfloat162float(orow[i]);
    zz[i] = __bfloat162float(zrow[i]);
  }
  const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  const float rn = rsqrtf(ss * (1.0f / 128) + 1e-6f);
  __nv_bfloat16* dst = out + static_cast<int64_t>(r) * outs + h * 128 + lane * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    dst[i] = __float2bfloat16_rn(w[lane * 4 + i] * (v[i] * rn) * (zz[i] / (1.0f + expf(-zz[i]))));
}

}  // namespace

extern "C" int ria_conv1d_prefill(const void* x, int64_t x_stride_b, int64_t x_stride_t, void* conv_state,
                                  const void* weight, void* out, int64_t out_stride_b, int64_t out_stride_t,
                                  int32_t batch, int32_t seq_len, int32_t channels, ria_stream_t stream) {
  if (batch < 0 || seq_len < 0 || channels <= 0) return ria::fail(RIA_ERR_INVALID, "ria_conv1d_prefill: bad sizes");
  if (batch == 0 || seq_len == 0) return RIA_OK;
  if (!x || !conv_state || !weight || !out) return ria::fail(RIA_ERR_INVALID, "ria_conv1d_prefill: null pointer");
  if (batch > 65535 || (seq_len + kConvTile - 1) / kConvTile > 65535)
    return ria::fail(RIA_ERR_INVALID, "ria_conv1d_prefill: grid too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  __nv_bfloat16* sb = static_cast<__nv_bfloat16*>(conv_state);
  const bool vec_ok = channels % kVecCh == 0 && ria::aligned(x, 16) && ria::aligned(out, 16) &&
                      ria::aligned(weight, 16) && x_stride_b % 8 == 0 && x_stride_t % 8 == 0 &&
                      out_stride_b % 8 == 0 && out_stride_t % 8 == 0;
  const bool pairs_ok = channels % 2 == 0 && ria::aligned(x, 4) && ria::aligned(out, 4) && x_stride_b % 2 == 0 &&
                        x_stride_t % 2 == 0 && out_stride_b % 2 == 0 && out_stride_t % 2 == 0;
  const int groups = (seq_len + kConvGroup - 1) / kConvGroup;
  const int64_t threads = static_cast<int64_t>(channels / 2) * groups;
  const int vgroups = (seq_len + kVecTok - 1) / kVecTok;
  const int64_t vthreads = static_cast<int64_t>(channels / kVecCh) * vgroups;
  // the vector form once it fills the GPU (two 256-thread CTAs per SM or more);
  // short prompts keep the pairs form's eight-token threads and four times the CTAs
  if (vec_ok && static_cast<int64_t>(vthreads) * batch >= 2LL * 256 * ria::num_sms() &&
      (vthreads + 255) / 256 <= INT32_MAX) {
    conv1d_prefill_vec_kernel<<<dim3(static_cast<unsigned>((vthreads + 255) / 256), batch), 256, 0, st>>>(
        xb, x_stride_b, x_stride_t, sb, static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
        out_stride_b, out_stride_t, seq_len, channels / kVecCh, vgroups);
  } else if (pairs_ok && (threads + 255) / 256 <= INT32_MAX) {
    conv1d_prefill_pairs_kernel<<<dim3(static_cast<unsigned>((threads + 255) / 256), batch), 256, 0, st>>>(
        xb, x_stride_b, x_stride_t, sb, static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
        out_stride_b, out_stride_t, seq_len, channels / 2, groups);
  } else {
    dim3 grid((channels + 255) / 256, (seq_len + kConvTile - 1) / kConvTile, batch);
    conv1d_prefill_kernel<<<grid, 256, 0, st>>>(xb, x_stride_b, x_stride_t, sb,
                                                static_cast<const __nv_bfloat16*>(weight),
                                                static_cast<__nv_bfloat16*>(out), out_stride_b, out_stride_t, seq_len,
                                                channels);
  }
  int rc = ria::check_launch("ria_conv1d_prefill");
  if (rc) return rc;
  conv1d_state_kernel<<<dim3((channels + 255) / 256, batch), 256, 0, st>>>(xb, x_stride_b, x_stride_t, sb, seq_len,
                                                                           channels);
  return ria::check_launch("ria_conv1d_prefill (state)");
}

extern "C" int ria_gdn_gates(const void* a, int64_t a_stride, const void* b, int64_t b_stride, const float* a_log,
                             const float* dt_bias, float* g, float* beta, int32_t rows, int32_t heads,
                             ria_stream_t stream) {
  if (rows < 0 || heads <= 0) return ria::fail(RIA_ERR_INVALID, "ria_gdn_gates: bad sizes");
  if (rows == 0) return RIA_OK;
  if (!a || !b || !a_log || !dt_bias || !g || !beta) return ria::fail(RIA_ERR_INVALID, "ria_gdn_gates: null pointer");
  const int64_t n = static_cast<int64_t>(rows) * heads;
  gdn_gates_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(a), a_stride, static_cast<const __nv_bfloat16*>(b), b_stride, a_log, dt_bias,
      g, beta, rows, heads);
  return ria::check_launch("ria_gdn_gates");
}

extern "C" int ria_gated_rmsnorm(const void* o, int64_t o_stride, const void* z, int64_t z_stride,
                                 const float* weight, void* out, int64_t out_stride, int32_t rows, int32_t heads,
                                 ria_stream_t stream) {
  if (rows < 0 || heads <= 0) return ria::fail(RIA_ERR_INVALID, "ria_gated_rmsnorm: bad sizes");
  if (rows == 0) return RIA_OK;
  if (!o || !z || !weight || !out) return ria::fail(RIA_ERR_INVALID, "ria_gated_rmsnorm: null pointer");
  const int64_t warps = static_cast<int64_t>(rows) * heads;
  gated_rmsnorm_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(o), o_stride, static_cast<const __nv_bfloat16*>(z), z_stride, weight,
      static_cast<__nv_bfloat16*>(out), out_stride, rows, heads);
  return ria::check_launch("ria_gated_rmsnorm");
}
