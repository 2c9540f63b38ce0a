// Greedy head of a decode step: final RMSNorm, lm_head projection, argmax.
//
// Reference: run_forward_token (router-ia qwen36_chat_batch.py:181-207) ends
// with x = rmsnorm(x, final_norm) in fp32 (qwen36_op_probe.py:55-67), then on
// CUDA logits = F.linear(x, lm_head) under fp16 autocast (:194-199: both
// operands rounded to fp16, fp32 accumulation, fp16 logits), and
// sample_next (qwen36_mini_chat.py:75-78) with temperature <= 0 returns
// argmax(logits) -- the first index among equal maxima, as torch.argmax.
//
// B200 design.  The head reads the whole fp16 lm_head (151936 x 2048, 622 MB)
// once per step: HBM-bound.  For batches up to 8, ria_lm_head_greedy is a
// norm launch (B rows to fp16) and one weight stream: a persistent grid (two
// CTAs per SM), each warp streaming 16-row vocab tiles straight from HBM into
// mma.sync A fragments (the batch is the N = 8 side, fp16 operands, fp32
// accumulation as the autocast GEMM), the fp16-rounded logits compared on the
// fly against the lane's best.  CTAs publish their best (value, row) per
// token and the last CTA to finish reduces them (a fence and an atomic
// counter, no waiting).  Larger batches use ria_final_norm_f16, a library
// GEMM and ria_argmax_f16_rows.
#include <cuda_fp16.h>

#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

constexpr int kH = 2048;
constexpr int kKC = kH / 256;  // 16-byte chunks per lane per row
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBatch = 8;

struct Best {
  float v;
  int i;
};

// (value desc, index asc): true when a ranks before b.
__device__ __forceinline__ bool better(float av, int ai, float bv, int bi) {
  return av > bv || (av == bv && ai < bi);
}

// One CTA per row: out = fp16(x * rsqrt(mean(x^2) + 1e-6) * (1 + w)), the
// reference's fp32 RMSNorm followed by the autocast rounding to fp16.
__global__ void __launch_bounds__(256) final_norm_f16_kernel(const float* __restrict__ x, int64_t xs,
                                                             const float* __restrict__ w, __half* __restrict__ out,
                                                             int64_t os, int n) {
  __shared__ float red[8];
  const float* xr = x + blockIdx.x * xs;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(n) + 1e-6f);
  __half* o = out + blockIdx.x * os;
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 ww = *reinterpret_cast<const float4*>(w + i);
    const __half2 a = __floats2half2_rn(v.x * r * (1.f + ww.x), v.y * r * (1.f + ww.y));
    const __half2 b = __floats2half2_rn(v.z * r * (1.f + ww.z), v.w * r * (1.f + ww.w));
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&a);
    pk.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(o + i) = pk;
  }
}

// D (16 rows x 8 columns, fp32) += A (16 x 16, fp16, row) * B (16 x 8, fp16, col).
__device__ __forceinline__ void mma_f16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One warp stage: vocab rows r0 + g and r0 + g + 8 (clamped to the last row;
// their results are dropped), 128 columns from c0; lane (g, t) loads the 16
// bytes at column c0 + 32 q + 8 t of each row.  Within each 32 columns the
// MMA k index is permuted (lane t's 8 columns are k-step 0's {2t, 2t+1, 2t+8,
// 2t+9} then k-step 1's) and the activations are read with the same
// permutation, so every dot product is unchanged.
__device__ __forceinline__ void load_rows(uint4 (&buf)[8], const __half* __restrict__ wt, int64_t ws, int vocab, int r0,
                                          int c0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const __half* ra = wt + static_cast<int64_t>(min(r0 + g, vocab - 1)) * ws + c0 + 8 * t;
  const __half* rb = wt + static_cast<int64_t>(min(r0 + g + 8, vocab - 1)) * ws + c0 + 8 * t;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    buf[q] = __ldg(reinterpret_cast<const uint4*>(ra + 32 * q));
    buf[4 + q] = __ldg(reinterpret_cast<const uint4*>(rb + 32 * q));
  }
}

// Persistent grid; warp w takes 16-row vocab tiles w, w + W, ... (W warps in
// the grid), each over 16 stages of 128 columns, through two register buffers
// (one stage loading while the other multiplies).  The batch's normalised rows
// are the N = 8 side of mma.sync (columns >= batch are zero and ignored).
__global__ void __launch_bounds__(kThreads, 2)
    lm_head_greedy_kernel(const __half* __restrict__ hn, int batch, const __half* __restrict__ wt, int64_t ws,
                          int vocab, __half* __restrict__ logits, int64_t ls, int* __restrict__ next_ids,
                          Best* __restrict__ cand, unsigned* __restrict__ counter) {
  constexpr int kXS = kH + 32;  // staged row (fp16): 64 bytes past a multiple of 128, conflict-free B loads
  constexpr int kStages = kH / 128;
  __shared__ __align__(16) __half xs[kMaxBatch * kXS];
  __shared__ Best wbest[kWarps][kMaxBatch];
  __shared__ int last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int W = gridDim.x * kWarps, w0 = blockIdx.x * kWarps + warp;
  const int tiles = (vocab + 15) / 16;
  const int nst = w0 < tiles ? ((tiles - 1 - w0) / W + 1) * kStages : 0;
  auto tile_of = [&](int idx) { return w0 + (idx / kStages) * W; };
  uint4 ra[8], rb[8];
  if (nst > 0) load_rows(ra, wt, ws, vocab, tile_of(0) * 16, 0);
  if (nst > 1) load_rows(rb, wt, ws, vocab, tile_of(1) * 16, 128);
  for (int i = threadIdx.x; i < kMaxBatch * kH / 8; i += kThreads) {
    const int r = i / (kH / 8), c8 = (i % (kH / 8)) * 8;
    const uint4 v = r < batch ? reinterpret_cast<const uint4*>(hn)[i] : make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(xs + r * kXS + c8) = v;
  }
  __syncthreads();
  const __half* xrow = xs + g * kXS + 8 * t;  // this lane's token column (g) of the B fragments
  // best (value, row) of tokens 2t and 2t + 1 over this lane's rows
  Best best0 = {-INFINITY, 0x7fffffff}, best1 = {-INFINITY, 0x7fffffff};
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  auto stage = [&](const uint4 (&buf)[8], int idx) {
    const __half* xc = xrow + (idx % kStages) * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 bx = *reinterpret_cast<const uint4*>(xc + 32 * q);
      mma_f16_16816(acc, buf[q].x, buf[4 + q].x, buf[q].y, buf[4 + q].y, bx.x, bx.y);
      mma_f16_16816(acc, buf[q].z, buf[4 + q].z, buf[q].w, buf[4 + q].w, bx.z, bx.w);
    }
  };
  auto finish_tile = [&](int idx) {
    const int r0 = tile_of(idx) * 16;
    const int rows[4] = {r0 + g, r0 + g, r0 + g + 8, r0 + g + 8};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int tok = 2 * t + (j & 1);
      const __half l16 = __float2half_rn(acc[j]);
      const float lv = __half2float(l16);
      if (rows[j] < vocab && tok < batch) {
        if (logits) logits[tok * ls + rows[j]] = l16;
        Best& bb = (j & 1) ? best1 : best0;
        if (lv > bb.v || bb.i == 0x7fffffff) bb = {lv, rows[j]};  // rows rise per lane: the first max is kept
      }
      acc[j] = 0.f;
    }
  };
  for (int idx = 0; idx < nst; idx += 2) {
    stage(ra, idx);
    if (idx + 2 < nst) load_rows(ra, wt, ws, vocab, tile_of(idx + 2) * 16, ((idx + 2) % kStages) * 128);
    if (idx % kStages == kStages - 1) finish_tile(idx);
    if (idx + 1 < nst) {
      stage(rb, idx + 1);
      if (idx + 3 < nst) load_rows(rb, wt, ws, vocab, tile_of(idx + 3) * 16, ((idx + 3) % kStages) * 128);
      if ((idx + 1) % kStages == kStages - 1) finish_tile(idx + 1);
    }
  }
  // reduce over the 8 row groups (lanes with the same t), then over warps and CTAs
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best0.v, o);
    int oi = __shfl_xor_sync(0xffffffffu, best0.i, o);
    if (better(ov, oi, best0.v, best0.i)) best0 = {ov, oi};
    ov = __shfl_xor_sync(0xffffffffu, best1.v, o);
    oi = __shfl_xor_sync(0xffffffffu, best1.i, o);
    if (better(ov, oi, best1.v, best1.i)) best1 = {ov, oi};
  }
  if (g == 0) {
    wbest[warp][2 * t] = best0;
    wbest[warp][2 * t + 1] = best1;
  }
  __syncthreads();
  if (threadIdx.x < batch) {
    const int b = threadIdx.x;
    Best bb = wbest[0][b];
    for (int w = 1; w < kWarps; ++w)
      if (better(wbest[w][b].v, wbest[w][b].i, bb.v, bb.i)) bb = wbest[w][b];
    cand[blockIdx.x * kMaxBatch + b] = bb;
  }
  // the last CTA to finish reduces every CTA's candidates
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(counter, 1u);
    last = prev + 1 == gridDim.x;
    if (last) *counter = 0u;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (warp < batch) {
    const int b = warp;
    Best bb = {-INFINITY, 0x7fffffff};
    for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
      const float v = __ldcg(&cand[c * kMaxBatch + b].v);
      const int i = __ldcg(&cand[c * kMaxBatch + b].i);
      if (better(v, i, bb.v, bb.i)) bb = {v, i};
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bb.v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bb.i, o);
      if (better(ov, oi, bb.v, bb.i)) bb = {ov, oi};
    }
    if (lane == 0) next_ids[b] = bb.i;
  }
}

// One 1024-thread CTA per row: the first index of the largest fp16 logit.
// 16-byte loads when the row start and length allow (8 logits per load),
// indices rising per thread so the first maximum is kept.
__global__ void __launch_bounds__(1024) argmax_f16_rows_kernel(const __half* __restrict__ logits, int64_t ls,
                                                               int vocab, int* __restrict__ out) {
  __shared__ Best wb[32];
  const __half* row = logits + blockIdx.x * ls;
  Best bb = {-INFINITY, 0x7fffffff};
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int nvec = vec ? vocab / 8 : 0;
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + c * 8);
    const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = __half2float(h[e]);
      if (v > bb.v || bb.i == 0x7fffffff) bb = {v, c * 8 + e};
    }
  }
  for (int i = nvec * 8 + threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = __half2float(row[i]);
    if (better(v, i, bb.v, bb.i) || bb.i == 0x7fffffff) bb = {v, i};
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bb.v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bb.i, o);
    if (better(ov, oi, bb.v, bb.i)) bb = {ov, oi};
  }
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = bb;
  __syncthreads();
  if (threadIdx.x < 32) {
    bb = wb[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bb.v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bb.i, o);
      if (better(ov, oi, bb.v, bb.i)) bb = {ov, oi};
    }
    if (threadIdx.x == 0) out[blockIdx.x] = bb.i;
  }
}

int grid_ctas() { return 2 * ria::num_sms(); }

}  // namespace

// Workspace: the counter (256 bytes, zero before the first call; every call
// leaves it at zero), the normalised fp16 rows [batch][kH], then the per-CTA
// candidates.
extern "C" int64_t ria_lm_head_workspace_bytes(int32_t batch) {
  if (batch <= 0) return 0;
  return 256 + static_cast<int64_t>(kMaxBatch) * kH * 2 +
         static_cast<int64_t>(grid_ctas()) * kMaxBatch * static_cast<int64_t>(sizeof(Best));
}

extern "C" int ria_lm_head_greedy(const float* x, int64_t x_stride, const float* norm_weight, const void* lm_head,
                                  int64_t w_stride, int32_t vocab, void* logits, int64_t logits_stride,
                                  int32_t* next_ids, void* workspace, int64_t workspace_bytes, int32_t batch,
                                  ria_stream_t stream) {
  if (batch < 0 || batch > kMaxBatch)
    return ria::fail(RIA_ERR_INVALID, "ria_lm_head_greedy: batch %d outside 0..%d", batch, kMaxBatch);
  if (batch == 0) return RIA_OK;
  if (vocab <= 0) return ria::fail(RIA_ERR_INVALID, "ria_lm_head_greedy: vocab %d", vocab);
  if (!x || !norm_weight || !lm_head || !next_ids || !workspace)
    return ria::fail(RIA_ERR_INVALID, "ria_lm_head_greedy: null pointer argument");
  if (workspace_bytes < ria_lm_head_workspace_bytes(batch))
    return ria::fail(RIA_ERR_INVALID, "ria_lm_head_greedy: workspace of %lld bytes, %lld needed",
                     static_cast<long long>(workspace_bytes),
                     static_cast<long long>(ria_lm_head_workspace_bytes(batch)));
  if (!ria::aligned(x, 16) || !ria::aligned(norm_weight, 16) || !ria::aligned(lm_head, 16) ||
      !ria::aligned(workspace, 16) || x_stride % 4 || w_stride % 8 || w_stride < kH)
    return ria::fail(RIA_ERR_INVALID, "ria_lm_head_greedy: rows must be 16-byte aligned (w_stride >= %d)", kH);
  if (logits && logits_stride < vocab)
    return ria::fail(RIA_ERR_INVALID, "ria_lm_head_greedy: logits_stride < vocab");
  unsigned char* wsb = static_cast<unsigned char*>(workspace);
  unsigned* counter = reinterpret_cast<unsigned*>(wsb);
  __half* hn = reinterpret_cast<__half*>(wsb + 256);
  Best* cand = reinterpret_cast<Best*>(wsb + 256 + static_cast<int64_t>(kMaxBatch) * kH * 2);
  const auto* w = static_cast<const __half*>(lm_head);
  auto* lg = static_cast<__half*>(logits);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  final_norm_f16_kernel<<<batch, 256, 0, st>>>(x, x_stride, norm_weight, hn, kH, kH);
  const int rc = ria::check_launch("ria_lm_head_greedy (norm)");
  if (rc) return rc;
  lm_head_greedy_kernel<<<grid_ctas(), kThreads, 0, st>>>(hn, batch, w, w_stride, vocab, lg, logits_stride, next_ids,
                                                           cand, counter);
  return ria::check_launch("ria_lm_head_greedy");
}

extern "C" int ria_final_norm_f16(const float* x, int64_t x_stride, const float* weight, void* out,
                                  int64_t out_stride, int32_t rows, int32_t n, ria_stream_t stream) {
  if (rows < 0 || n <= 0 || n % 4 != 0) return ria::fail(RIA_ERR_INVALID, "ria_final_norm_f16: bad rows/n");
  if (rows == 0) return RIA_OK;
  if (!x || !weight || !out) return ria::fail(RIA_ERR_INVALID, "ria_final_norm_f16: null pointer");
  if (!ria::aligned(x, 16) || !ria::aligned(weight, 16) || !ria::aligned(out, 8) || x_stride % 4 || out_stride % 4)
    return ria::fail(RIA_ERR_INVALID, "ria_final_norm_f16: misaligned rows");
  final_norm_f16_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, x_stride, weight,
                                                                               static_cast<__half*>(out), out_stride, n);
  return ria::check_launch("ria_final_norm_f16");
}

extern "C" int ria_argmax_f16_rows(const void* logits, int64_t stride, int32_t vocab, int32_t rows, int32_t* out,
                                   ria_stream_t stream) {
  if (rows < 0 || vocab <= 0 || stride < vocab)
    return ria::fail(RIA_ERR_INVALID, "ria_argmax_f16_rows: bad rows/vocab/stride");
  if (rows == 0) return RIA_OK;
  if (!logits || !out) return ria::fail(RIA_ERR_INVALID, "ria_argmax_f16_rows: null pointer");
  argmax_f16_rows_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const __half*>(logits),
                                                                                stride, vocab, out);
  return ria::check_launch("ria_argmax_f16_rows");
}
