// K5: the MoE block of a decode step for a batch of tokens: router top-k,
// the chosen experts' SwiGLU FFNs, the gated shared expert and the residual
// add.  Weights bf16 (the checkpoint's), activations and accumulation fp32.
//
// Reference semantics: router-ia's batched_moe_step (qwen36_chat_batch.py:
// 127-178) run one token at a time, with route (qwen36_router.py:96-133) and
// the Qwen RMSNorm (qwen36_op_probe.py:55-67):
//   moe_in = x * rsqrt(mean(x^2) + 1e-6) * (1 + w_post)
//   logits = moe_in . W_router^T (fp32); top-k; weights = softmax(top-k logits)
//   out = x + sum_j weights_j * down_e(silu(gate_e moe_in) * up_e moe_in)
//           + sigmoid(moe_in . w_sg) * down_s(silu(gate_s moe_in) * up_s moe_in)
//
// B200 design.  At decode batch sizes the block is bound by the bytes of the
// experts that some token chose (6 MB of bf16 weights per expert: 54 MB for
// one token, about 1.3 GB for 64 tokens), so the expert kernels are weight
// streams: every weight byte is loaded once, straight from HBM into MMA
// fragments, and applied to all of that expert's tokens at once.  Two
// launches:
//   * moe_route_kernel, a CTA per (8 or 16 router rows, 8 tokens): the norm of its
//     tokens, then router and shared-gate logits (fp32 sums over the bf16
//     rows).  The last CTA to finish a token group takes the group's top-k
//     (a warp per token: rounds of a warp-wide max, ties to the lower expert
//     id as a stable sort picks), the softmax of the chosen logits and the
//     shared-gate sigmoid; the last group to finish writes the plan: for each
//     expert some token chose, units of up to 8 of its (token, slot) pairs in
//     token order, then the shared expert's units of 8 tokens.  Experts
//     nobody chose get no unit; their weights are never read.
//   * moe_experts_kernel, persistent and cooperative (every CTA resident),
//     two phases per CTA:
//     - gate/up over 16-row tiles: finds a unit's pairs in the routing
//       table, stages their activations in SMEM as bf16 hi + lo parts; warps
//       stream gate / up rows through mma.sync m16n8k16 (weight rows = M,
//       activations = N, fp32 accumulation) with the next stage's loads in
//       flight, write h = silu(gate) * up per (token, slot) and publish the
//       unit's finished tiles on a per-unit counter;
//     - down over 128-row tiles of the down rows (a warp per 16 rows, all
//       512 columns), each segment starting once its unit's gate/up tiles
//       are all published (a bounded wait): y[token][slot] = scale * down .
//       h, scale = the slot's router weight (the shared gate for the shared
//       slot).  The CTA that finishes the last of a (token, tile)'s k + 1
//       slots writes that piece of the output: x + (routed slots summed in
//       slot order + shared slot).
// "Last CTA" hand-offs use a fence and an atomic counter (no waiting); the
// last arrival resets the counter, so the workspace counters stay zero
// between calls.  Every sum runs in a fixed order: results are deterministic
// run to run.
//
// The N side of an expert's GEMM is at most 8 tokens (two bf16 parts each),
// too narrow for a tcgen05 MMA (M = 128, N >= 16), whose issue cost per 16
// weight columns would then bound the stream instead of HBM.  mma.sync takes
// its A operand from the registers the weight rows are loaded into, so the
// weights need no SMEM staging; units of at most 4 tokens pack their hi and
// lo parts into the 8 columns of one MMA, halving the MMA count.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

constexpr int kH = 2048;          // hidden size
constexpr int kI = 512;           // expert and shared-expert intermediate size
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 16;
constexpr int kMaxPairs = 2048;   // batch * top_k per launch
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTokens = 8;        // tokens per unit and per route CTA
constexpr int kLogitSmem = kTokens * kH * 4;
constexpr int kGuTiles = kI / 16;  // 16-row gate/up tiles per unit
constexpr int kDnRows = 16 * kWarps;  // down rows per tile: 16 per warp
constexpr int kDnTiles = kH / kDnRows;  // down tiles per unit
constexpr int kXStride = kH + 32;  // staged activation row (bf16): 64 bytes past a multiple of 128
constexpr int kHStride = kI + 32;
constexpr int kMaxGroups = kMaxPairs / kTokens;

struct MoeParams {
  const float* residual;
  int64_t rs;
  const __nv_bfloat16* post_w;
  const __nv_bfloat16* router_w;       // [E][kH]
  const __nv_bfloat16* shared_gate_w;  // [kH]
  const __nv_bfloat16* eg;             // [E][kI][kH]
  const __nv_bfloat16* eu;             // [E][kI][kH]
  const __nv_bfloat16* ed;             // [E][kH][kI]
  const __nv_bfloat16* sgp;            // [kI][kH]
  const __nv_bfloat16* sup;            // [kI][kH]
  const __nv_bfloat16* sdp;            // [kH][kI]
  float* out;
  int64_t os;
  int32_t* ids;   // [B][k]
  float* wts;     // [B][k]
  float* sgate;   // [B]
  float* xin;     // [B][kH] expert input
  float* logits;  // [B][E + 1]
  float* hbuf;    // [B][k + 1][kI]
  float* ybuf;    // [B][k + 1][kH]
  int4* units;    // {expert, first rank among the expert's pairs (shared: first token), pairs, 0}
  int* n_units;
  unsigned* cnt_group;  // [kMaxGroups] route CTAs done per token group
  unsigned* cnt_plan;   // token groups done
  unsigned* cnt_out;    // [B][kDnTiles] slots done per (token, down row tile)
  unsigned* unit_done;  // [units] gate/up tiles finished per unit (zeroed by the plan)
  unsigned int* err;    // device error word
  int B, E, k;
};

__device__ __forceinline__ void bf16x8(const uint4& u, float* f) {
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 v = __bfloat1622float2(h2[e]);
    f[2 * e] = v.x;
    f[2 * e + 1] = v.y;
  }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// After a CTA's global writes: true in the CTA whose arrival completes the
// group of `expected` CTAs counted by *counter, which also resets the counter.
__device__ __forceinline__ bool last_arrival(unsigned* counter, unsigned expected, int* flag) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(counter, 1u);
    *flag = prev + 1 == expected;
    if (*flag) *counter = 0u;
  }
  __syncthreads();
  if (*flag) __threadfence();
  return *flag;
}

// Top-k of token b's router logits by one warp: k rounds of a warp argmax
// over the remaining experts (kPer logits per lane), the softmax of the
// chosen logits and the shared-gate sigmoid.
template <int kPer>
__device__ __forceinline__ void topk_token(const MoeParams& p, int b) {
  const int lane = threadIdx.x & 31;
  const float* lg = p.logits + static_cast<int64_t>(b) * (p.E + 1);
  float v[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < p.E ? __ldcg(lg + e) : -INFINITY;
  }
  float my_sel = -INFINITY;  // lane j < k: the logit and id chosen in round j
  int my_id = 0;
  unsigned taken = 0;  // bit i: expert lane + 32 i already chosen
  for (int rnd = 0; rnd < p.k; ++rnd) {
    // this lane's best remaining expert: the largest logit, the lowest id
    // among equals (ids rise with i)
    float best = -INFINITY;
    int bi = -1;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < p.E && !((taken >> i) & 1u) && (bi < 0 || v[i] > best)) {
        best = v[i];
        bi = e;
      }
    }
    // the warp's largest (order-preserving integer key), then the lowest id
    // holding it; some expert always remains (k <= E)
    const unsigned bits = __float_as_uint(best);
    const unsigned key = bi < 0 ? 0u : ((bits & 0x80000000u) ? ~bits : bits | 0x80000000u);
    const unsigned top = __reduce_max_sync(0xffffffffu, key);
    const unsigned id = __reduce_min_sync(0xffffffffu, (bi >= 0 && key == top) ? static_cast<unsigned>(bi) : 0xffffffffu);
    if (lane == rnd) {
      my_sel = __uint_as_float((top & 0x80000000u) ? top & 0x7fffffffu : ~top);
      my_id = static_cast<int>(id);
    }
    if (static_cast<int>(id & 31u) == lane) taken |= 1u << (id >> 5);
  }
  // softmax over the chosen logits (round 0 holds the largest)
  const float m = __shfl_sync(0xffffffffu, my_sel, 0);
  const float ex = lane < p.k ? expf(my_sel - m) : 0.f;
  const float den = warp_sum(ex);
  if (lane < p.k) {
    p.ids[b * p.k + lane] = my_id;
    p.wts[b * p.k + lane] = ex / den;
  }
  if (lane == 0) p.sgate[b] = 1.0f / (1.0f + expf(-__ldcg(lg + p.E)));
}

// The plan, by one CTA: the unit list -- for each expert some token chose
// (ascending id), units of up to kTokens of its pairs in token order, then the
// shared expert's units of kTokens tokens.  Thread tid owns experts
// 4 tid .. 4 tid + 3 (E <= 1024).
__device__ void build_plan(const MoeParams& p) {
  __shared__ int cnt[kMaxExperts];
  __shared__ int wsum_u[kWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int total = p.B * p.k;
  for (int e = tid; e < kMaxExperts; e += kThreads) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < total; i += kThreads) atomicAdd(&cnt[__ldcg(p.ids + i)], 1);
  __syncthreads();
  int c[4], u[4], su = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    c[j] = cnt[4 * tid + j];  // zero past E
    u[j] = (c[j] + kTokens - 1) / kTokens;
    su += u[j];
  }
  int iu = su;  // inclusive scan over the CTA
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int vu = __shfl_up_sync(0xffffffffu, iu, o);
    if (lane >= o) iu += vu;
  }
  if (lane == 31) wsum_u[warp] = iu;
  __syncthreads();
  int pu = iu - su, routed_units = 0;
  for (int w = 0; w < kWarps; ++w) {
    if (w < warp) pu += wsum_u[w];
    routed_units += wsum_u[w];
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    for (int q = 0; q < u[j]; ++q)
      p.units[pu + q] = make_int4(4 * tid + j, q * kTokens, min(kTokens, c[j] - q * kTokens), 0);
    pu += u[j];
  }
  const int shared_units = (p.B + kTokens - 1) / kTokens;
  for (int q = tid; q < shared_units; q += kThreads)
    p.units[routed_units + q] = make_int4(p.E, q * kTokens, min(kTokens, p.B - q * kTokens), 0);
  for (int q = tid; q < routed_units + shared_units; q += kThreads) p.unit_done[q] = 0u;
  if (tid == 0) *p.n_units = routed_units + shared_units;
}

// kRowsPerWarp router rows per warp, 8 kRowsPerWarp per CTA: one row for a
// single token group (a shorter logits chain per warp, twice the CTAs), two
// for more groups (each CTA also recomputes its group's norms).
template <int kPer, int kRowsPerWarp>
__global__ void __launch_bounds__(kThreads) moe_route_kernel(const MoeParams p) {
  constexpr int kLogitRows = kRowsPerWarp * kWarps;
  extern __shared__ __align__(16) unsigned char smem[];
  float* xs = reinterpret_cast<float*>(smem);  // [kTokens][kH]
  __shared__ int flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.y * kTokens;
  const int nt = min(kTokens, p.B - t0);
  // warp w < nt: the norm of token t0 + w.  Its row and the norm weight are
  // loaded first, then this warp's router row (row E is the shared gate),
  // which stay in flight while the norm runs.
  float4 v[kH / 128];
  float2 wa[kH / 128], wb[kH / 128];
  if (warp < nt) {
    const float* x = p.residual + static_cast<int64_t>(t0 + warp) * p.rs;
#pragma unroll
    for (int i = 0; i < kH / 128; ++i) {
      const int d = i * 128 + lane * 4;
      v[i] = *reinterpret_cast<const float4*>(x + d);
      wa[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p.post_w + d));
      wb[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p.post_w + d + 2));
    }
  }
  const int rbase = blockIdx.x * kLogitRows + warp * kRowsPerWarp;
  uint4 w[kRowsPerWarp][kH / 256];
#pragma unroll
  for (int q = 0; q < kRowsPerWarp; ++q) {
    const int r = min(rbase + q, p.E);
    const __nv_bfloat16* wr = r < p.E ? p.router_w + static_cast<int64_t>(r) * kH : p.shared_gate_w;
#pragma unroll
    for (int c = 0; c < kH / 256; ++c) w[q][c] = __ldg(reinterpret_cast<const uint4*>(wr + c * 256 + lane * 8));
  }
  if (warp < nt) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kH / 128; ++i)
      ss = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, ss))));
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(kH) + 1e-6f);
    float* xo = p.xin + static_cast<int64_t>(t0 + warp) * kH;
#pragma unroll
    for (int i = 0; i < kH / 128; ++i) {
      const int d = i * 128 + lane * 4;
      const float4 m = make_float4(v[i].x * r * (1.0f + wa[i].x), v[i].y * r * (1.0f + wa[i].y),
                                   v[i].z * r * (1.0f + wb[i].x), v[i].w * r * (1.0f + wb[i].y));
      *reinterpret_cast<float4*>(xs + warp * kH + d) = m;
      if (blockIdx.x == 0) *reinterpret_cast<float4*>(xo + d) = m;
    }
  }
  __syncthreads();
  float acc[kRowsPerWarp][kTokens];
#pragma unroll
  for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
    for (int t = 0; t < kTokens; ++t) acc[q][t] = 0.f;
#pragma unroll
  for (int c = 0; c < kH / 256; ++c) {
    float wf[kRowsPerWarp][8];
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q) bf16x8(w[q][c], wf[q]);
#pragma unroll
    for (int t = 0; t < kTokens; ++t) {
      if (t < nt) {
        const float4 xa = *reinterpret_cast<const float4*>(xs + t * kH + c * 256 + lane * 8);
        const float4 xb = *reinterpret_cast<const float4*>(xs + t * kH + c * 256 + lane * 8 + 4);
        const float xf[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[q][t] = fmaf(wf[q][j], xf[j], acc[q][t]);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
    for (int t = 0; t < kTokens; ++t) {
      if (t < nt) {
        const float s = warp_sum(acc[q][t]);
        if (lane == 0 && rbase + q <= p.E) p.logits[static_cast<int64_t>(t0 + t) * (p.E + 1) + rbase + q] = s;
      }
    }
  // the last CTA of this token group: top-k of its tokens
  if (!last_arrival(p.cnt_group + blockIdx.y, gridDim.x, &flag)) return;
  if (warp < nt) topk_token<kPer>(p, t0 + warp);
  // the last token group: the plan (one group: this CTA already is)
  if (gridDim.y > 1) {
    if (!last_arrival(p.cnt_plan, gridDim.y, &flag)) return;
  } else {
    __syncthreads();
  }
  build_plan(p);
}

__device__ __forceinline__ int64_t pair_row(const MoeParams& p, int pr) {
  return static_cast<int64_t>(pr / kMaxTopK) * (p.k + 1) + (pr % kMaxTopK);
}

// Activations of a unit's token as bf16 hi + lo parts (hi = bf16(v),
// lo = bf16(v - hi)), so that two bf16 MMAs against the bf16 weights give
// the fp32 product to about 2^-17 relative.  Rows padded so that the B
// fragment loads (8 rows x 64 contiguous bytes) hit all 32 banks.
__device__ __forceinline__ void stage_split(const float* __restrict__ src, int len, __nv_bfloat16* xh,
                                            __nv_bfloat16* xl) {
  for (int c4 = threadIdx.x * 4; c4 < len; c4 += kThreads * 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src + c4));
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y);
    const __nv_bfloat162 l23 = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
    uint2 hv, lv;
    hv.x = *reinterpret_cast<const uint32_t*>(&h01);
    hv.y = *reinterpret_cast<const uint32_t*>(&h23);
    lv.x = *reinterpret_cast<const uint32_t*>(&l01);
    lv.y = *reinterpret_cast<const uint32_t*>(&l23);
    *reinterpret_cast<uint2*>(xh + c4) = hv;
    *reinterpret_cast<uint2*>(xl + c4) = lv;
  }
}

// One stage of a warp's weight stream: rows g and g + 8 of a 16-row tile, 4
// k-step pairs of 32 columns; lane (g, t) loads the 16 bytes at column
// 32 q + 8 t of each row.  Within each 32 columns the MMA k index is permuted
// (lane t's 8 columns are k-step 0's {2t, 2t+1, 2t+8, 2t+9} then k-step 1's),
// and the activations are read with the same permutation, so the dot product
// is unchanged.
__device__ __forceinline__ void load_stage(uint4 (&buf)[8], const __nv_bfloat16* row_g, int64_t row_stride) {
  const __nv_bfloat16* row_g8 = row_g + 8 * row_stride;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    buf[q] = __ldg(reinterpret_cast<const uint4*>(row_g + 32 * q));
    buf[4 + q] = __ldg(reinterpret_cast<const uint4*>(row_g8 + 32 * q));
  }
}

// acc (16 rows x 8 columns) += the stage's weights . activations.  kPacked:
// column n < 4 is token n's hi part, n >= 4 token n - 4's lo part (one MMA per
// k-step; xa is this lane's row of that layout).  Otherwise column n is
// token n, hi (xa) and lo (xb) accumulate into it by two MMAs.
template <bool kPacked>
__device__ __forceinline__ void mma_stage(float (&acc)[4], const uint4 (&buf)[8], const __nv_bfloat16* xa,
                                          const __nv_bfloat16* xb) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 bh = *reinterpret_cast<const uint4*>(xa + 32 * q);
    mma_bf16_16816(acc, buf[q].x, buf[4 + q].x, buf[q].y, buf[4 + q].y, bh.x, bh.y);
    mma_bf16_16816(acc, buf[q].z, buf[4 + q].z, buf[q].w, buf[4 + q].w, bh.z, bh.w);
    if (!kPacked) {
      const uint4 bl = *reinterpret_cast<const uint4*>(xb + 32 * q);
      mma_bf16_16816(acc, buf[q].x, buf[4 + q].x, buf[q].y, buf[4 + q].y, bl.x, bl.y);
      mma_bf16_16816(acc, buf[q].z, buf[4 + q].z, buf[q].w, buf[4 + q].w, bl.z, bl.w);
    }
  }
}

__device__ __forceinline__ void store_partial(float* red, const float (&acc)[4], int g, int t) {
  red[g * kTokens + 2 * t] = acc[0];
  red[g * kTokens + 2 * t + 1] = acc[1];
  red[(g + 8) * kTokens + 2 * t] = acc[2];
  red[(g + 8) * kTokens + 2 * t + 1] = acc[3];
}

// A warp's stream of nst stages (two register buffers, one stage loading
// while the other multiplies).  addr(idx) gives stage idx's weight row g (the
// caller loaded stages 0 and 1), xcol(idx) its first activation column,
// done(idx, acc) runs after each stage.
template <bool kPacked, class Addr, class XCol, class Done>
__device__ __forceinline__ void stream_stages(int nst, int64_t row_stride, const __nv_bfloat16* xa_row,
                                              const __nv_bfloat16* xb_row, Addr&& addr, XCol&& xcol, Done&& done,
                                              uint4 (&ra)[8], uint4 (&rb)[8]) {
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int idx = 0; idx < nst; idx += 2) {
    {
      const int c = xcol(idx);
      mma_stage<kPacked>(acc, ra, xa_row + c, xb_row + c);
      if (idx + 2 < nst) load_stage(ra, addr(idx + 2), row_stride);
      done(idx, acc);
    }
    if (idx + 1 < nst) {
      const int c = xcol(idx + 1);
      mma_stage<kPacked>(acc, rb, xa_row + c, xb_row + c);
      if (idx + 3 < nst) load_stage(rb, addr(idx + 3), row_stride);
      done(idx + 1, acc);
    }
  }
}

// A warp's partial for (row, token n) in the reduction buffer: packed units
// hold the hi and lo parts in columns n and n + 4.
__device__ __forceinline__ float partial(const float* red_row, int n, bool packed) {
  return packed ? red_row[n] + red_row[n + 4] : red_row[n];
}

// The unit's pairs (token * kMaxTopK + slot) into pr_s, in token order: for
// a routed expert the pairs of rank [start, start + ntok) among the pairs
// that chose it, found by warp 0 from the routing table staged in ids_s; for
// the shared expert tokens start .. start + ntok - 1 with slot k.
__device__ __forceinline__ void unit_pairs(const MoeParams& p, int e, int start, int ntok, const int* ids_s,
                                           int* pr_s) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (e == p.E) {
    if (tid < ntok) pr_s[tid] = (start + tid) * kMaxTopK + p.k;
  } else if (tid < 32) {
    const int total = p.B * p.k;
    int rank = 0;
    for (int i0 = 0; i0 < total && rank < start + ntok; i0 += 32) {
      const int i = i0 + lane;
      const bool hit = i < total && ids_s[i] == e;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      const int r = rank + __popc(m & ((1u << lane) - 1u));
      if (hit && r >= start && r < start + ntok) pr_s[r - start] = (i / p.k) * kMaxTopK + (i % p.k);
      rank += __popc(m);
    }
  }
}

// The expert kernels run a persistent grid over the flattened list of
// (unit, tile) pairs: CTA c takes the contiguous range [c T / G, (c + 1) T / G)
// of the T = units x tiles pairs, so every CTA streams the same number of
// weight bytes (within one tile) and no partial last wave idles the machine.
// A range crosses into a new unit a few times; each crossing re-stages the
// activations.  seg(tt) gives the segment that starts at flattened index tt.
struct Segment {
  int unit, ta, tb;  // tiles [ta, tb) of unit
};

__device__ __forceinline__ Segment segment_at(int64_t tt, int64_t t_end, int tiles) {
  Segment sg;
  sg.unit = static_cast<int>(tt / tiles);
  sg.ta = static_cast<int>(tt % tiles);
  const int64_t end = sg.ta + (t_end - tt);
  sg.tb = static_cast<int>(end < tiles ? end : tiles);
  return sg;
}

// gate/up: tiles of 16 rows.  Warps 0-3 stream the gate rows, warps 4-7 the
// up rows, each over a quarter of the 2048 columns; at each tile's end the
// quarters are summed in a fixed order and h = silu(gate) * up is written per
// (token, slot) for the down kernel.
__device__ __forceinline__ void gate_up_phase(const MoeParams& p, unsigned char* smem) {
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);  // rows 0-7 hi, 8-15 lo
  float* red = reinterpret_cast<float*>(xs + 2 * kTokens * kXStride);  // [2][8 warps][16][8]
  int* ids_s = reinterpret_cast<int*>(red + 2 * kWarps * 16 * kTokens);  // [B * k]
  __shared__ int pr_s[kTokens];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t total = static_cast<int64_t>(*p.n_units) * kGuTiles;
  const int64_t t_begin = total * blockIdx.x / gridDim.x, t_end = total * (blockIdx.x + 1) / gridDim.x;
  for (int i = tid; i < p.B * p.k; i += kThreads) ids_s[i] = p.ids[i];
  const int kq = (warp & 3) * (kH / 4);
  for (int64_t tt = t_begin; tt < t_end;) {
    const Segment sg = segment_at(tt, t_end, kGuTiles);
    tt += sg.tb - sg.ta;
    const int4 ui = p.units[sg.unit];
    const int e = ui.x, start = ui.y, ntok = ui.z;
    const bool shared = e == p.E, packed = ntok <= 4;
    const __nv_bfloat16* wm = warp < 4 ? (shared ? p.sgp : p.eg + static_cast<int64_t>(e) * kI * kH)
                                       : (shared ? p.sup : p.eu + static_cast<int64_t>(e) * kI * kH);
    auto addr = [&](int idx) {  // idx = (tile - ta) * 4 + stage
      return wm + static_cast<int64_t>((sg.ta + (idx >> 2)) * 16 + g) * kH + kq + (idx & 3) * 128 + 8 * t;
    };
    const int nst = (sg.tb - sg.ta) * 4;
    // the activations first (L2 hits that would otherwise queue behind the
    // weight misses), then the first two weight stages
    __syncthreads();  // the previous segment is done with pr_s, xs and red; ids_s is complete
    unit_pairs(p, e, start, ntok, ids_s, pr_s);
    __syncthreads();
    for (int j = 0; j < ntok; ++j)
      stage_split(p.xin + static_cast<int64_t>(pr_s[j] / kMaxTopK) * kH, kH, xs + j * kXStride,
                  xs + (kTokens + j) * kXStride);
    uint4 ra[8], rb[8];
    load_stage(ra, addr(0), kH);
    load_stage(rb, addr(1), kH);
    __syncthreads();
    auto xcol = [&](int idx) { return kq + (idx & 3) * 128; };
    auto done = [&](int idx, float (&acc)[4]) {
      if ((idx & 3) != 3) return;
      const int j = idx >> 2;
      float* rb_tile = red + (j & 1) * kWarps * 16 * kTokens;  // double-buffered by tile parity
      store_partial(rb_tile + warp * 16 * kTokens, acc, g, t);
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      __syncthreads();
      if (tid < 16 * kTokens) {
        const int n = tid % kTokens, r = tid / kTokens;
        if (n < ntok) {
          const float* rj = rb_tile + r * kTokens;
          constexpr int W = 16 * kTokens;  // one warp's partials
          const float gs = ((partial(rj, n, packed) + partial(rj + W, n, packed)) + partial(rj + 2 * W, n, packed)) +
                           partial(rj + 3 * W, n, packed);
          const float us = ((partial(rj + 4 * W, n, packed) + partial(rj + 5 * W, n, packed)) +
                            partial(rj + 6 * W, n, packed)) +
                           partial(rj + 7 * W, n, packed);
          p.hbuf[pair_row(p, pr_s[n]) * kI + (sg.ta + j) * 16 + r] = silu_mul(gs, us);
        }
      }
    };
    if (packed)
      stream_stages<true>(nst, kH, xs + (g < 4 ? g : g + 4) * kXStride + 8 * t, nullptr, addr, xcol, done, ra, rb);
    else
      stream_stages<false>(nst, kH, xs + g * kXStride + 8 * t, xs + (kTokens + g) * kXStride + 8 * t, addr, xcol,
                           done, ra, rb);
    // publish the segment's h rows: the down phase of any CTA waits for all
    // kGuTiles tiles of a unit before reading its h
    __threadfence();
    __syncthreads();
    if (tid == 0) atomicAdd(p.unit_done + sg.unit, static_cast<unsigned>(sg.tb - sg.ta));
  }
}

// Bounded wait (one thread) until all kGuTiles gate/up tiles of unit u are
// published.  Every CTA of the cooperative launch is resident and the
// gate/up phase never waits, so the count always completes; one that does
// not sets device error 8 after about a second, and the kernel finishes on
// whatever h holds instead of hanging.
__device__ __forceinline__ void wait_unit(const MoeParams& p, int u) {
  const volatile unsigned* c = p.unit_done + u;
  for (uint32_t i = 0; *c < static_cast<unsigned>(kGuTiles); ++i) {
    if (i >= (1u << 22)) {
      ria_set_error(p.err, RIA_DEVERR_MOE_WAIT);
      break;
    }
    __nanosleep(256);
  }
  __threadfence();
}

// down: tiles of 128 rows; warp w streams rows 16 w .. 16 w + 15 of each tile
// over all 512 columns (no cross-warp sum) and writes them per (token, slot)
// scaled by the slot's router weight (or the shared gate).  Each (token,
// tile) counts its k + 1 slots; the CTA that brings the count to k + 1
// writes that token's tile of the output: x + (routed slots in slot order +
// shared slot).
__device__ __forceinline__ void down_phase(const MoeParams& p, unsigned char* smem) {
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);  // rows 0-7 hi, 8-15 lo
  int* ids_s = reinterpret_cast<int*>(xs + 2 * kTokens * kHStride);  // [B * k]
  __shared__ int pr_s[kTokens];
  __shared__ float sc_s[kTokens];
  __shared__ int fin_s[kTokens * kDnTiles];
  __shared__ int n_fin;
  constexpr int kSt = kI / 128;  // stages per tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t total = static_cast<int64_t>(*p.n_units) * kDnTiles;
  const int64_t t_begin = total * blockIdx.x / gridDim.x, t_end = total * (blockIdx.x + 1) / gridDim.x;
  for (int i = tid; i < p.B * p.k; i += kThreads) ids_s[i] = p.ids[i];
  for (int64_t tt = t_begin; tt < t_end;) {
    const Segment sg = segment_at(tt, t_end, kDnTiles);
    tt += sg.tb - sg.ta;
    const int4 ui = p.units[sg.unit];
    const int e = ui.x, start = ui.y, ntok = ui.z;
    const bool shared = e == p.E, packed = ntok <= 4;
    const __nv_bfloat16* wd = shared ? p.sdp : p.ed + static_cast<int64_t>(e) * kH * kI;
    auto row_of = [&](int idx) { return (sg.ta + idx / kSt) * kDnRows + warp * 16; };
    auto addr = [&](int idx) {  // idx = (tile - ta) * kSt + stage
      return wd + static_cast<int64_t>(row_of(idx) + g) * kI + (idx % kSt) * 128 + 8 * t;
    };
    const int nst = (sg.tb - sg.ta) * kSt;
    __syncthreads();  // the previous segment is done with pr_s, sc_s, xs and fin_s; ids_s is complete
    if (tid == 0) n_fin = 0;
    unit_pairs(p, e, start, ntok, ids_s, pr_s);
    if (tid == 0) wait_unit(p, sg.unit);  // the unit's h rows, from the gate/up phase of any CTA
    __syncthreads();
    if (tid < ntok) {
      const int tok = pr_s[tid] / kMaxTopK, slot = pr_s[tid] % kMaxTopK;
      sc_s[tid] = slot < p.k ? p.wts[tok * p.k + slot] : p.sgate[tok];
    }
    for (int j = 0; j < ntok; ++j)
      stage_split(p.hbuf + pair_row(p, pr_s[j]) * kI, kI, xs + j * kHStride, xs + (kTokens + j) * kHStride);
    uint4 ra[8], rb[8];
    load_stage(ra, addr(0), kI);
    load_stage(rb, addr(1), kI);
    __syncthreads();
    auto xcol = [&](int idx) { return (idx % kSt) * 128; };
    // a finished tile straight from the accumulators: lane (g, t) holds rows
    // g, g + 8 of the warp's 16 and columns 2t, 2t + 1 (packed: columns n and
    // n + 4 are token n's hi and lo parts, held by lanes t and t + 2)
    auto done = [&](int idx, float (&acc)[4]) {
      if (idx % kSt != kSt - 1) return;
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, acc[j], 2);
        v[j] = packed ? acc[j] + other : acc[j];
        acc[j] = 0.f;
      }
      if (!packed || t < 2) {
        const int r0 = row_of(idx) + g;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int n = 2 * t + (j & 1);
          if (n < ntok) p.ybuf[pair_row(p, pr_s[n]) * kH + r0 + (j >> 1) * 8] = v[j] * sc_s[n];
        }
      }
    };
    if (packed)
      stream_stages<true>(nst, kI, xs + (g < 4 ? g : g + 4) * kHStride + 8 * t, nullptr, addr, xcol, done, ra, rb);
    else
      stream_stages<false>(nst, kI, xs + g * kHStride + 8 * t, xs + (kTokens + g) * kHStride + 8 * t, addr, xcol,
                           done, ra, rb);
    // hand-off: the last of a (token, tile)'s k + 1 slots to finish combines it
    __threadfence();
    __syncthreads();
    const int ntiles = sg.tb - sg.ta;
    if (tid < ntok * ntiles) {
      const int n = tid % ntok, tile = sg.ta + tid / ntok;
      unsigned* c = p.cnt_out + (pr_s[n] / kMaxTopK) * kDnTiles + tile;
      if (atomicAdd(c, 1u) == static_cast<unsigned>(p.k)) {
        *c = 0u;
        fin_s[atomicAdd(&n_fin, 1)] = (pr_s[n] / kMaxTopK) * kDnTiles + tile;
      }
    }
    __syncthreads();
    if (n_fin > 0) {
      __threadfence();
      for (int i = tid; i < n_fin * (kDnRows / 4); i += kThreads) {
        const int item = fin_s[i / (kDnRows / 4)];
        const int b = item / kDnTiles, d = (item % kDnTiles) * kDnRows + (i % (kDnRows / 4)) * 4;
        const float* y = p.ybuf + static_cast<int64_t>(b) * (p.k + 1) * kH + d;
        float4 routed = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < p.k; ++s) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(y + static_cast<int64_t>(s) * kH));
          routed.x += v.x;
          routed.y += v.y;
          routed.z += v.z;
          routed.w += v.w;
        }
        const float4 sh = __ldcg(reinterpret_cast<const float4*>(y + static_cast<int64_t>(p.k) * kH));
        const float4 x = *reinterpret_cast<const float4*>(p.residual + static_cast<int64_t>(b) * p.rs + d);
        *reinterpret_cast<float4*>(p.out + static_cast<int64_t>(b) * p.os + d) = make_float4(
            x.x + (routed.x + sh.x), x.y + (routed.y + sh.y), x.z + (routed.z + sh.z), x.w + (routed.w + sh.w));
      }
    }
  }
}

// The expert FFNs as one persistent launch (cooperative: every CTA is
// resident): each CTA streams its gate/up range, then its down range.  A
// down segment starts as soon as its unit's gate/up tiles are published, so
// the CTAs that finish gate/up early move on instead of waiting for the
// slowest one and a second launch.  The per-tile arithmetic and every sum
// order are those of two separate launches: results are unchanged.
__global__ void __launch_bounds__(kThreads, 2) moe_experts_kernel(const MoeParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  gate_up_phase(p, smem);
  __syncthreads();  // the gate/up phase is done with the shared memory
  down_phase(p, smem);
}

int64_t round_up(int64_t v) { return (v + 255) / 256 * 256; }

int64_t max_units(int64_t b, int64_t e, int64_t k) {
  return std::min(e, b * k) + (b * k + kTokens - 1) / kTokens + (b + kTokens - 1) / kTokens;
}

struct Layout {
  int64_t counters, xin, logits, hbuf, ybuf, units, unit_done, total;
};

// The counters come first (a workspace zeroed once stays valid: every call
// returns them to zero): cnt_group [kMaxGroups], cnt_plan, n_units, then
// cnt_out [B][kDnTiles].
Layout layout(int64_t b, int64_t e, int64_t k) {
  Layout l;
  int64_t off = 0;
  l.counters = off;
  off += round_up((kMaxGroups + 2 + b * kDnTiles) * 4);
  l.xin = off;
  off += round_up(b * kH * 4);
  l.logits = off;
  off += round_up(b * (e + 1) * 4);
  l.hbuf = off;
  off += round_up(b * (k + 1) * kI * 4);
  l.ybuf = off;
  off += round_up(b * (k + 1) * kH * 4);
  l.units = off;
  off += round_up(max_units(b, e, k) * 16);
  l.unit_done = off;
  off += round_up(max_units(b, e, k) * 4);
  l.total = off;
  return l;
}

}  // namespace

extern "C" int64_t ria_moe_workspace_bytes(int32_t batch, int32_t num_experts, int32_t top_k) {
  if (batch <= 0 || num_experts <= 0 || top_k <= 0) return 0;
  return layout(batch, num_experts, top_k).total;
}

extern "C" int ria_moe_decode(const float* residual, int64_t residual_stride, const void* post_norm_weight,
                              const void* router_weight, const void* shared_gate_weight, const void* experts_gate,
                              const void* experts_up, const void* experts_down, const void* shared_gate_proj,
                              const void* shared_up_proj, const void* shared_down_proj, float* out, int64_t out_stride,
                              int32_t* expert_ids, float* expert_weights, float* shared_gate, void* workspace,
                              int64_t workspace_bytes, int32_t batch, int32_t num_experts, int32_t top_k,
                              ria_stream_t stream) {
  if (batch < 0) return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: batch %d < 0", batch);
  if (batch == 0) return RIA_OK;
  if (num_experts < 1 || num_experts > kMaxExperts || top_k < 1 || top_k > kMaxTopK || top_k > num_experts)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: %d experts, top-%d (at most %d experts, top-%d)",
                     num_experts, top_k, kMaxExperts, kMaxTopK);
  if (static_cast<int64_t>(batch) * top_k > kMaxPairs)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: batch %d x top_k %d exceeds %d", batch, top_k, kMaxPairs);
  if (!residual || !post_norm_weight || !router_weight || !shared_gate_weight || !experts_gate || !experts_up ||
      !experts_down || !shared_gate_proj || !shared_up_proj || !shared_down_proj || !out || !expert_ids ||
      !expert_weights || !shared_gate || !workspace)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: null pointer argument");
  if (residual_stride < kH || out_stride < kH || residual_stride % 4 || out_stride % 4)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: row strides must be >= %d and multiples of 4", kH);
  const Layout l = layout(batch, num_experts, top_k);
  if (workspace_bytes < l.total)
    return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: workspace of %lld bytes, %lld needed",
                     static_cast<long long>(workspace_bytes), static_cast<long long>(l.total));
  const void* a16[] = {residual, out, router_weight, shared_gate_weight, experts_gate, experts_up, experts_down,
                       shared_gate_proj, shared_up_proj, shared_down_proj, workspace};
  for (const void* q : a16)
    if (!ria::aligned(q, 16))
      return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: activations, weights and workspace must be 16-byte aligned");
  if (!ria::aligned(post_norm_weight, 4))
    return ria::fail(RIA_ERR_INVALID, "ria_moe_decode: post_norm_weight must be 4-byte aligned");
  const int ids_bytes = batch * top_k * 4;
  const int gu_smem = 2 * kTokens * kXStride * 2 + 2 * kWarps * 16 * kTokens * 4 + ids_bytes;
  const int dn_smem = 2 * kTokens * kHStride * 2 + ids_bytes;
  const int ex_smem = std::max(gu_smem, dn_smem);
  static std::mutex attr_mu;  // the SMEM opt-ins are per-device function attributes
  static bool attr_set[64] = {false};
  static int resident_per_sm[64] = {0};  // experts-kernel CTAs resident per SM at the largest SMEM size
  int dev = -1;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> attr_lock(attr_mu);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    const int max_ids = kMaxPairs * 4;
    cudaError_t e = cudaFuncSetAttribute(moe_route_kernel<8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kLogitSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_route_kernel<8, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kLogitSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_route_kernel<kMaxExperts / 32, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kLogitSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_route_kernel<kMaxExperts / 32, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kLogitSmem);
    const int ex_max = std::max(2 * kTokens * kXStride * 2 + 2 * kWarps * 16 * kTokens * 4, 2 * kTokens * kHStride * 2) +
                       max_ids;
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_experts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ex_max);
    int per_sm = 0;
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_experts_kernel, kThreads, ex_max);
    if (e != cudaSuccess)
      return ria::fail(RIA_ERR_CUDA, "ria_moe_decode: kernel attributes: %s", cudaGetErrorString(e));
    if (per_sm < 1) return ria::fail(RIA_ERR_CUDA, "ria_moe_decode: the experts kernel does not fit an SM");
    if (dev >= 0 && dev < 64) {
      resident_per_sm[dev] = std::min(per_sm, 2);
      attr_set[dev] = true;
    }
  }
  const int per_sm = (dev >= 0 && dev < 64) ? resident_per_sm[dev] : 1;
  MoeParams p;
  p.residual = residual;
  p.rs = residual_stride;
  p.post_w = static_cast<const __nv_bfloat16*>(post_norm_weight);
  p.router_w = static_cast<const __nv_bfloat16*>(router_weight);
  p.shared_gate_w = static_cast<const __nv_bfloat16*>(shared_gate_weight);
  p.eg = static_cast<const __nv_bfloat16*>(experts_gate);
  p.eu = static_cast<const __nv_bfloat16*>(experts_up);
  p.ed = static_cast<const __nv_bfloat16*>(experts_down);
  p.sgp = static_cast<const __nv_bfloat16*>(shared_gate_proj);
  p.sup = static_cast<const __nv_bfloat16*>(shared_up_proj);
  p.sdp = static_cast<const __nv_bfloat16*>(shared_down_proj);
  p.out = out;
  p.os = out_stride;
  p.ids = expert_ids;
  p.wts = expert_weights;
  p.sgate = shared_gate;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  p.cnt_group = reinterpret_cast<unsigned*>(ws + l.counters);
  p.cnt_plan = p.cnt_group + kMaxGroups;
  p.n_units = reinterpret_cast<int*>(p.cnt_plan + 1);
  p.cnt_out = p.cnt_plan + 2;
  p.xin = reinterpret_cast<float*>(ws + l.xin);
  p.logits = reinterpret_cast<float*>(ws + l.logits);
  p.hbuf = reinterpret_cast<float*>(ws + l.hbuf);
  p.ybuf = reinterpret_cast<float*>(ws + l.ybuf);
  p.units = reinterpret_cast<int4*>(ws + l.units);
  p.unit_done = reinterpret_cast<unsigned*>(ws + l.unit_done);
  p.err = ria::device_error_word();
  p.B = batch;
  p.E = num_experts;
  p.k = top_k;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rows_per_warp = batch <= kTokens ? 1 : 2;
  const dim3 route_grid((num_experts + kWarps * rows_per_warp) / (kWarps * rows_per_warp),
                        (batch + kTokens - 1) / kTokens);
  if (num_experts <= 256) {
    if (rows_per_warp == 1)
      moe_route_kernel<8, 1><<<route_grid, kThreads, kLogitSmem, st>>>(p);
    else
      moe_route_kernel<8, 2><<<route_grid, kThreads, kLogitSmem, st>>>(p);
  } else {
    if (rows_per_warp == 1)
      moe_route_kernel<kMaxExperts / 32, 1><<<route_grid, kThreads, kLogitSmem, st>>>(p);
    else
      moe_route_kernel<kMaxExperts / 32, 2><<<route_grid, kThreads, kLogitSmem, st>>>(p);
  }
  int rc = ria::check_launch("ria_moe_decode (route and plan)");
  if (rc) return rc;
  const int64_t units = max_units(batch, num_experts, top_k);
  // one persistent cooperative grid: two CTAs per SM (all resident), or
  // fewer when there are fewer gate/up tiles
  const int resident = per_sm * ria::num_sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(resident, units * kGuTiles)));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(ex_smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, moe_experts_kernel, p);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_moe_decode (experts): %s", cudaGetErrorString(e));
  return ria::check_launch("ria_moe_decode (experts)");
}
