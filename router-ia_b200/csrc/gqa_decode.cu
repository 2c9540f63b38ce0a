// K3: paged, ragged, split-KV GQA decode with fused q/k RMSNorm, partial RoPE,
// KV append and the sigmoid output gate.
//
// Reference semantics (router-ia v2/src/router_ia/qwen36_attention_cache.py
// _full_stateful :285-324): q_gate = h W_q^T viewed (16, 512) -> q | gate per
// head; q, k per-head rmsnorm with (1+w) (qwen36_op_probe.py:55-67); RoPE on
// dims [0,64) with rotate-half inside that slice at position tokens_seen
// (:137-162); the new K/V token is appended (:334-373); query head h reads KV
// head h/8 (repeat_interleave(8)); softmax(q K^T * 256^-0.5) V in fp32; output
// times sigmoid(gate) (:317).
//
// B200 design
//   * KV lives in a paged bf16 pool [kv_head][pool_tokens][256]; a block is 64
//     tokens (32 KiB of K + 32 KiB of V per KV head).
//   * Grid (split, kv_head, sequence).  Each CTA streams its blocks through a
//     3-stage SMEM ring with 2-D TMA tensor copies (4 boxes of 64 tokens x 64
//     dims per tensor, 128-byte swizzle, no multicast), completion on mbarriers.
//   * The 8 query heads of a KV head are the N=8 side of mma.m16n8k16, so no
//     tensor-core work is padded: S^T = K Q^T (tokens x heads), then the
//     probabilities are transposed in registers (movmatrix) into the B operand
//     of O^T = V^T P^T (dims x heads).  Each of the 4 warps owns 16 tokens of a
//     block with its own online softmax; warps and splits are merged in
//     log-sum-exp form (splits by a second small kernel, no inter-CTA waits).
//   * The CTA whose split holds the new token writes it into the pool first and
//     publishes it to the TMA (async) proxy with fence.proxy.async.global.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

constexpr int kHq = 16;
constexpr int kHkv = 2;
constexpr int kGroup = 8;  // query heads per KV head
constexpr int kD = 256;
constexpr int kRope = 64;
constexpr int kBlock = 64;  // tokens per KV block
constexpr int kThreads = 128;
constexpr int kStages = 3;
constexpr uint32_t kBoxBytes = 64 * 128;               // 64 rows x 128 bytes
constexpr uint32_t kTensorBytes = 4 * kBoxBytes;       // one 64x256 bf16 tile
constexpr uint32_t kStageBytes = 2 * kTensorBytes;     // K + V
constexpr int kQRow = 264;                             // padded bf16 row of the q tile
constexpr float kLog2e = 1.4426950408889634f;

struct GqaParams {
  const __nv_bfloat16* q;
  int64_t q_stride;
  const __nv_bfloat16* k;
  int64_t k_stride;
  const __nv_bfloat16* v;
  int64_t v_stride;
  const float* q_norm_w;
  const float* k_norm_w;
  const float* inv_freq;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  int64_t pool_tokens;
  const int32_t* block_table;
  int32_t bt_stride;
  const int32_t* seq_lens;   // device [B], or null: use seq_len0 (batch 1)
  const int32_t* positions;  // device [B], or null: use position0 (batch 1)
  int32_t seq_len0;
  int32_t position0;
  __nv_bfloat16* out;
  int64_t out_stride;
  float* part_o;    // [B][max_splits][16][256]
  float* part_lse;  // [B][max_splits][16]
  int batch;
  int split_pages;
  int max_splits;
  int num_blocks;
  unsigned int* err;
};

// SMEM map (bytes); stage buffers first (1024-byte aligned for the swizzle atoms).
constexpr int kOffStage = 0;
constexpr int kOffQ = kOffStage + kStages * kStageBytes;   // [8][kQRow] bf16
constexpr int kOffKn = kOffQ + kGroup * kQRow * 2;         // [256] f32 staging for the appended k
constexpr int kOffRed = kOffKn + kD * 4;                   // [8] f32
constexpr int kOffML = kOffRed + 8 * 4;                    // [4 warps][2][8] f32
constexpr int kOffBar = kOffML + 4 * 2 * 8 * 4;
constexpr int kSmemBytes = kOffBar + kStages * 8;
// After the main loop the stage area is reused for the cross-warp merge:
// [4 warps][256 dims][8 heads] f32 = 32 KiB.

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

__global__ void __launch_bounds__(kThreads, 1)
    gqa_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const GqaParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  pdl_wait();
  __nv_bfloat16* qsm = reinterpret_cast<__nv_bfloat16*>(smem + kOffQ);
  float* kn = reinterpret_cast<float*>(smem + kOffKn);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* mls = reinterpret_cast<float*>(smem + kOffML);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;
  const int tig = lane & 3;

  const int L = p.seq_lens ? p.seq_lens[b] : p.seq_len0;
  const int total = L + 1;
  const int npages = cdiv(total, kBlock);
  const int nsplit = cdiv(npages, p.split_pages);
  // A split plan too small for this sequence (the launch covers
  // max_splits * split_pages pages): record it and leave the sequence alone --
  // no pool, partial or output write, since the trailing splits (the one that
  // appends the new token among them) were never launched.
  if (nsplit > static_cast<int>(gridDim.x)) {
    if (split == 0 && kvh == 0 && tid == 0) ria_set_error(p.err, RIA_DEVERR_SPLIT_PLAN);
    return;
  }
  const int p_begin = split * p.split_pages;
  if (p_begin >= npages) return;
  const int p_end = min(npages, p_begin + p.split_pages);
  const int my_pages = p_end - p_begin;
  const int pos = p.positions ? p.positions[b] : p.position0;
  const int32_t* bt = p.block_table + static_cast<int64_t>(b) * p.bt_stride;

  if (tid == 0) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }

  // ---- KV append (the split that holds token L), before any TMA read.
  if (p_end == npages) {
    const int lp = L / kBlock;
    int phys = (lp < p.bt_stride) ? bt[lp] : -1;
    const bool ok = phys >= 0 && phys < p.num_blocks;
    const __nv_bfloat16* krow = p.k + static_cast<int64_t>(b) * p.k_stride + kvh * kD;
    const float k0 = __bfloat162float(krow[tid]);
    const float k1 = __bfloat162float(krow[tid + 128]);
    float ss = warp_sum(k0 * k0 + k1 * k1);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    const float tot = red[0] + red[1] + red[2] + red[3];
    const float r = rsqrtf(tot * (1.0f / kD) + 1e-6f);
    kn[tid] = k0 * r * (1.0f + p.k_norm_w[tid]);
    kn[tid + 128] = k1 * r * (1.0f + p.k_norm_w[tid + 128]);
    __syncthreads();
    if (ok) {
      const int64_t row = static_cast<int64_t>(kvh) * p.pool_tokens + static_cast<int64_t>(phys) * kBlock + (L % kBlock);
      for (int d = tid; d < kD; d += kThreads) {
        float val = kn[d];
        if (d < kRope) {
          const int i = d & 31;
          float sn, cs;
          sincosf(static_cast<float>(pos) * p.inv_freq[i], &sn, &cs);
          val = (d < 32) ? (kn[d] * cs - kn[d + 32] * sn) : (kn[d] * cs + kn[d - 32] * sn);
        }
        p.k_pool[row * kD + d] = __float2bfloat16_rn(val);
        p.v_pool[row * kD + d] = p.v[static_cast<int64_t>(b) * p.v_stride + kvh * kD + d];
      }
      fence_proxy_async_global();
    } else if (tid == 0) {
      ria_set_error(p.err, RIA_DEVERR_BAD_BLOCK);
    }
  }
  __syncthreads();

  // ---- producer: TMA for the first stages
  auto issue = [&](int n) {
    const int s = n % kStages;
    const int lp = p_begin + n;
    int phys = (lp < p.bt_stride) ? bt[lp] : -1;
    if (phys < 0 || phys >= p.num_blocks) {
      ria_set_error(p.err, RIA_DEVERR_BAD_BLOCK);
      phys = 0;
    }
    const int32_t row = static_cast<int32_t>(kvh * p.pool_tokens + static_cast<int64_t>(phys) * kBlock);
    unsigned char* st = smem + kOffStage + s * kStageBytes;
    mbar_arrive_expect_tx(&full[s], kStageBytes);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      tma_load_2d(st + i * kBoxBytes, &tmK, i * 64, row, &full[s]);
      tma_load_2d(st + kTensorBytes + i * kBoxBytes, &tmV, i * 64, row, &full[s]);
    }
  };
  if (tid == 0) {
    for (int n = 0; n < kStages && n < my_pages; ++n) issue(n);
  }

  // ---- q: rmsnorm (1+w), RoPE, fold in 1/16, round to bf16 -> SMEM
  {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int hl = warp * 2 + hh;  // local head 0..7
      const int hq = kvh * kGroup + hl;
      const __nv_bfloat16* qrow = p.q + static_cast<int64_t>(b) * p.q_stride + hq * 2 * kD;
      float x[8];
      const uint4 raw = *reinterpret_cast<const uint4*>(qrow + lane * 8);
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(r2[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
      ss = warp_sum(ss);
      const float r = rsqrtf(ss * (1.0f / kD) + 1e-6f);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = x[i] * r * (1.0f + p.q_norm_w[lane * 8 + i]);
      // dims [0,64) live in lanes 0..7; the rotate-half partner of dim d is
      // d +- 32, i.e. lane +- 4.
      float partner[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float up = __shfl_down_sync(0xffffffffu, x[i], 4);
        const float dn = __shfl_up_sync(0xffffffffu, x[i], 4);
        partner[i] = (lane < 4) ? up : dn;
      }
      if (lane < 8) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int d = lane * 8 + i;
          float sn, cs;
          sincosf(static_cast<float>(pos) * p.inv_freq[d & 31], &sn, &cs);
          x[i] = (d < 32) ? (x[i] * cs - partner[i] * sn) : (x[i] * cs + partner[i] * sn);
        }
      }
      uint4 packed;
      packed.x = pack_bf16x2(x[0] * 0.0625f, x[1] * 0.0625f);
      packed.y = pack_bf16x2(x[2] * 0.0625f, x[3] * 0.0625f);
      packed.z = pack_bf16x2(x[4] * 0.0625f, x[5] * 0.0625f);
      packed.w = pack_bf16x2(x[6] * 0.0625f, x[7] * 0.0625f);
      *reinterpret_cast<uint4*>(qsm + hl * kQRow + lane * 8) = packed;
    }
  }
  __syncthreads();

  // B fragments of Q^T (dims x heads) for the 16 k-steps over 256 dims.
  uint32_t qf[16][2];
#pragma unroll
  for (int ks = 0; ks < 16; ++ks) {
    const __nv_bfloat16* base = qsm + g * kQRow + ks * 16 + 2 * tig;
    qf[ks][0] = *reinterpret_cast<const uint32_t*>(base);
    qf[ks][1] = *reinterpret_cast<const uint32_t*>(base + 8);
  }

  float o[16][4];
#pragma unroll
  for (int mt = 0; mt < 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  const uint32_t smem_base = smem_u32(smem);
  const int mi = lane >> 3;
  const int ri = lane & 7;

  for (int n = 0; n < my_pages; ++n) {
    const int s = n % kStages;
    const int lp = p_begin + n;
    const int nvalid = min(kBlock, total - lp * kBlock);
    mbar_wait_bounded(&full[s], (n / kStages) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_GQA);
    const uint32_t kbase = smem_base + kOffStage + s * kStageBytes;
    const uint32_t vbase = kbase + kTensorBytes;
    const int t0 = warp * 16;

    if (t0 < nvalid) {
      if (t0 + 16 > nvalid) {
        // Last, partial block: zero this warp's V rows past the end so that
        // 0-probability rows cannot inject non-finite values into P V.
        unsigned char* vst = smem + kOffStage + s * kStageBytes + kTensorBytes;
        for (int idx = lane; idx < 16 * 32; idx += 32) {
          const int rr = t0 + (idx >> 5);
          if (rr >= nvalid) {
            const int c = idx & 31;  // 32 chunks of 16 B per row across the 4 boxes
            *reinterpret_cast<uint4*>(vst + (c >> 3) * kBoxBytes + swz128(rr, c & 7)) = make_uint4(0, 0, 0, 0);
          }
        }
        __syncwarp();
      }

      // S^T[16 tokens x 8 heads] = K[tokens, 256] Q^T
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 16; ++ks) {
        const int row = t0 + ri + ((mi & 1) << 3);
        const int ch = (ks & 3) * 2 + (mi >> 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kbase + (ks >> 2) * kBoxBytes + swz128(row, ch), a0, a1, a2, a3);
        mma_bf16_16816(sc, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
      }
      const bool v0 = (t0 + g) < nvalid;
      const bool v1 = (t0 + g + 8) < nvalid;
      const float s00 = v0 ? sc[0] * kLog2e : -INFINITY;  // token g,   head 2tig
      const float s01 = v0 ? sc[1] * kLog2e : -INFINITY;  // token g,   head 2tig+1
      const float s10 = v1 ? sc[2] * kLog2e : -INFINITY;  // token g+8, head 2tig
      const float s11 = v1 ? sc[3] * kLog2e : -INFINITY;  // token g+8, head 2tig+1
      float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;
      const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
      const float sc0 = exp2f(m0 - mu0), sc1 = exp2f(m1 - mu1);
      const float p00 = exp2f(s00 - mu0), p01 = exp2f(s01 - mu1);
      const float p10 = exp2f(s10 - mu0), p11 = exp2f(s11 - mu1);
      l0 = l0 * sc0 + p00 + p10;
      l1 = l1 * sc1 + p01 + p11;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 16; ++mt) {
        o[mt][0] *= sc0;
        o[mt][1] *= sc1;
        o[mt][2] *= sc0;
        o[mt][3] *= sc1;
      }
      // P^T (tokens x heads) in C layout -> B operand (tokens x heads, k-major per head)
      const uint32_t b0 = movm_t(pack_bf16x2(p00, p01));
      const uint32_t b1 = movm_t(pack_bf16x2(p10, p11));
      // O^T[256 dims x 8 heads] += V^T[dims, 16 tokens] P^T
#pragma unroll
      for (int mt = 0; mt < 16; ++mt) {
        const int row = t0 + ri + ((mi >> 1) << 3);
        const int ch = (mt & 3) * 2 + (mi & 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vbase + (mt >> 2) * kBoxBytes + swz128(row, ch), a0, a1, a2, a3);
        mma_bf16_16816(o[mt], a0, a1, a2, a3, b0, b1);
      }
    }
    __syncthreads();  // stage s consumed by all warps
    if (tid == 0 && n + kStages < my_pages) issue(n + kStages);
  }

  // ---- merge the 4 warps (log-sum-exp), then write the split result
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  float* om = reinterpret_cast<float*>(smem + kOffStage);  // [4][256][8]
  if (g == 0) {
    mls[(warp * 2 + 0) * 8 + 2 * tig] = m0;
    mls[(warp * 2 + 0) * 8 + 2 * tig + 1] = m1;
    mls[(warp * 2 + 1) * 8 + 2 * tig] = l0;
    mls[(warp * 2 + 1) * 8 + 2 * tig + 1] = l1;
  }
#pragma unroll
  for (int mt = 0; mt < 16; ++mt) {
    float* w = om + warp * (kD * kGroup);
    w[(mt * 16 + g) * kGroup + 2 * tig] = o[mt][0];
    w[(mt * 16 + g) * kGroup + 2 * tig + 1] = o[mt][1];
    w[(mt * 16 + g + 8) * kGroup + 2 * tig] = o[mt][2];
    w[(mt * 16 + g + 8) * kGroup + 2 * tig + 1] = o[mt][3];
  }
  __syncthreads();
  {
    const int hl = tid >> 4;         // local head 0..7
    const int d0 = (tid & 15) * 16;  // 16 dims per thread
    float mw[4], lw[4], M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      mw[w] = mls[(w * 2 + 0) * 8 + hl];
      lw[w] = mls[(w * 2 + 1) * 8 + hl];
      M = fmaxf(M, mw[w]);
    }
    float ew[4], Ls = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      ew[w] = (mw[w] == -INFINITY) ? 0.f : exp2f(mw[w] - M);
      Ls += ew[w] * lw[w];
    }
    const float inv = 1.0f / Ls;
    const int hq = kvh * kGroup + hl;
    if (nsplit == 1) {
      const __nv_bfloat16* gate = p.q + static_cast<int64_t>(b) * p.q_stride + hq * 2 * kD + kD;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(b) * p.out_stride + hq * kD;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int d = d0 + i;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) acc += ew[w] * om[w * (kD * kGroup) + d * kGroup + hl];
        const float gz = __bfloat162float(gate[d]);
        dst[d] = __float2bfloat16_rn(acc * inv * (1.0f / (1.0f + expf(-gz))));
      }
    } else {
      float* dst = p.part_o + ((static_cast<int64_t>(b) * p.max_splits + split) * kHq + hq) * kD;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int d = d0 + i;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) acc += ew[w] * om[w * (kD * kGroup) + d * kGroup + hl];
        dst[d] = acc * inv;
      }
      if ((tid & 15) == 0)
        p.part_lse[(static_cast<int64_t>(b) * p.max_splits + split) * kHq + hq] = M + log2f(Ls);
    }
  }
}

// Second pass: merge split partials in log-sum-exp form, apply the gate.
__global__ void __launch_bounds__(kD) gqa_combine_kernel(const GqaParams p) {
  pdl_wait();
  const int b = blockIdx.x;
  const int hq = blockIdx.y;
  const int d = threadIdx.x;
  const int npages = cdiv((p.seq_lens ? p.seq_lens[b] : p.seq_len0) + 1, kBlock);
  // A sequence needing more splits than were launched was skipped by the
  // attention kernel (device error RIA_DEVERR_SPLIT_PLAN): leave its output
  // alone and never read partials beyond the workspace.
  const int nsplit = cdiv(npages, p.split_pages);
  if (nsplit <= 1 || nsplit > p.max_splits) return;
  const float* lse = p.part_lse + static_cast<int64_t>(b) * p.max_splits * kHq + hq;
  // Per-split weights 2^(lse - max) once, in chunks of kD splits in shared
  // memory; then each thread sums its dimension over the chunk with 16
  // partial loads in flight.
  __shared__ float wts[kD];
  __shared__ float red[kD / 32];
  float M = -INFINITY;
  for (int s = d; s < nsplit; s += kD) M = fmaxf(M, lse[s * kHq]);
  M = warp_max(M);
  if ((d & 31) == 0) red[d >> 5] = M;
  __syncthreads();
  M = red[0];
#pragma unroll
  for (int i = 1; i < kD / 32; ++i) M = fmaxf(M, red[i]);
  float acc = 0.f, wsum = 0.f;
  const float* po = p.part_o + (static_cast<int64_t>(b) * p.max_splits * kHq + hq) * kD + d;
  for (int c0 = 0; c0 < nsplit; c0 += kD) {
    const int cn = min(kD, nsplit - c0);
    __syncthreads();  // the previous chunk's weights are consumed
    if (d < cn) wts[d] = exp2f(lse[(c0 + d) * kHq] - M);
    __syncthreads();
    constexpr int kInFlight = 16;
    for (int s0 = 0; s0 < cn; s0 += kInFlight) {
      float o[kInFlight];
#pragma unroll
      for (int i = 0; i < kInFlight; ++i)
        o[i] = s0 + i < cn ? po[static_cast<int64_t>(c0 + s0 + i) * kHq * kD] : 0.f;
#pragma unroll
      for (int i = 0; i < kInFlight; ++i) {
        const float w = s0 + i < cn ? wts[s0 + i] : 0.f;
        wsum += w;
        acc = fmaf(w, o[i], acc);
      }
    }
  }
  const float gz = __bfloat162float(p.q[static_cast<int64_t>(b) * p.q_stride + hq * 2 * kD + kD + d]);
  p.out[static_cast<int64_t>(b) * p.out_stride + hq * kD + d] =
      __float2bfloat16_rn((acc / wsum) * (1.0f / (1.0f + expf(-gz))));
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D map over a pool [rows, 256] bf16 with 64x64 boxes and 128-byte swizzle.
int make_pool_map(CUtensorMap* m, void* base, int64_t rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return ria::fail(RIA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD) * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ria::fail(RIA_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return RIA_OK;
}

}  // namespace

extern "C" int64_t ria_gqa_decode_workspace_bytes(int32_t batch, int32_t max_splits) {
  if (batch <= 0 || max_splits <= 0) return 0;
  return static_cast<int64_t>(batch) * max_splits * kHq * (kD + 1) * 4;
}

extern "C" int32_t ria_gqa_decode_split_pages(int64_t total_blocks, int32_t num_kv_heads) {
  const int64_t work = std::max<int64_t>(1, total_blocks * std::max(1, num_kv_heads));
  const int64_t target_ctas = static_cast<int64_t>(ria::num_sms()) * 4;
  int64_t sp = (work + target_ctas - 1) / target_ctas;
  // at least two pages per split once there are a few: a CTA's prologue (q
  // norm and RoPE, the append) then covers two TMA loads (batch 1 at 4096
  // tokens: 26.7 us per layer step against 28.7 with one page per split)
  const int64_t floor_pages = total_blocks >= 4 ? 2 : 1;
  return static_cast<int32_t>(std::max<int64_t>(floor_pages, sp));
}

extern "C" int ria_gqa_decode_paged(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                                    int64_t v_stride, const float* q_norm_weight, const float* k_norm_weight,
                                    const float* inv_freq, void* k_pool, void* v_pool, int64_t pool_tokens,
                                    const int32_t* block_table, int32_t block_table_stride, const int32_t* seq_lens,
                                    const int32_t* positions, int32_t seq_len0, int32_t position0, void* out,
                                    int64_t out_stride, void* workspace,
                                    int64_t workspace_bytes, int32_t batch, int32_t split_pages, int32_t max_splits,
                                    ria_stream_t stream) {
  if (batch < 0) return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: batch=%d < 0", batch);
  if (batch == 0) return RIA_OK;
  if (!q || !k || !v || !q_norm_weight || !k_norm_weight || !inv_freq || !k_pool || !v_pool || !block_table ||
      !out)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: null pointer argument");
  if ((!seq_lens || !positions) && batch != 1)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: seq_lens/positions may be null only for batch 1");
  if ((!seq_lens && seq_len0 < 0) || (!positions && position0 < 0))
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: negative seq_len0/position0");
  if (!seq_lens && (seq_len0 / kBlock) >= block_table_stride)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: seq_len0=%d needs a block past the table (stride %d)",
                     seq_len0, block_table_stride);
  if (split_pages < 1 || max_splits < 1)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: split_pages=%d max_splits=%d must be >= 1", split_pages,
                     max_splits);
  if (!seq_lens && (seq_len0 / kBlock) + 1 > static_cast<int64_t>(split_pages) * max_splits)
    return ria::fail(RIA_ERR_INVALID,
                     "ria_gqa_decode_paged: seq_len0=%d needs %d pages, more than split_pages=%d x max_splits=%d",
                     seq_len0, seq_len0 / kBlock + 1, split_pages, max_splits);
  if (max_splits > 65535)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: max_splits=%d exceeds the grid limit", max_splits);
  if (pool_tokens <= 0 || pool_tokens % kBlock != 0)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: pool_tokens=%lld must be a positive multiple of 64",
                     static_cast<long long>(pool_tokens));
  if (static_cast<int64_t>(kHkv) * pool_tokens > INT32_MAX)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: pool too large for 32-bit TMA coordinates");
  if (block_table_stride < 1)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: block_table_stride must be >= 1");
  if (q_stride < kHq * 2 * kD || k_stride < kHkv * kD || v_stride < kHkv * kD || out_stride < kHq * kD)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: row stride smaller than the row width");
  if (!ria::aligned(k_pool, 16) || !ria::aligned(v_pool, 16) || !ria::aligned(q, 16) || (q_stride % 8) != 0)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: q rows and KV pools must be 16-byte aligned");
  const int64_t need = ria_gqa_decode_workspace_bytes(batch, max_splits);
  if (max_splits > 1 && (!workspace || workspace_bytes < need || !ria::aligned(workspace, 16)))
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged: workspace needs %lld bytes (16-byte aligned), got %lld",
                     static_cast<long long>(need), static_cast<long long>(workspace_bytes));

  CUtensorMap tmK, tmV;
  int rc = make_pool_map(&tmK, k_pool, kHkv * pool_tokens);
  if (rc) return rc;
  rc = make_pool_map(&tmV, v_pool, kHkv * pool_tokens);
  if (rc) return rc;

  GqaParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride = q_stride;
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.k_stride = k_stride;
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.v_stride = v_stride;
  p.q_norm_w = q_norm_weight;
  p.k_norm_w = k_norm_weight;
  p.inv_freq = inv_freq;
  p.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  p.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  p.pool_tokens = pool_tokens;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.seq_lens = seq_lens;
  p.positions = positions;
  p.seq_len0 = seq_len0;
  p.position0 = position0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.part_o = static_cast<float*>(workspace);
  p.part_lse = workspace ? static_cast<float*>(workspace) + static_cast<int64_t>(batch) * max_splits * kHq * kD
                         : nullptr;
  p.batch = batch;
  p.split_pages = split_pages;
  p.max_splits = max_splits;
  p.num_blocks = static_cast<int>(pool_tokens / kBlock);
  p.err = ria::device_error_word();

  {  // the SMEM opt-in is a per-device function attribute
    static std::mutex mu;
    static bool attr_set[64] = {false};
    int dev = -1;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      cudaError_t e =
          cudaFuncSetAttribute(gqa_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess)
        return ria::fail(RIA_ERR_CUDA, "ria_gqa_decode_paged: smem attribute: %s", cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(max_splits, kHkv, batch);
  cudaError_t le = ria::launch_pdl(gqa_decode_kernel, grid, dim3(kThreads), kSmemBytes, st, tmK, tmV, p);
  if (le != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_gqa_decode_paged: %s", cudaGetErrorString(le));
  rc = ria::check_launch("ria_gqa_decode_paged");
  if (rc) return rc;
  if (max_splits > 1) {
    le = ria::launch_pdl(gqa_combine_kernel, dim3(batch, kHq), dim3(kD), 0, st, p);
    if (le != cudaSuccess)
      return ria::fail(RIA_ERR_CUDA, "ria_gqa_decode_paged (combine): %s", cudaGetErrorString(le));
    rc = ria::check_launch("ria_gqa_decode_paged (combine)");
  }
  return rc;
}

// ---------------------------------------------------------------- allocation-free variant
//
// Some callers cannot allocate device memory at the point where they decode:
// host runtimes that own all GPU memory through their own pools, processes
// held to a hard VRAM budget, and plugin interfaces that hand a kernel its
// inputs and outputs but no workspace -- a cudaMalloc there fails, breaks the
// budget or bypasses the host's accounting.  For them
// ria_gqa_decode_paged_static keeps the split partials in a fixed array that
// is part of the library image instead of a caller workspace.  Its first call
// on a device looks the array's address up (cudaGetSymbolAddress with that
// device current); make that first call before any stream capture.
//
// The array lives for as long as the library is loaded, on every GPU that
// loads it (RIA_GQA_STATIC_SCRATCH_BYTES each).  All calls on a device share
// it, so two calls whose kernels overlap on the GPU (different streams without
// ordering between them) race on it; calls ordered on one stream are safe.
// Nothing in it has to start at zero: every partial the combine pass reads was
// written by the attention pass of the same call.  The array keeps the last
// call's partials.
namespace {

static __device__ __align__(256) unsigned char g_gqa_static_scratch[RIA_GQA_STATIC_SCRATCH_BYTES];

// Device address of g_gqa_static_scratch on the current device.  Host code
// cannot use the symbol itself (it names a host-side shadow, not device
// memory), so the address is looked up once per device, with that device
// current, and cached.
void* gqa_static_scratch(int* rc_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *rc_out = ria::fail(RIA_ERR_CUDA, "ria_gqa_decode_paged_static: cudaGetDevice: %s", cudaGetErrorString(e));
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *rc_out = ria::fail(RIA_ERR_UNSUPPORTED, "ria_gqa_decode_paged_static: device %d out of range", dev);
    return nullptr;
  }
  static std::mutex mu;
  static void* cache[64] = {nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_gqa_static_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      *rc_out = ria::fail(RIA_ERR_CUDA, "ria_gqa_decode_paged_static: cudaGetSymbolAddress: %s",
                          cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = ptr;
  }
  *rc_out = RIA_OK;
  return cache[dev];
}

}  // namespace

extern "C" int ria_gqa_decode_paged_static(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                                           const void* v, int64_t v_stride, const float* q_norm_weight,
                                           const float* k_norm_weight, const float* inv_freq, void* k_pool,
                                           void* v_pool, int64_t pool_tokens, const int32_t* block_table,
                                           int32_t block_table_stride, const int32_t* seq_lens,
                                           const int32_t* positions, int32_t seq_len0, int32_t position0, void* out,
                                           int64_t out_stride, int32_t batch, int32_t split_pages, int32_t max_splits,
                                           ria_stream_t stream) {
  if (batch < 0 || max_splits < 1)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_decode_paged_static: batch=%d max_splits=%d", batch, max_splits);
  if (batch == 0) return RIA_OK;
  const int64_t need = ria_gqa_decode_workspace_bytes(batch, max_splits);
  if (max_splits > 1 && need > static_cast<int64_t>(RIA_GQA_STATIC_SCRATCH_BYTES))
    return ria::fail(RIA_ERR_INVALID,
                     "ria_gqa_decode_paged_static: batch=%d x max_splits=%d needs %lld bytes of split scratch, more "
                     "than the fixed %lld-byte array; use a larger split_pages or ria_gqa_decode_paged with a workspace",
                     batch, max_splits, static_cast<long long>(need),
                     static_cast<long long>(RIA_GQA_STATIC_SCRATCH_BYTES));
  int rc = RIA_OK;
  void* scratch = gqa_static_scratch(&rc);
  if (!scratch) return rc;
  return ria_gqa_decode_paged(q, q_stride, k, k_stride, v, v_stride, q_norm_weight, k_norm_weight, inv_freq, k_pool,
                              v_pool, pool_tokens, block_table, block_table_stride, seq_lens, positions, seq_len0,
                              position0, out, out_stride, scratch, RIA_GQA_STATIC_SCRATCH_BYTES, batch, split_pages,
                              max_splits, stream);
}
