// K4: GQA prefill -- a prompt of T tokens through one full-attention layer:
// per-head q/k RMSNorm (1+w), partial RoPE, KV append into the paged cache,
// causal attention over the cached prefix plus the new tokens, sigmoid gate.
//
// Reference semantics: router-ia runs a prompt token by token through
// _full_stateful (qwen36_attention_cache.py:285-324); token t attends to every
// cached token and to the new tokens 0..t (its own key included), with q/k
// norms, RoPE at position tokens_seen, softmax(q K^T / 16) V and the gate
// exactly as in the decode step.  This kernel computes all T tokens at once.
//
// B200 design
//   * gqa_prefill_prep: one CTA per token; q/k RMSNorm + RoPE (in-kernel
//     sincosf, host inverse frequencies), the normalised q (x 1/16) to a bf16
//     workspace, K and V appended to the 64-token pages.
//   * gqa_prefill_attn: one CTA per (128-token query tile, query head,
//     sequence), key tiles of 128 (two pages).  Q is loaded once by TMA and
//     moved into TMEM as bf16 pairs; a producer warp streams K tiles (double
//     buffered) and V tiles straight from the pool pages by TMA (no
//     multicast) and issues the tcgen05 UMMAs: S = Q K^T (M = 128 tokens,
//     N = 128 keys, K = 256, A from TMEM) and O += P V (M = 128, N = 256,
//     K = 128, P and V in 128-byte-swizzled SMEM), fp32 accumulators in TMEM.
//     Four softmax warps own one query row each (= TMEM lane); they release
//     S_j as soon as it is in registers, so S_{j+1} runs on the tensor core
//     while they form P_j.  O is rescaled in TMEM only when a row's running
//     maximum grows by more than 8 (log2 units).  The gated bf16 output
//     leaves by TMA tensor store.
#include <mutex>

#include "ria_capi_internal.h"
#include "ria_common.cuh"
#include "tcgen05.cuh"

namespace {

constexpr int kHq = 16;
constexpr int kHkv = 2;
constexpr int kGroup = 8;
constexpr int kD = 256;
constexpr int kRope = 64;
constexpr int kBlock = 64;
constexpr int kTile = 128;  // query tokens per CTA
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleSlack = 8.0f;  // log2 units

struct PrepParams {
  const __nv_bfloat16* q;  // [B][T][16*512], per head: q 256 | gate 256
  int64_t qs_b, qs_t;
  const __nv_bfloat16* k;  // [B][T][2*256]
  int64_t ks_b, ks_t;
  const __nv_bfloat16* v;
  int64_t vs_b, vs_t;
  const float* q_norm_w;
  const float* k_norm_w;
  const float* inv_freq;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  int64_t pool_tokens;
  const int32_t* block_table;
  int32_t bt_stride;
  const int32_t* seq_lens;   // cached tokens before the prompt
  const int32_t* positions;  // absolute position of prompt token 0
  __nv_bfloat16* qbuf;       // [B][T][16][256]
  int T;
  int num_blocks;
  unsigned int* err;
};

// RMSNorm (1+w) and partial RoPE of one 256-dim head row held as 8 values per
// lane (lane l has dims 8l..8l+7); dims [0,64) rotate-half inside the slice.
// w1: this lane's 8 values of (1 + norm weight), held in registers.
// cs_row / sn_row: cos / sin of position x inv_freq[f], f = 0..31, in SMEM.
__device__ __forceinline__ void norm_rope_8(float (&x)[8], const float (&w1)[8], const float* cs_row,
                                            const float* sn_row, int lane) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss * (1.0f / kD) + 1e-6f);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = x[i] * r * w1[i];
  float partner[8];  // lanes 0-3 <-> 4-7: dims d and d + 32 of the rotated slice
#pragma unroll
  for (int i = 0; i < 8; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, x[i], 4);
  if (lane < kRope / 8) {
    const int f0 = (lane * 8) & (kRope / 2 - 1);
    float cs[8], sn[8];
    *reinterpret_cast<float4*>(cs) = *reinterpret_cast<const float4*>(cs_row + f0);
    *reinterpret_cast<float4*>(cs + 4) = *reinterpret_cast<const float4*>(cs_row + f0 + 4);
    *reinterpret_cast<float4*>(sn) = *reinterpret_cast<const float4*>(sn_row + f0);
    *reinterpret_cast<float4*>(sn + 4) = *reinterpret_cast<const float4*>(sn_row + f0 + 4);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      x[i] = (lane < kRope / 16) ? (x[i] * cs[i] - partner[i] * sn[i]) : (x[i] * cs[i] + partner[i] * sn[i]);
  }
}

__device__ __forceinline__ void load8(const __nv_bfloat16* src, float (&x)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(r2[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&x)[8], float s) {
  uint4 u;
  u.x = pack_bf16x2(x[0] * s, x[1] * s);
  u.y = pack_bf16x2(x[2] * s, x[3] * s);
  u.z = pack_bf16x2(x[4] * s, x[5] * s);
  u.w = pack_bf16x2(x[6] * s, x[7] * s);
  return u;
}

constexpr int kPrepTokens = 8;  // prompt tokens per prep CTA

// One CTA per 8 prompt tokens: the tokens' RoPE angles once (cos / sin of
// position x inv_freq, 32 frequencies each), then 8 x (16 q heads + 2 k
// heads) RMSNorm + RoPE rows and 8 x 2 V rows spread over the 8 warps.
__global__ void __launch_bounds__(256, 4) gqa_prefill_prep_kernel(const PrepParams p) {
  __shared__ __align__(16) float cs_tab[kPrepTokens][kRope / 2];
  __shared__ __align__(16) float sn_tab[kPrepTokens][kRope / 2];
  const int tb = blockIdx.x * kPrepTokens, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L0 = p.seq_lens[b];
  {
    const int tt = threadIdx.x >> 5, f = threadIdx.x & 31;  // 8 tokens x 32 frequencies
    float sn, cs;
    sincosf(static_cast<float>(p.positions[b] + tb + tt) * p.inv_freq[f], &sn, &cs);
    cs_tab[tt][f] = cs;
    sn_tab[tt][f] = sn;
  }
  __syncthreads();
  float wq1[8];  // (1 + q norm weight) for this lane's 8 dims (the k weight is read per k row: 2 of 20 rows)
#pragma unroll
  for (int i = 0; i < 8; ++i) wq1[i] = 1.0f + p.q_norm_w[lane * 8 + i];
  constexpr int kTasks = kHq + 2 * kHkv;  // per token: q heads, k heads, v heads
  constexpr int kPerWarp = kPrepTokens * kTasks / 8;
  constexpr int kInFlight = 4;  // rows a warp loads before it works on them
  static_assert(kPerWarp % kInFlight == 0, "task batches");
  for (int i0 = 0; i0 < kPerWarp; i0 += kInFlight) {
    uint4 raw[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {  // warp task i: token i / kTasks, row kind i % kTasks
      const int task = warp + 8 * (i0 + u);
      const int tt = task / kTasks, kind = task % kTasks;
      const int t = tb + tt;
      raw[u] = make_uint4(0u, 0u, 0u, 0u);
      if (t >= p.T) continue;
      const __nv_bfloat16* src =
          kind < kHq ? p.q + static_cast<int64_t>(b) * p.qs_b + static_cast<int64_t>(t) * p.qs_t + kind * 2 * kD
          : kind < kHq + kHkv
              ? p.k + static_cast<int64_t>(b) * p.ks_b + static_cast<int64_t>(t) * p.ks_t + (kind - kHq) * kD
              : p.v + static_cast<int64_t>(b) * p.vs_b + static_cast<int64_t>(t) * p.vs_t + (kind - kHq - kHkv) * kD;
      raw[u] = *reinterpret_cast<const uint4*>(src + lane * 8);
    }
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int task = warp + 8 * (i0 + u);
      const int tt = task / kTasks, kind = task % kTasks;
      const int t = tb + tt;
      if (t >= p.T) continue;  // warp-uniform
      float x[8];
      {
        const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&raw[u]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(r2[i]);
          x[2 * i] = f.x;
          x[2 * i + 1] = f.y;
        }
      }
      if (kind < kHq) {
        norm_rope_8(x, wq1, cs_tab[tt], sn_tab[tt], lane);
        *reinterpret_cast<uint4*>(p.qbuf + ((static_cast<int64_t>(b) * p.T + t) * kHq + kind) * kD + lane * 8) =
            pack8(x, 0.0625f);
        continue;
      }
      const int cidx = L0 + t;
      const int lp = cidx / kBlock;
      const int phys = (lp < p.bt_stride) ? p.block_table[static_cast<int64_t>(b) * p.bt_stride + lp] : -1;
      if (phys < 0 || phys >= p.num_blocks) {
        if (lane == 0) ria_set_error(p.err, RIA_DEVERR_BAD_BLOCK);
        continue;
      }
      const int kvh = (kind - kHq) & 1;
      const int64_t row =
          static_cast<int64_t>(kvh) * p.pool_tokens + static_cast<int64_t>(phys) * kBlock + (cidx % kBlock);
      if (kind < kHq + kHkv) {
        float wk1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) wk1[i] = 1.0f + p.k_norm_w[lane * 8 + i];
        norm_rope_8(x, wk1, cs_tab[tt], sn_tab[tt], lane);
        *reinterpret_cast<uint4*>(p.k_pool + row * kD + lane * 8) = pack8(x, 1.0f);
      } else {
        *reinterpret_cast<uint4*>(p.v_pool + row * kD + lane * 8) = raw[u];
      }
    }
  }
}

struct AttnParams {
  const __nv_bfloat16* gate;  // q projection + 256: head h gate at [h*512, h*512+256)
  int64_t gs_b, gs_t;
  const int32_t* block_table;
  int32_t bt_stride;
  const int32_t* seq_lens;
  int T;
  int64_t pool_tokens;
  int num_blocks;
  unsigned int* err;
};

// SMEM map: two K tiles and one V tile of 128 keys (two pages), each four
// 16 KiB [128 rows][64 bf16] column chunks; P [128 rows][128 keys] bf16 as two
// chunks.  Q arrives once by TMA into the second K tile and moves to TMEM.
constexpr uint32_t kBox = 64 * 128;       // one [64 rows][64 bf16] TMA box
constexpr uint32_t kChunk = 2 * kBox;     // [128 rows][64 bf16]
constexpr int kKeys = 2 * kBlock;         // keys per tile
constexpr uint32_t kOffK = 0;             // two tiles
constexpr uint32_t kOffV = 8 * kChunk;
constexpr uint32_t kOffP = 12 * kChunk;
constexpr uint32_t kOffBar = 14 * kChunk;  // tma_q, tma_k[2], tma_v, bar_s, bar_pv, s_free, p_ready
constexpr uint32_t kOffTslot = kOffBar + 64;
constexpr uint32_t kOffXchg = kOffTslot + 16;  // [tile parity][half][row] partial maxima
constexpr uint32_t kAttnSmem = kOffXchg + 2 * 2 * 128 * 4;
static_assert(kAttnSmem <= 227 * 1024, "attention SMEM");
// TMEM columns: O fp32 [128][256], S fp32 [128][128], Q bf16 pairs [128][128]
constexpr uint32_t kTmO = 0, kTmS = 256, kTmQ = 384;
constexpr int kAttnThreads = 320;  // warps 0-7: softmax half-rows; 8: S issue + K loads; 9: PV issue + V loads
constexpr int kSoftmax = 256;
constexpr uint32_t kBarRows = 1;  // named barrier of the softmax threads

__device__ __forceinline__ float ex2(float x) {  // 2^x (PTX ex2.approx, flush-to-zero)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    gqa_prefill_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                            const AttnParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int qt = gridDim.x - 1 - blockIdx.x;  // the longest (last) query tiles start first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / kGroup;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = qt * kTile;
  if (t0 >= p.T) return;
  uint64_t* tma_q = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* tma_k = tma_q + 1;  // [2]
  uint64_t* tma_v = tma_q + 3;
  uint64_t* bar_s = tma_q + 4;
  uint64_t* bar_pv = tma_q + 5;
  uint64_t* s_free = tma_q + 6;
  uint64_t* p_ready = tma_q + 7;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kOffTslot);
  const uint32_t sbase = smem_u32(smem);
  const int L0 = p.seq_lens[b];
  const int last_q = min(t0 + kTile - 1, p.T - 1);
  const int last_key = L0 + last_q;  // the last key any row of this tile sees
  const int ntiles = last_key / kKeys + 1;
  const int32_t* bt = p.block_table + static_cast<int64_t>(b) * p.bt_stride;

  // Loads one K or V tile: the pages of keys [128 j, 128 j + 128) that some
  // row of this query tile can see (pages past that are not loaded).
  auto load_tile = [&](int j, uint32_t off, const CUtensorMap* map, uint64_t* bar) {
    int npages = 0;
    int32_t rows[2];
    for (int pg = 0; pg < 2; ++pg) {
      const int lp = 2 * j + pg;
      if (lp * kBlock > last_key) break;
      int phys = (lp < p.bt_stride) ? bt[lp] : -1;
      if (phys < 0 || phys >= p.num_blocks) {
        ria_set_error(p.err, RIA_DEVERR_BAD_BLOCK);
        phys = 0;
      }
      rows[npages++] = static_cast<int32_t>(kvh * p.pool_tokens + static_cast<int64_t>(phys) * kBlock);
    }
    mbar_arrive_expect_tx(bar, npages * 4 * kBox);
    for (int pg = 0; pg < npages; ++pg)
#pragma unroll
      for (int c = 0; c < 4; ++c) tma_load_2d(smem + off + c * kChunk + pg * kBox, map, c * 64, rows[pg], bar);
  };

  if (tid == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmO);
    for (int i = 0; i < 6; ++i) mbar_init(&tma_q[i], 1);
    mbar_init(s_free, kSoftmax);
    mbar_init(p_ready, kSoftmax);
    mbar_fence_init();
    // Q (once, into the second K tile), K_0, V_0
    mbar_arrive_expect_tx(tma_q, 4 * kChunk);
#pragma unroll
    for (int c = 0; c < 4; ++c) tma_load_3d(smem + kOffK + 4 * kChunk + c * kChunk, &tmQ, h * kD + c * 64, t0, b, tma_q);
    load_tile(0, kOffK, &tmK, &tma_k[0]);
    load_tile(0, kOffV, &tmV, tma_v);
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *tslot;
  if (warp < 8) {  // Q rows -> TMEM (bf16 pairs, the A operand of S = Q K^T); half-row each
    mbar_wait_bounded(tma_q, 0, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
    const uint32_t my_lane = tm + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int row = tid & 127;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * (tid >> 7) + cc;
      const unsigned char* q = smem + kOffK + 4 * kChunk + c * kChunk;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[16];
#pragma unroll
        for (int piece = 0; piece < 4; ++piece) {
          const uint4 u = *reinterpret_cast<const uint4*>(q + tc::sw128_off(row, 32 * half + 8 * piece));
          pk[4 * piece] = u.x;
          pk[4 * piece + 1] = u.y;
          pk[4 * piece + 2] = u.z;
          pk[4 * piece + 3] = u.w;
        }
        tc::st16(my_lane + kTmQ + 32 * c + 16 * half, pk);
      }
    }
    tc::wait_st();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (warp == 8) {
    // ============================================================ S = Q K^T issue, K tiles
    if (lane == 0) {
      auto issue_s = [&](int j) {
        tc::fence_after_sync();
        const uint32_t id = tc::idesc_bf16(128, kKeys, false, false);
        const uint32_t kt = sbase + kOffK + (j & 1) * 4 * kChunk;
#pragma unroll
        for (int ks = 0; ks < 16; ++ks)
          tc::mma_bf16_ts(tm + kTmS, tm + kTmQ + ks * 8,
                          tc::sdesc_sw128(kt + (ks >> 2) * kChunk + (ks & 3) * 32, 16, 1024), id, ks > 0);
        tc::commit(bar_s);
      };
      if (ntiles > 1) load_tile(1, kOffK + 4 * kChunk, &tmK, &tma_k[1]);
      mbar_wait_bounded(&tma_k[0], 0, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      issue_s(0);
      for (int j = 0; j < ntiles; ++j) {
        // the softmax rows hold S_j (so S_j is complete): S_{j+1} may overwrite
        // it, and K_j's buffer takes K_{j+2}
        mbar_wait_bounded(s_free, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
        if (j + 1 < ntiles) {
          mbar_wait_bounded(&tma_k[(j + 1) & 1], ((j + 1) >> 1) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
          issue_s(j + 1);
        }
        if (j + 2 < ntiles) load_tile(j + 2, kOffK + (j & 1) * 4 * kChunk, &tmK, &tma_k[j & 1]);
      }
    }
  } else if (warp == 9) {
    // ============================================================ O += P V issue, V tiles
    for (int j = 0; j < ntiles; ++j) {
      // V_j has landed: zero its rows past the sequence end (the pool holds
      // anything there; 0-probability keys must not bring non-finite values)
      mbar_wait_bounded(tma_v, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      {
        const int first_bad = L0 + p.T - j * kKeys;
        if (first_bad < kKeys) {
          const int r0 = max(first_bad, 0);
          for (int idx = lane; idx < (kKeys - r0) * 32; idx += 32) {
            const int row = r0 + (idx >> 5), ch = idx & 31;
            *reinterpret_cast<uint4*>(smem + kOffV + (ch >> 3) * kChunk + row * 128 + (ch & 7) * 16) =
                make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
      }
      __syncwarp();
      if (lane == 0) {
        // P_j is staged: O += P_j V_j; once it has read V_j, bring in V_{j+1}
        mbar_wait_bounded(p_ready, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
        tc::fence_after_sync();
        const uint32_t id = tc::idesc_bf16(128, 256, false, true);
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks)
          tc::mma_bf16(tm + kTmO, tc::sdesc_sw128(sbase + kOffP + (ks >> 2) * kChunk + (ks & 3) * 32, 16, 1024),
                       tc::sdesc_sw128(sbase + kOffV + ks * 2048, kChunk, 1024), id, j > 0 || ks > 0);
        tc::commit(bar_pv);
        mbar_wait_bounded(bar_pv, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
        if (j + 1 < ntiles) load_tile(j + 1, kOffV, &tmV, tma_v);
      }
      __syncwarp();
    }
  } else {
    // ============================================================ softmax rows
    // Two threads per query row (= TMEM lane): half hf takes keys
    // [64 hf, 64 hf + 64) of every tile and O columns [128 hf, 128 hf + 128).
    const int r = tid & 127;
    const int hf = tid >> 7;
    const uint32_t my_lane = tm + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int qidx = L0 + t0 + r;  // cache index of this query token
    const bool row_ok = (t0 + r) < p.T;
    float* xchg = reinterpret_cast<float*>(smem + kOffXchg);  // [2][2][128]
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < ntiles; ++j) {
      mbar_wait_bounded(bar_s, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      tc::fence_after_sync();
      float s[64];
      tc::ld32(my_lane + kTmS + 64 * hf, s);
      tc::ld32(my_lane + kTmS + 64 * hf + 32, s + 32);
      tc::wait_ld();
      tc::fence_before_sync();
      mbar_arrive(s_free);
      // causal / length mask only where the tile reaches past some row's last key
      const bool full = (j + 1) * kKeys - 1 <= L0 + t0 && t0 + kTile <= p.T;
      if (!full) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const bool ok = row_ok && (j * kKeys + 64 * hf + c) <= qidx;
          s[c] = ok ? s[c] : -INFINITY;
        }
      }
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], s[c]);
      const float mine = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * kLog2e;
      float* xt = xchg + (j & 1) * 256;  // a slot is rewritten only after the next tile's barrier
      xt[hf * 128 + r] = mine;
      named_bar_sync(kBarRows, kSoftmax);
      const float mx = fmaxf(mine, xt[(hf ^ 1) * 128 + r]);
      float f = 1.f;  // rescale of O and l when the running maximum moves
      const bool rescale = mx > m_used + kRescaleSlack;
      const bool scale_o = rescale && m_used != -INFINITY;  // O holds earlier tiles
      if (rescale) {
        f = (m_used == -INFINITY) ? 0.f : ex2(m_used - mx);
        l *= f;
        m_used = mx;
      }
      const float mu = (m_used == -INFINITY) ? 0.f : m_used;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        s[c] = ex2(fmaf(s[c], kLog2e, -mu));
        l4[c & 3] += s[c];
      }
      l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      // P_{j-1} V_{j-1} must be done: it reads the P staging tile, and writes O
      if (j > 0) {
        mbar_wait_bounded(bar_pv, (j - 1) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
        tc::fence_after_sync();
        if (scale_o) {
          for (int c0 = 128 * hf; c0 < 128 * hf + 128; c0 += 32) {
            float o[32];
            tc::ld32(my_lane + kTmO + c0, o);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= f;
            tc::st32(my_lane + kTmO + c0, o);
          }
          tc::wait_st();
        }
      }
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        uint4 u;
        u.x = pack_bf16x2(s[c], s[c + 1]);
        u.y = pack_bf16x2(s[c + 2], s[c + 3]);
        u.z = pack_bf16x2(s[c + 4], s[c + 5]);
        u.w = pack_bf16x2(s[c + 6], s[c + 7]);
        *reinterpret_cast<uint4*>(smem + kOffP + hf * kChunk + tc::sw128_off(r, c)) = u;
      }
      fence_proxy_async_smem();
      tc::fence_before_sync();
      mbar_arrive(p_ready);
    }
    mbar_wait_bounded(bar_pv, (ntiles - 1) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
    tc::fence_after_sync();
    // the two halves' sums (both use the same running maximum)
    named_bar_sync(kBarRows, kSoftmax);  // every max exchange of the loop is read
    xchg[hf * 128 + r] = l;
    named_bar_sync(kBarRows, kSoftmax);
    l += xchg[(hf ^ 1) * 128 + r];

    // ---- epilogue: O / l * sigmoid(gate) -> bf16 staging over the first K tile -> TMA store
    unsigned char* stg = smem + kOffK;  // 4 chunks of [128 rows][128 B]
    const float inv = (l > 0.f) ? 1.0f / l : 0.f;
    const __nv_bfloat16* grow =
        p.gate + static_cast<int64_t>(b) * p.gs_b + static_cast<int64_t>(row_ok ? t0 + r : t0) * p.gs_t + h * 2 * kD;
    for (int c0 = 128 * hf; c0 < 128 * hf + 128; c0 += 32) {
      float o[32];
      tc::ld32(my_lane + kTmO + c0, o);
      tc::wait_ld();
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        float gz[8];
        load8(grow + c0 + i, gz);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[i + e] = o[i + e] * inv * (1.0f / (1.0f + expf(-gz[e])));
        uint4 u;
        u.x = pack_bf16x2(o[i], o[i + 1]);
        u.y = pack_bf16x2(o[i + 2], o[i + 3]);
        u.z = pack_bf16x2(o[i + 4], o[i + 5]);
        u.w = pack_bf16x2(o[i + 6], o[i + 7]);
        const int col = c0 + i;
        *reinterpret_cast<uint4*>(stg + (col >> 6) * kChunk + tc::sw128_off(r, col & 63)) = u;
      }
    }
    fence_proxy_async_smem();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) tma_store_3d(&tmO, smem + kOffK + i * kChunk, h * kD + i * 64, t0, b);
    bulk_commit_group();
    bulk_wait_all0();
  }
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 512);
}

int pool_map(CUtensorMap* m, void* base, int64_t pool_tokens) {
  const uint64_t dims[2] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(kHkv * pool_tokens)};
  const uint64_t strides[1] = {static_cast<uint64_t>(kD) * 2};
  const uint32_t box[2] = {64, 64};
  return ria::encode_bf16_sw128_map(m, base, 2, dims, strides, box);
}

}  // namespace

extern "C" int64_t ria_gqa_prefill_workspace_bytes(int32_t batch, int32_t seq_len) {
  if (batch <= 0 || seq_len <= 0) return 0;
  return static_cast<int64_t>(batch) * seq_len * kHq * kD * 2;
}

extern "C" int ria_gqa_prefill(const void* q, int64_t q_stride_b, int64_t q_stride_t, const void* k, int64_t k_stride_b,
                               int64_t k_stride_t, const void* v, int64_t v_stride_b, int64_t v_stride_t,
                               const float* q_norm_weight, const float* k_norm_weight, const float* inv_freq,
                               void* k_pool, void* v_pool, int64_t pool_tokens, const int32_t* block_table,
                               int32_t block_table_stride, const int32_t* seq_lens, const int32_t* positions,
                               void* out, int64_t out_stride_b, int64_t out_stride_t, void* workspace,
                               int64_t workspace_bytes, int32_t batch, int32_t seq_len, ria_stream_t stream) {
  if (batch < 0 || seq_len < 0) return ria::fail(RIA_ERR_INVALID, "ria_gqa_prefill: negative size");
  if (batch == 0 || seq_len == 0) return RIA_OK;
  if (!q || !k || !v || !q_norm_weight || !k_norm_weight || !inv_freq || !k_pool || !v_pool || !block_table ||
      !seq_lens || !positions || !out || !workspace)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_prefill: null pointer argument");
  if (batch > 65535) return ria::fail(RIA_ERR_INVALID, "ria_gqa_prefill: batch too large");
  if (pool_tokens <= 0 || pool_tokens % kBlock || kHkv * pool_tokens > INT32_MAX)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_prefill: bad pool_tokens");
  if (q_stride_t < kHq * 2 * kD || k_stride_t < kHkv * kD || v_stride_t < kHkv * kD || out_stride_t < kHq * kD)
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_prefill: token stride smaller than the row width");
  if (!ria::aligned(q, 16) || !ria::aligned(k, 16) || !ria::aligned(v, 16) || !ria::aligned(out, 16) ||
      !ria::aligned(k_pool, 16) || !ria::aligned(v_pool, 16) || !ria::aligned(workspace, 16) || (q_stride_t % 8) ||
      (k_stride_t % 8) || (v_stride_t % 8) || (out_stride_t % 8) || (q_stride_b % 8) || (k_stride_b % 8) ||
      (v_stride_b % 8) || (out_stride_b % 8))
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_prefill: tensors must be 16-byte aligned with 16-byte strides");
  if (workspace_bytes < ria_gqa_prefill_workspace_bytes(batch, seq_len))
    return ria::fail(RIA_ERR_INVALID, "ria_gqa_prefill: workspace needs %lld bytes",
                     static_cast<long long>(ria_gqa_prefill_workspace_bytes(batch, seq_len)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int* err = ria::device_error_word();

  PrepParams pp;
  pp.q = static_cast<const __nv_bfloat16*>(q);
  pp.qs_b = q_stride_b;
  pp.qs_t = q_stride_t;
  pp.k = static_cast<const __nv_bfloat16*>(k);
  pp.ks_b = k_stride_b;
  pp.ks_t = k_stride_t;
  pp.v = static_cast<const __nv_bfloat16*>(v);
  pp.vs_b = v_stride_b;
  pp.vs_t = v_stride_t;
  pp.q_norm_w = q_norm_weight;
  pp.k_norm_w = k_norm_weight;
  pp.inv_freq = inv_freq;
  pp.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  pp.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  pp.pool_tokens = pool_tokens;
  pp.block_table = block_table;
  pp.bt_stride = block_table_stride;
  pp.seq_lens = seq_lens;
  pp.positions = positions;
  pp.qbuf = static_cast<__nv_bfloat16*>(workspace);
  pp.T = seq_len;
  pp.num_blocks = static_cast<int>(pool_tokens / kBlock);
  pp.err = err;
  gqa_prefill_prep_kernel<<<dim3((seq_len + kPrepTokens - 1) / kPrepTokens, batch), 256, 0, st>>>(pp);
  int rc = ria::check_launch("ria_gqa_prefill (prep)");
  if (rc) return rc;

  CUtensorMap tmQ, tmK, tmV, tmO;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHq * kD), static_cast<uint64_t>(seq_len),
                              static_cast<uint64_t>(batch)};
    const uint64_t sq[2] = {static_cast<uint64_t>(kHq * kD) * 2, static_cast<uint64_t>(seq_len) * kHq * kD * 2};
    const uint64_t so[2] = {static_cast<uint64_t>(out_stride_t) * 2, static_cast<uint64_t>(out_stride_b) * 2};
    const uint32_t box[3] = {64, kTile, 1};
    rc = ria::encode_bf16_sw128_map(&tmQ, workspace, 3, dims, sq, box);
    if (rc) return rc;
    rc = ria::encode_bf16_sw128_map(&tmO, out, 3, dims, so, box);
    if (rc) return rc;
  }
  rc = pool_map(&tmK, k_pool, pool_tokens);
  if (rc) return rc;
  rc = pool_map(&tmV, v_pool, pool_tokens);
  if (rc) return rc;

  AttnParams ap;
  ap.gate = static_cast<const __nv_bfloat16*>(q) + kD;
  ap.gs_b = q_stride_b;
  ap.gs_t = q_stride_t;
  ap.block_table = block_table;
  ap.bt_stride = block_table_stride;
  ap.seq_lens = seq_lens;
  ap.T = seq_len;
  ap.pool_tokens = pool_tokens;
  ap.num_blocks = static_cast<int>(pool_tokens / kBlock);
  ap.err = err;
  cudaError_t e = cudaFuncSetAttribute(gqa_prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_gqa_prefill: smem attribute: %s", cudaGetErrorString(e));
  dim3 grid((seq_len + kTile - 1) / kTile, kHq, batch);
  gqa_prefill_attn_kernel<<<grid, kAttnThreads, kAttnSmem, st>>>(tmQ, tmK, tmV, tmO, ap);
  return ria::check_launch("ria_gqa_prefill (attention)");
}
