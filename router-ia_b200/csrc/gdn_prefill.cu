// K2: chunked Gated DeltaNet prefill (chunk 64, WY/UT form) on tcgen05.
//
// Reference semantics: the chunked gated delta rule router-ia runs for a
// prompt through transformers' torch_chunk_gated_delta_rule
// (qwen36_linear_attention_hf.py:91-100, use_qk_l2norm_in_kernel=True), equal
// to the token-by-token rule of qwen36_attention_cache.py:256-266.  Per chunk
// of C = 64 tokens with in-chunk log-decay cumsum gamma, L2-normalised k and
// q (q also scaled by 128^-0.5):
//   A  = strict_lower(beta_i k_i.k_j exp(gamma_i - gamma_j)),  T = (I + A)^-1
//   W  = T diag(beta e^gamma) K,  U = T diag(beta) V
//   V' = U - W S,   O = diag(e^gamma) Q S + (Q K^T o causal decay) V'
//   S <- e^gamma_C S + K^T diag(e^(gamma_C - gamma)) V'
//
// B200 design: one CTA per (sequence, value head), two warpgroups.
//   * Warpgroup 0 (prep) works one chunk ahead on everything that does not
//     depend on the state: TMA loads of the Q/K/V tiles (3-D tensor maps, no
//     multicast), gates and norms, G = [Q;K] K^T on the tensor cores, the
//     causal score tile P and the 64x64 unit-lower-triangular inverse (CUDA
//     cores, 16x16 blocks), W^T = K^T TW^T and U^T = V^T TU^T on the tensor
//     cores, and the row-scaled Q (the output scale e^gamma s_q 128^-0.5 moved
//     onto Q so both output products share one accumulator).
//   * Warpgroup 1 (recurrence) owns the fp32 state S^T in TMEM:
//     X = S^T W^T and O = S^T Qr^T, V'^T = U^T - X, O += V'^T P^T and
//     S^T = e^gamma_C S^T + V's^T K, then the bf16 output.
//   The two hand chunks over through a two-slot SMEM ring: prep arrives on a
//   "full" mbarrier when a slot is ready, and the recurrence refills a slot
//   with the TMA of chunk c + 2 as soon as its MMAs have read it.  Every product is an M = 128 UMMA
//   (tcgen05.mma cta_group::1, bf16 operands in 128-byte-swizzled SMEM, fp32
//   accumulation in TMEM); all waits are bounded.
#include "ria_capi_internal.h"
#include "ria_common.cuh"
#include "tcgen05.cuh"

namespace {

constexpr int kC = 64;
constexpr int kDK = 128;
constexpr int kDV = 128;
constexpr int kThreads = 256;
constexpr float kQScale = 0.08838834764831845f;  // 128 ** -0.5
constexpr float kLog2e = 1.4426950408889634f;

// SMEM map (bytes).  A chunk slot holds X = [Q dims 0-63 | K dims 0-63],
// Y = [Q dims 64-127 | K dims 64-127], V (then U^T bf16 [128 dv][64]), W^T
// bf16 [128 dk][64] (MN-major B), P bf16 [64][64], and the chunk scalars.
// Every box is 64 rows x 128 bytes, 128-byte swizzled.
constexpr uint32_t kBox = 8192;
constexpr uint32_t kSlX = 0, kSlY = 2 * kBox, kSlV = 4 * kBox, kSlWT = 6 * kBox, kSlP = 8 * kBox;
constexpr uint32_t kSlScal = 9 * kBox;  // eC, colscale[64]
constexpr uint32_t kSlotBytes = 9 * kBox + 1024;
constexpr uint32_t kOffSlot0 = 0;
constexpr int kLd = 65;                            // padded fp32 row of A and T (bank-conflict free)
constexpr uint32_t kOffAT = 2 * kSlotBytes;        // fp32 A [64][kLd], then TW | TU bf16
constexpr uint32_t kOffTf = kOffAT + 64 * kLd * 4; // fp32 T [64][kLd]
constexpr uint32_t kOffST = kOffAT + 33 * 1024;    // bf16 S^T [128][128] (two boxes); later VN | VNS, O staging
constexpr uint32_t kOffMisc = kOffST + 4 * kBox;
constexpr uint32_t kOffGraw = kOffMisc;
constexpr uint32_t kOffGam = kOffMisc + 256;  // gamma * log2(e)
constexpr uint32_t kOffBet = kOffMisc + 512;
constexpr uint32_t kOffSq = kOffMisc + 768;
constexpr uint32_t kOffSk = kOffMisc + 1024;
constexpr uint32_t kOffZ = kOffMisc + 1280;  // inversion scratch, 4 warps x 16 x 17 f32
constexpr uint32_t kOffBar = kOffZ + 4 * 16 * 17 * 4;   // tma[2] full[2] (unused x2) mma_p mma_r
constexpr uint32_t kOffTslot = kOffBar + 64;
constexpr uint32_t kSmemBytes = kOffTslot + 16;

// TMEM columns
constexpr uint32_t kTmS = 0, kTmX = 128, kTmO = 192, kTmG = 256, kTmWT = 320, kTmUT = 384;

constexpr uint32_t kBarPrep = 1, kBarRec = 2;

struct PrefillParams {
  const float* g;  // [B][T][Hv] log decay
  const float* beta;
  int64_t gs_b, gs_t;
  const float* init_state;  // [B][Hv][128 k][128 v] or null (zeros)
  float* final_state;
  __nv_bfloat16* out;  // [B][T][Hv][128]
  int64_t os_b, os_t;
  int T;
  int Hv;
  int group;  // value heads per key head
  unsigned int* err;
};

template <int N>
__device__ __forceinline__ void store_row_bf16(unsigned char* tile, int row, int col0, const float* v) {
#pragma unroll
  for (int i = 0; i < N; i += 8) {
    uint4 pk;
    pk.x = pack_bf16x2(v[i], v[i + 1]);
    pk.y = pack_bf16x2(v[i + 2], v[i + 3]);
    pk.z = pack_bf16x2(v[i + 4], v[i + 5]);
    pk.w = pack_bf16x2(v[i + 6], v[i + 7]);
    *reinterpret_cast<uint4*>(tile + tc::sw128_off(row, col0 + i)) = pk;
  }
}

template <int N>
__device__ __forceinline__ void load_row_bf16(const unsigned char* tile, int row, int col0, float* v) {
#pragma unroll
  for (int i = 0; i < N; i += 8) {
    const uint4 pk = *reinterpret_cast<const uint4*>(tile + tc::sw128_off(row, col0 + i));
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h2[e]);
      v[i + 2 * e] = f.x;
      v[i + 2 * e + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float sumsq_row(const unsigned char* box0, const unsigned char* box1, int r) {
  float ss = 0.f;
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    const unsigned char* rowp = (part ? box1 : box0) + r * 128;
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      // visit the row's 16-byte chunks in swizzled order so that the 32 lanes
      // (32 different rows) spread over all banks
      const uint4 u = *reinterpret_cast<const uint4*>(rowp + ((ch ^ (r & 7)) << 4));
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  }
  return ss;
}

// Multiply the 128 bf16 of row r (two boxes) by s in place.
__device__ __forceinline__ void scale_row_bf16(unsigned char* box, int r, float s) {
  unsigned char* rowp = box + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int ch = c ^ (r & 7);  // bank-spread visiting order
    uint4 u = *reinterpret_cast<uint4*>(rowp + ch * 16);
    __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h2[e]);
      h2[e] = __floats2bfloat162_rn(f.x * s, f.y * s);
    }
    *reinterpret_cast<uint4*>(rowp + ch * 16) = u;
  }
}

// D (+)= A(16x8 tf32, row) * B(8x8 tf32, col), fp32 accumulate.
__device__ __forceinline__ void mma_tf32_1688(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// d[2][4] += X[16x16] * Y[16x16] for one warp; X, Y fp32 in SMEM with row
// strides ldx, ldy.  C layout: d[nt][0..3] = rows g, g, g+8, g+8 and columns
// 8nt + 2tig, +1, 2tig, +1.
__device__ __forceinline__ void warp_mma16(float (&d)[2][4], const float* X, int ldx, const float* Y, int ldy,
                                           int lane) {
  const int g = lane >> 2, tg = lane & 3;
#pragma unroll
  for (int kk = 0; kk < 16; kk += 8) {
    const uint32_t a0 = to_tf32(X[g * ldx + kk + tg]);
    const uint32_t a1 = to_tf32(X[(g + 8) * ldx + kk + tg]);
    const uint32_t a2 = to_tf32(X[g * ldx + kk + tg + 4]);
    const uint32_t a3 = to_tf32(X[(g + 8) * ldx + kk + tg + 4]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint32_t b0 = to_tf32(Y[(kk + tg) * ldy + 8 * nt + g]);
      const uint32_t b1 = to_tf32(Y[(kk + tg + 4) * ldy + 8 * nt + g]);
      mma_tf32_1688(d[nt], a0, a1, a2, a3, b0, b1);
    }
  }
}

// T = (I + A)^-1 for strictly-lower A (fp32 [64][kLd]) by the 128 prep
// threads.  The four 16x16 diagonal blocks are inverted by substitution
// (threads 0-63, one column each; threads 64-127 meanwhile scale Q rows and
// clear the upper blocks).  Off-diagonal blocks follow in order of distance d
// from the diagonal, one warp per block, on the tensor cores (tf32 in, fp32
// accumulate): T_ij = -T_ii (sum_{m=j}^{i-1} A_im T_mj).
template <class Side>
__device__ void invert_unit_lower64(const float* A, float* T, float* Z, int tid, Side&& side_work) {
  if (tid < 64) {
    const int d = tid >> 4, jj = tid & 15, j = 16 * d + jj;
    float col[16];
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < ii; ++m)
        if (m >= jj) acc = fmaf(A[(16 * d + ii) * kLd + 16 * d + m], col[m], acc);
      col[ii] = (ii < jj) ? 0.f : (ii == jj ? 1.f : -acc);
    }
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) T[(16 * d + ii) * kLd + j] = col[ii];
  } else {
    for (int e = tid - 64; e < 6 * 256; e += 64) {
      const int blk = e >> 8;
      const int bi = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
      const int bj = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
      T[(16 * bi + ((e >> 4) & 15)) * kLd + 16 * bj + (e & 15)] = 0.f;
    }
    side_work(tid - 64);
  }
  named_bar_sync(kBarPrep, 128);
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tg = lane & 3;
  float* zw = Z + warp * 16 * 17;  // warp-private 16x16 (row stride 17)
#pragma unroll
  for (int dist = 1; dist < 4; ++dist) {
    if (warp < 4 - dist) {
      const int bi = warp + dist, bj = warp;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int mb = bj; mb < bi; ++mb)
        warp_mma16(acc, A + (16 * bi) * kLd + 16 * mb, kLd, T + (16 * mb) * kLd + 16 * bj, kLd, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        zw[g * 17 + 8 * nt + 2 * tg] = acc[nt][0];
        zw[g * 17 + 8 * nt + 2 * tg + 1] = acc[nt][1];
        zw[(g + 8) * 17 + 8 * nt + 2 * tg] = acc[nt][2];
        zw[(g + 8) * 17 + 8 * nt + 2 * tg + 1] = acc[nt][3];
      }
      __syncwarp();
      float tt[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      warp_mma16(tt, T + (16 * bi) * kLd + 16 * bi, kLd, zw, 17, lane);
      float* out = T + (16 * bi) * kLd + 16 * bj;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        out[g * kLd + 8 * nt + 2 * tg] = -tt[nt][0];
        out[g * kLd + 8 * nt + 2 * tg + 1] = -tt[nt][1];
        out[(g + 8) * kLd + 8 * nt + 2 * tg] = -tt[nt][2];
        out[(g + 8) * kLd + 8 * nt + 2 * tg + 1] = -tt[nt][3];
      }
      __syncwarp();
    }
    named_bar_sync(kBarPrep, 128);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gdn_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                       const PrefillParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int hk = h / p.group;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int wg = tid >> 7;    // 0: prep, 1: recurrence
  const int lt = tid & 127;   // thread index inside the warpgroup == TMEM lane
  uint64_t* tma_bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full_bar = tma_bar + 2;
  uint64_t* mma_p = tma_bar + 6;
  uint64_t* mma_r = tma_bar + 7;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kOffTslot);
  const uint32_t sbase = smem_u32(smem);
  const int nchunks = (p.T + kC - 1) / kC;

  if (tid == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmO);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tma_bar[i], 1);
      mbar_init(&full_bar[i], 128);
    }
    mbar_init(mma_p, 1);
    mbar_init(mma_r, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t my_lane = tm + lane_base;

  // TMA of chunk c's Q/K/V tiles into slot c & 1 (issued by one thread).
  auto issue_chunk = [&](int c) {
    const int s = c & 1;
    unsigned char* slot = smem + kOffSlot0 + s * kSlotBytes;
    mbar_arrive_expect_tx(&tma_bar[s], 6 * kBox);
    tma_load_3d(slot + kSlX, &tmQ, hk * kDK, c * kC, b, &tma_bar[s]);
    tma_load_3d(slot + kSlX + kBox, &tmK, hk * kDK, c * kC, b, &tma_bar[s]);
    tma_load_3d(slot + kSlY, &tmQ, hk * kDK + 64, c * kC, b, &tma_bar[s]);
    tma_load_3d(slot + kSlY + kBox, &tmK, hk * kDK + 64, c * kC, b, &tma_bar[s]);
    tma_load_3d(slot + kSlV, &tmV, h * kDV, c * kC, b, &tma_bar[s]);
    tma_load_3d(slot + kSlV + kBox, &tmV, h * kDV + 64, c * kC, b, &tma_bar[s]);
  };
  auto load_gates = [&](int c, float& gv, float& bv) {
    const int t = c * kC + lt;
    const bool ok = t < p.T;
    const int64_t gi = static_cast<int64_t>(b) * p.gs_b + static_cast<int64_t>(t) * p.gs_t + h;
    gv = ok ? p.g[gi] : 0.f;
    bv = ok ? p.beta[gi] : 0.f;
  };

  if (wg == 0) {
    // =================================================================== prep
    float* graw = reinterpret_cast<float*>(smem + kOffGraw);
    float* gam = reinterpret_cast<float*>(smem + kOffGam);
    float* bet = reinterpret_cast<float*>(smem + kOffBet);
    float* sq = reinterpret_cast<float*>(smem + kOffSq);
    float* sk = reinterpret_cast<float*>(smem + kOffSk);
    uint32_t ph_p = 0;
    if (lt == 0) {
      issue_chunk(0);
      if (nchunks > 1) issue_chunk(1);
    }
    float g_next = 0.f, b_next = 0.f;
    if (lt < kC) load_gates(0, g_next, b_next);
    for (int c = 0; c < nchunks; ++c) {
      const int s = c & 1;
      unsigned char* slot = smem + kOffSlot0 + s * kSlotBytes;
      const uint32_t aslot = sbase + kOffSlot0 + s * kSlotBytes;
      float gscan = 0.f;
      if (lt < kC) {
        // inclusive scan of the chunk's log decays inside each of the two warps
        gscan = g_next;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float up = __shfl_up_sync(0xffffffffu, gscan, o);
          if ((lt & 31) >= o) gscan += up;
        }
        if (lt == 31) graw[0] = gscan;  // warp 0 total
        bet[lt] = b_next;
        if (c + 1 < nchunks) load_gates(c + 1, g_next, b_next);  // in flight during this chunk
      }
      mbar_wait_bounded(&tma_bar[s], (c >> 1) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      // ---- G = [Q;K] K^T (raw q, k) runs while the gates and norms are formed
      if (lt == 0) {
        tc::fence_after_sync();
        const uint32_t id = tc::idesc_bf16(128, 64, false, false);
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t kb = aslot + (ks < 4 ? kSlX : kSlY) + (ks & 3) * 32;
          tc::mma_bf16(tm + kTmG, tc::sdesc_sw128(kb, 16, 1024), tc::sdesc_sw128(kb + kBox, 16, 1024), id, ks > 0);
        }
        tc::commit(mma_p);
      }
      named_bar_sync(kBarPrep, 128);
      if (lt < kC) gam[lt] = (lt >= 32 ? gscan + graw[0] : gscan) * kLog2e;
      {
        const int r = lt & 63;
        const uint32_t off = lt >= 64 ? kBox : 0;
        const float rn = rsqrtf(sumsq_row(slot + kSlX + off, slot + kSlY + off, r) + 1e-6f);
        if (lt < 64) sq[r] = rn; else sk[r] = rn;
      }
      named_bar_sync(kBarPrep, 128);

      mbar_wait_bounded(mma_p, ph_p, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      ph_p ^= 1u;
      tc::fence_after_sync();

      // ---- P rows (lanes 0-63), A rows (lanes 64-127); then Q rows scaled in place
      {
        float v[64];
        tc::ld32(my_lane + kTmG, v);
        tc::ld32(my_lane + kTmG + 32, v + 32);
        tc::wait_ld();
        if (lt < 64) {
          const int i = lt;
          const float gi = gam[i], si = sq[i] * kQScale;
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float val = v[j] * si * sk[j] * exp2f(gi - gam[j]);
            v[j] = (j <= i) ? val : 0.f;
          }
          store_row_bf16<64>(slot + kSlP, i, 0, v);
        } else {
          const int i = lt - 64;
          const float gi = gam[i], bi = bet[i] * sk[i];
          float* A = reinterpret_cast<float*>(smem + kOffAT);
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float val = bi * v[j] * sk[j] * exp2f(gi - gam[j]);
            A[i * kLd + j] = (j < i) ? val : 0.f;
          }
        }
      }
      tc::fence_before_sync();
      named_bar_sync(kBarPrep, 128);  // G consumed, A complete
      // Qr = diag(e^gamma s_q 128^-0.5) Q (both 64-dim boxes of row r), done by
      // the threads idle during the diagonal-block substitution
      invert_unit_lower64(reinterpret_cast<const float*>(smem + kOffAT), reinterpret_cast<float*>(smem + kOffTf),
                          reinterpret_cast<float*>(smem + kOffZ), lt, [&](int r) {
                            const float sc = exp2f(gam[r]) * sq[r] * kQScale;
                            scale_row_bf16(slot + kSlX, r, sc);
                            scale_row_bf16(slot + kSlY, r, sc);
                          });
      {
        const int i = lt & 63;
        const float* T = reinterpret_cast<const float*>(smem + kOffTf);
        float v[64];
        if (lt < 64) {
#pragma unroll
          for (int j = 0; j < 64; ++j) v[j] = T[i * kLd + j] * bet[j] * exp2f(gam[j]) * sk[j];
          store_row_bf16<64>(smem + kOffAT, i, 0, v);  // TW
        } else {
#pragma unroll
          for (int j = 0; j < 64; ++j) v[j] = T[i * kLd + j] * bet[j];
          store_row_bf16<64>(smem + kOffAT + kBox, i, 0, v);  // TU
        }
      }
      fence_proxy_async_smem();
      tc::fence_before_sync();
      named_bar_sync(kBarPrep, 128);
      tc::fence_after_sync();

      // ---- W^T = K^T TW^T, U^T = V^T TU^T (A operands MN-major from the TMA tiles)
      if (lt == 0) {
        tc::fence_after_sync();
        const uint32_t id = tc::idesc_bf16(128, 64, true, false);
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tm + kTmWT, tc::sdesc_sw128(aslot + kSlX + kBox + ks * 2048, kSlY - kSlX, 1024),
                       tc::sdesc_sw128(sbase + kOffAT + ks * 32, 16, 1024), id, ks > 0);
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tm + kTmUT, tc::sdesc_sw128(aslot + kSlV + ks * 2048, kBox, 1024),
                       tc::sdesc_sw128(sbase + kOffAT + kBox + ks * 32, 16, 1024), id, ks > 0);
        tc::commit(mma_p);
      }
      mbar_wait_bounded(mma_p, ph_p, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      ph_p ^= 1u;
      tc::fence_after_sync();
      {
        float v[64];
        tc::ld32(my_lane + kTmWT, v);
        tc::ld32(my_lane + kTmWT + 32, v + 32);
        tc::wait_ld();
        store_row_bf16<64>(slot + kSlWT, lt, 0, v);  // row = dk
        tc::ld32(my_lane + kTmUT, v);
        tc::ld32(my_lane + kTmUT + 32, v + 32);
        tc::wait_ld();
        store_row_bf16<64>(slot + kSlV, lt, 0, v);  // U^T row = dv (V tile is consumed)
      }
      {
        float* scal = reinterpret_cast<float*>(slot + kSlScal);
        const float gC = gam[kC - 1];
        if (lt < kC) scal[4 + lt] = sk[lt] * exp2f(gC - gam[lt]);
        if (lt == 0) scal[0] = exp2f(gC);
      }
      fence_proxy_async_smem();
      tc::fence_before_sync();
      mbar_arrive(&full_bar[s]);
      // prep-private SMEM (gates, A/T scratch) is rewritten next chunk only
      // after this barrier
      named_bar_sync(kBarPrep, 128);
    }
  } else {
    // =================================================================== recurrence
    {
      const float* s0 = p.init_state ? p.init_state + (static_cast<int64_t>(b) * p.Hv + h) * kDK * kDV : nullptr;
      for (int k0 = 0; k0 < kDK; k0 += 32) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = s0 ? s0[(k0 + i) * kDV + lt] : 0.f;
        tc::st32(my_lane + kTmS + k0, v);
      }
      tc::wait_st();
    }
    uint32_t ph_r = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int s = c & 1;
      unsigned char* slot = smem + kOffSlot0 + s * kSlotBytes;
      const uint32_t aslot = sbase + kOffSlot0 + s * kSlotBytes;
      const float* scal = reinterpret_cast<const float*>(slot + kSlScal);
      mbar_wait_bounded(&full_bar[s], (c >> 1) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      tc::fence_after_sync();
      const float eC = scal[0];
      // the previous chunk's output store must have read the staging tile
      // (it shares SMEM with the bf16 state written next)
      if (lt == 0) bulk_wait_read0();
      named_bar_sync(kBarRec, 128);

      // ---- bf16(S_c) -> SMEM, S^T *= e^gamma_C in TMEM
      for (int k0 = 0; k0 < kDK; k0 += 32) {
        float v[32];
        tc::ld32(my_lane + kTmS + k0, v);
        tc::wait_ld();
        store_row_bf16<32>(smem + kOffST + (k0 >> 6) * (2 * kBox), lt, k0 & 63, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= eC;
        tc::st32(my_lane + kTmS + k0, v);
      }
      tc::wait_st();
      fence_proxy_async_smem();
      tc::fence_before_sync();
      named_bar_sync(kBarRec, 128);
      tc::fence_after_sync();

      // ---- X = S^T W^T and O = S^T Qr^T
      if (lt == 0) {
        const uint32_t idX = tc::idesc_bf16(128, 64, false, true);
        const uint32_t idO = tc::idesc_bf16(128, 64, false, false);
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t sa = sbase + kOffST + (ks >> 2) * (2 * kBox) + (ks & 3) * 32;
          tc::mma_bf16(tm + kTmX, tc::sdesc_sw128(sa, 16, 1024),
                       tc::sdesc_sw128(aslot + kSlWT + ks * 2048, 2 * kBox, 1024), idX, ks > 0);
          const uint32_t qb = aslot + (ks < 4 ? kSlX : kSlY) + (ks & 3) * 32;
          tc::mma_bf16(tm + kTmO, tc::sdesc_sw128(sa, 16, 1024), tc::sdesc_sw128(qb, 16, 1024), idO, ks > 0);
        }
        tc::commit(mma_r);
      }
      mbar_wait_bounded(mma_r, ph_r, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      ph_r ^= 1u;
      tc::fence_after_sync();

      // ---- V'^T = U^T - X: raw for O, column-scaled for the state update
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float u[32], x[32];
        tc::ld32(my_lane + kTmX + 32 * half, x);
        load_row_bf16<32>(slot + kSlV, lt, 32 * half, u);
        tc::wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) u[i] -= x[i];
        store_row_bf16<32>(smem + kOffST, lt, 32 * half, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) u[i] *= scal[4 + 32 * half + i];
        store_row_bf16<32>(smem + kOffST + 2 * kBox, lt, 32 * half, u);
      }
      fence_proxy_async_smem();
      tc::fence_before_sync();
      named_bar_sync(kBarRec, 128);
      tc::fence_after_sync();

      // ---- O += V'^T P^T and S^T += V's^T K
      if (lt == 0) {
        const uint32_t idO = tc::idesc_bf16(128, 64, false, false);
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tm + kTmO, tc::sdesc_sw128(sbase + kOffST + ks * 32, 16, 1024),
                       tc::sdesc_sw128(aslot + kSlP + ks * 32, 16, 1024), idO, true);
        const uint32_t idS = tc::idesc_bf16(128, 128, false, true);
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tm + kTmS, tc::sdesc_sw128(sbase + kOffST + 2 * kBox + ks * 32, 16, 1024),
                       tc::sdesc_sw128(aslot + kSlX + kBox + ks * 2048, kSlY - kSlX, 1024), idS, true);
        tc::commit(mma_r);
      }
      mbar_wait_bounded(mma_r, ph_r, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
      ph_r ^= 1u;
      tc::fence_after_sync();
      // every read of this slot is complete: refill it with chunk c + 2
      if (lt == 0 && c + 2 < nchunks) issue_chunk(c + 2);

      // ---- output: O^T (lane = dv) -> bf16 [64 tokens][128 dv] staging tile
      // (two 64-dv boxes, 128-byte swizzled) -> one TMA tensor store per box;
      // rows past the sequence end are clipped by the tensor map.
      {
        unsigned char* stg = smem + kOffST;
        unsigned char* box = stg + (lt >> 6) * kBox;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float o[32];
          tc::ld32(my_lane + kTmO + 32 * half, o);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            *reinterpret_cast<__nv_bfloat16*>(box + tc::sw128_off(32 * half + i, lt & 63)) = __float2bfloat16_rn(o[i]);
        }
        fence_proxy_async_smem();
        tc::fence_before_sync();
        named_bar_sync(kBarRec, 128);  // O, X and the V' tiles are free; staging is written
        tc::fence_after_sync();
        if (lt == 0) {
          tma_store_3d(&tmO, stg, h * kDV, c * kC, b);
          tma_store_3d(&tmO, stg + kBox, h * kDV + 64, c * kC, b);
          bulk_commit_group();
        }
      }
    }
    if (lt == 0) bulk_wait_all0();
    {
      float* sf = p.final_state + (static_cast<int64_t>(b) * p.Hv + h) * kDK * kDV;
      for (int k0 = 0; k0 < kDK; k0 += 32) {
        float v[32];
        tc::ld32(my_lane + kTmS + k0, v);
        tc::wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) sf[(k0 + i) * kDV + lt] = v[i];
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 512);
}

}  // namespace

extern "C" int ria_gdn_chunk_prefill(const void* q, int64_t q_stride_b, int64_t q_stride_t, const void* k,
                                     int64_t k_stride_b, int64_t k_stride_t, const void* v, int64_t v_stride_b,
                                     int64_t v_stride_t, const float* g, const float* beta, int64_t gb_stride_b,
                                     int64_t gb_stride_t, const float* initial_state, float* final_state, void* out,
                                     int64_t o_stride_b, int64_t o_stride_t, int32_t batch, int32_t seq_len,
                                     int32_t num_k_heads, int32_t num_v_heads, ria_stream_t stream) {
  if (batch < 0 || seq_len < 0) return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: negative size");
  if (batch == 0 || seq_len == 0) return RIA_OK;
  if (!q || !k || !v || !g || !beta || !final_state || !out)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: null pointer argument");
  if (num_k_heads < 1 || num_v_heads < num_k_heads || num_v_heads % num_k_heads)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: %d value heads do not group over %d key heads",
                     num_v_heads, num_k_heads);
  if (batch > 65535) return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: batch too large");
  const int64_t qk_row = static_cast<int64_t>(num_k_heads) * kDK, v_row = static_cast<int64_t>(num_v_heads) * kDV;
  if (q_stride_t < qk_row || k_stride_t < qk_row || v_stride_t < v_row || o_stride_t < v_row ||
      gb_stride_t < num_v_heads)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: token stride smaller than the row width");
  if (!ria::aligned(q, 16) || !ria::aligned(k, 16) || !ria::aligned(v, 16) || (q_stride_t % 8) ||
      (k_stride_t % 8) || (v_stride_t % 8) || (q_stride_b % 8) || (k_stride_b % 8) || (v_stride_b % 8))
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: q/k/v must be 16-byte aligned with 16-byte strides");

  CUtensorMap tmQ, tmK, tmV;
  const uint32_t box[3] = {64, 64, 1};
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(qk_row), static_cast<uint64_t>(seq_len),
                              static_cast<uint64_t>(batch)};
    const uint64_t sq[2] = {static_cast<uint64_t>(q_stride_t) * 2, static_cast<uint64_t>(q_stride_b) * 2};
    const uint64_t sk[2] = {static_cast<uint64_t>(k_stride_t) * 2, static_cast<uint64_t>(k_stride_b) * 2};
    int rc = ria::encode_bf16_sw128_map(&tmQ, q, 3, dims, sq, box);
    if (rc) return rc;
    rc = ria::encode_bf16_sw128_map(&tmK, k, 3, dims, sk, box);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(v_row), static_cast<uint64_t>(seq_len),
                              static_cast<uint64_t>(batch)};
    const uint64_t sv[2] = {static_cast<uint64_t>(v_stride_t) * 2, static_cast<uint64_t>(v_stride_b) * 2};
    int rc = ria::encode_bf16_sw128_map(&tmV, v, 3, dims, sv, box);
    if (rc) return rc;
  }

  CUtensorMap tmO;
  {
    if (!ria::aligned(out, 16) || (o_stride_t % 8) || (o_stride_b % 8))
      return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: out must be 16-byte aligned with 16-byte strides");
    const uint64_t dims[3] = {static_cast<uint64_t>(v_row), static_cast<uint64_t>(seq_len),
                              static_cast<uint64_t>(batch)};
    const uint64_t so[2] = {static_cast<uint64_t>(o_stride_t) * 2, static_cast<uint64_t>(o_stride_b) * 2};
    int rc = ria::encode_bf16_sw128_map(&tmO, out, 3, dims, so, box);
    if (rc) return rc;
  }

  PrefillParams p;
  p.g = g;
  p.beta = beta;
  p.gs_b = gb_stride_b;
  p.gs_t = gb_stride_t;
  p.init_state = initial_state;
  p.final_state = final_state;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.os_b = o_stride_b;
  p.os_t = o_stride_t;
  p.T = seq_len;
  p.Hv = num_v_heads;
  p.group = num_v_heads / num_k_heads;
  p.err = ria::device_error_word();

  cudaError_t e = cudaFuncSetAttribute(gdn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_gdn_chunk_prefill: smem attribute: %s", cudaGetErrorString(e));
  gdn_prefill_kernel<<<dim3(num_v_heads, batch), kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(tmQ, tmK,
                                                                                                          tmV, tmO, p);
  return ria::check_launch("ria_gdn_chunk_prefill");
}
