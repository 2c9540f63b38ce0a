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
// B200 design: everything that does not depend on the state is chunk-parallel
// and runs in its own kernel, so the state recurrence is a short chain of
// tensor-core steps.
//   * gdn_chunk_prep_kernel: one 128-thread CTA per (chunk, value head,
//     sequence), four CTAs per SM.  TMA loads of the Q/K tiles (3-D tensor
//     maps, no multicast), gates, G = [Q;K] [Q;K]^T on the tensor cores (the
//     q / k norms from its diagonal), the causal score tile P and A, the
//     64x64 unit-lower-triangular inverse (16x16 diagonal blocks by
//     substitution, off-diagonal blocks by the 2x2 block rule on tf32
//     mma.sync), then U^T = V^T TU^T and the token-major W = TW K on the
//     tensor cores.  Writes one 41,600-byte record per (sequence, head, chunk)
//     to the workspace: W [64][128 dk] bf16, U^T [128 dv][64] fp16, P [64][64] bf16
//     and the chunk scalars (e^gamma_C, the per-token state-update scale
//     s_k e^(gamma_C - gamma), the per-token output scale e^gamma s_q 128^-0.5).
//   * gdn_chunk_recurrence_kernel: one 512-thread CTA per (sequence, value
//     head), four threads per TMEM lane, each on a quarter of the columns.  The fp32 state S^T (lane = dv, column = dk) stays in TMEM for
//     the whole prompt; per chunk: bf16 copy of S^T into TMEM, then
//     [X | O] = S^T [W | Qr]^T as one N = 128 product (A read from TMEM),
//     V'^T = U^T - X (raw as bf16 for O, column-scaled as fp16 for the state,
//     both back into TMEM),
//     S^T += V's^T K and O += V'^T P^T.  The chunk's operands (Q, K, W, U^T,
//     P, scalars) arrive by TMA through a three-slot ring refilled as soon as a chunk's MMAs are
//     complete; O is double-buffered in TMEM so the output of chunk c-1 is
//     written while chunk c's MMAs run.
// When the workspace holds fewer chunks than the prompt, the host runs the
// pair over blocks of chunks with the state carried in final_state.  Every
// product is an M = 128 UMMA (tcgen05.mma cta_group::1 kind::f16, fp32
// accumulation in TMEM); every wait is bounded.
//
// Operand precision: q, k, v arrive as bf16.  The products that feed the
// state run on fp16 operands (11-bit significand: rounding 2^-12 against
// bf16's 2^-9): U^T = V^T TU^T (TU and V in fp16, U^T stored fp16) and the
// state update S^T += V's^T K (V's^T and K in fp16), with K and V converted
// in shared memory.  With bf16 there, the final fp32 state sat about 3e-3
// (relative RMS) from the token-by-token rule, set by the roundings of TU,
// U^T and V's^T; fp16 brings it to about 4e-4 at the same instruction count.
// The other products keep bf16 operands (the Gram product on the raw q / k,
// W = TW K, [X | O] = S^T [W | Qr]^T with a bf16 copy of the state, O +=
// V'^T P^T): they reach the final state only through tokens whose weight in it
// has decayed, and the outputs through errors far inside their bar.  fp16's
// range holds every fp16 operand for inputs below 65504 in magnitude (T has a
// unit diagonal and entries of order one; U and the state are of the order of
// v) -- the range router-ia's own CUDA path computes q, k and v in (its
// projections are fp16).
#include <algorithm>
#include <climits>

#include "ria_capi_internal.h"
#include "ria_common.cuh"
#include "tcgen05.cuh"

namespace {

constexpr int kC = 64;
constexpr int kDK = 128;
constexpr int kDV = 128;
constexpr float kQScale = 0.08838834764831845f;  // 128 ** -0.5
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kBox = 8192;  // 64 rows x 128 bytes, 128-byte swizzled

// Workspace record of one (sequence, value head, chunk).
constexpr uint32_t kRecW = 0;          // W [64 tokens][128 dk] bf16 as two [64][64] boxes (dk 0-63, 64-127)
constexpr uint32_t kRecUT = 16384;     // U^T [128 dv][64 tokens] fp16
constexpr uint32_t kRecP = 32768;      // P [64 t][64 j] bf16
constexpr uint32_t kRecScal = 40960;   // f32: [0] e^gamma_C, [4..67] state scale, [68..131] output scale
constexpr uint32_t kScalBytes = 528;   // 132 floats
constexpr uint32_t kRecBytes = 41600;  // 325 rows of 128 bytes
constexpr uint32_t kRecRows = kRecBytes / 128;

// ---------------------------------------------------------------- prep SMEM
// X = [Q dims 0-63 | K dims 0-63], Y = [Q dims 64-127 | K dims 64-127]
// (128-byte-swizzled 64-row boxes).  Once G is done, P is staged in the first
// Q box for its TMA store, then V (dims 0-63, 64-127) is loaded over the two
// Q boxes, and once U^T is computed its staging tile goes over V.  A and T
// are fp32 and keep only their ten lower-triangular 16x16 blocks (padded rows
// of kBl floats); after the inverse the operand tiles TW (bf16) | TU (fp16) go over A
// and the front of T, and W is staged over them once its product is done.
// Four CTAs fit on an SM.
constexpr int kBl = 17;
constexpr uint32_t kBlkBytes = 16 * kBl * 4;  // 1088
constexpr uint32_t kPX = 0, kPY = 2 * kBox;
constexpr uint32_t kPA = 4 * kBox;              // fp32 A, packed blocks
constexpr uint32_t kPT = kPA + 10 * kBlkBytes;  // fp32 T, packed blocks
constexpr uint32_t kPTw = kPA;                  // TW (bf16) | TU (fp16), two boxes, once T is consumed
constexpr uint32_t kPMisc = kPT + 10 * kBlkBytes;
constexpr uint32_t kPGam = kPMisc, kPBet = kPMisc + 256, kPSq = kPMisc + 512, kPSk = kPMisc + 768,
                   kPEbk = kPMisc + 1024, kPGraw = kPMisc + 1280;
constexpr uint32_t kPBar = kPMisc + 1296;  // tma_qk, tma_v, mma, tslot
constexpr uint32_t kPSmem = kPBar + 32;
static_assert(kPA % 1024 == 0, "operand tiles need 1024-byte alignment");
static_assert(2 * kBox <= 20 * kBlkBytes, "TW | TU over A and T");
static_assert(kPMisc % 16 == 0 && kPBar % 8 == 0, "misc alignment");
static_assert(4 * (kPSmem + 1024) <= 228 * 1024, "four prep CTAs per SM");

// Packed lower-triangular 16x16 block (bi, bj), bj <= bi.
__device__ __forceinline__ int tri_blk(int bi, int bj) { return (bi * (bi + 1)) / 2 + bj; }

// ---------------------------------------------------------------- recurrence SMEM
// [W dk 0-63 | Q dk 0-63 | W dk 64-127 | Q dk 64-127]: per 64-dk half a
// 128-row K-major operand whose rows 0-63 are W and 64-127 are Q (scaled in
// place to Qr), the B operand of the combined [X | O] product.
constexpr uint32_t kSlWQ = 0;
constexpr uint32_t kSlK = 4 * kBox;     // K dims 0-63 | 64-127
constexpr uint32_t kSlUT = 6 * kBox;    // U^T, two 64-row boxes
constexpr uint32_t kSlP = 8 * kBox;     // P
constexpr uint32_t kSlScal = 9 * kBox;  // chunk scalars
constexpr uint32_t kSlotBytes = 9 * kBox + 1024;
constexpr int kSlots = 3;
constexpr uint32_t kRBar = kSlots * kSlotBytes;  // full[3], bar_x, bar_s, bar_o, tslot
constexpr uint32_t kRSmem = kRBar + 128;
constexpr uint32_t kChunkTx = 9 * kBox + kScalBytes;
static_assert(kRSmem <= 227 * 1024, "recurrence SMEM");

// Recurrence TMEM columns: S^T fp32, [X | O] (two buffers of 128), bf16 S^T,
// bf16 V'^T, fp16 V's^T -- all 512 columns.
constexpr uint32_t kTS = 0, kTD = 128, kTSb = 384, kTV = 448, kTVs = 480;

constexpr uint32_t kBarPrep = 1;

__device__ __forceinline__ uint32_t pack16x2(bool f16, float lo, float hi) {
  return f16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
}

// N fp32 values as fp16 (F16) or bf16 into row `row`, columns col0.. of a
// 128-byte-swizzled 16-bit tile.
template <bool F16, int N>
__device__ __forceinline__ void store_row(unsigned char* tile, int row, int col0, const float* v) {
#pragma unroll
  for (int i = 0; i < N; i += 8) {
    uint4 pk;
    pk.x = pack16x2(F16, v[i], v[i + 1]);
    pk.y = pack16x2(F16, v[i + 2], v[i + 3]);
    pk.z = pack16x2(F16, v[i + 4], v[i + 5]);
    pk.w = pack16x2(F16, v[i + 6], v[i + 7]);
    *reinterpret_cast<uint4*>(tile + tc::sw128_off(row, col0 + i)) = pk;
  }
}

template <int N>
__device__ __forceinline__ void load_row_f16(const unsigned char* tile, int row, int col0, float* v) {
#pragma unroll
  for (int i = 0; i < N; i += 8) {
    const uint4 pk = *reinterpret_cast<const uint4*>(tile + tc::sw128_off(row, col0 + i));
    const __half2* h2 = reinterpret_cast<const __half2*>(&pk);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h2[e]);
      v[i + 2 * e] = f.x;
      v[i + 2 * e + 1] = f.y;
    }
  }
}

// bf16 -> fp16 in place over `chunks` 16-byte chunks starting at `tile`,
// threads `t` of `nt` taking every nt-th chunk (the conversion is exact for
// magnitudes in [6.1e-5, 65504]; smaller ones round to fp16's subnormal step,
// 6e-8).
__device__ __forceinline__ void bf16_to_f16_inplace(unsigned char* tile, int chunks, int t, int nt) {
  for (int c = t; c < chunks; c += nt) {
    uint4 u = *reinterpret_cast<uint4*>(tile + 16 * c);
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
      w[e] = pack_f16x2(f.x, f.y);
    }
    *reinterpret_cast<uint4*>(tile + 16 * c) = u;
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

// 2^x by the special-function unit (ex2.approx.ftz: relative error about
// 2^-22, results below 2^-126 flushed to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

// T = (I + A)^-1 for strictly-lower A by 128 threads; A and T are fp32 in
// packed lower blocks (tri_blk, row stride kBl).  The four 16x16 diagonal
// blocks are inverted by substitution (threads 0-63, one column each; the
// blocks' upper parts are written as zeros).  The off-diagonal blocks follow
// by the 2x2 block rule L^-1 = [[L11^-1, 0], [-L22^-1 L21 L11^-1, L22^-1]],
// first inside each 32x32 diagonal half, then for the lower-left 32x32
// quarter with all four warps, on the tensor cores (tf32 in, fp32
// accumulate).
__device__ void invert_unit_lower64(float* A, float* T, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  if (tid < 64) {
    // column jj of diagonal block d: col[ii] = -sum_{m=jj}^{ii-1} A[ii][m] col[m]
    // (col[m] = 0 for m < jj, so the sum may run over all m < ii).  The next
    // row of A is loaded while this one is used, and four partial sums keep
    // the FMA chain short.
    const int d = tid >> 4, jj = tid & 15;
    const float* Ad = A + tri_blk(d, d) * 16 * kBl;
    float col[16];
    float cur[16], nxt[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) cur[m] = m < 1 ? Ad[kBl + m] : 0.f;  // row 1
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) {  // cur holds row ii (ii >= 1); row ii + 1 loads meanwhile
      if (ii >= 1 && ii + 1 < 16) {
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m <= ii) nxt[m] = Ad[(ii + 1) * kBl + m];
      }
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (ii >= 1) {
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m < ii) acc[m & 3] = fmaf(cur[m], col[m], acc[m & 3]);
      }
      const float sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
      col[ii] = (ii < jj) ? 0.f : (ii == jj ? 1.f : -sum);
      if (ii >= 1 && ii + 1 < 16) {
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m <= ii) cur[m] = nxt[m];
      }
    }
    float* Td = T + tri_blk(d, d) * 16 * kBl;
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) Td[ii * kBl + jj] = col[ii];
  }
  named_bar_sync(kBarPrep, 128);
  const int g = lane >> 2, tg = lane & 3;
  auto blk = [&](float* M, int bi, int bj) { return M + tri_blk(bi, bj) * 16 * kBl; };
  auto put = [&](float* z, const float (&acc)[2][4], float sgn) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      z[g * kBl + 8 * nt + 2 * tg] = sgn * acc[nt][0];
      z[g * kBl + 8 * nt + 2 * tg + 1] = sgn * acc[nt][1];
      z[(g + 8) * kBl + 8 * nt + 2 * tg] = sgn * acc[nt][2];
      z[(g + 8) * kBl + 8 * nt + 2 * tg + 1] = sgn * acc[nt][3];
    }
  };
  // 32x32 diagonal halves: T10 = -T11 A10 T00 (warp 0), T32 = -T33 A32 T22
  // (warp 1), the sum parked in the result's own block.
  if (warp < 2) {
    const int bi = 2 * warp + 1, bj = 2 * warp;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    warp_mma16(acc, blk(A, bi, bj), kBl, blk(T, bj, bj), kBl, lane);
    float* z = blk(T, bi, bj);
    put(z, acc, 1.f);
    __syncwarp();
    float tt[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    warp_mma16(tt, blk(T, bi, bi), kBl, z, kBl, lane);
    __syncwarp();  // every lane has read the sum
    put(z, tt, -1.f);
  }
  named_bar_sync(kBarPrep, 128);
  // The lower-left 32x32 quarter, T[2:4, 0:2] = -T[2:4, 2:4] (A[2:4, 0:2]
  // T[0:2, 0:2]), warp w on block (2 + w / 2, w % 2): first Z = A T into the
  // block, then the product with the lower-right half (read before anyone
  // overwrites a Z block).
  const int bi = 2 + (warp >> 1), bj = warp & 1;
  {
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int m = bj; m < 2; ++m) warp_mma16(acc, blk(A, bi, m), kBl, blk(T, m, bj), kBl, lane);
    put(blk(T, bi, bj), acc, 1.f);
  }
  named_bar_sync(kBarPrep, 128);
  float tt[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int m = 2; m <= bi; ++m) warp_mma16(tt, blk(T, bi, m), kBl, blk(T, m, bj), kBl, lane);
  named_bar_sync(kBarPrep, 128);
  put(blk(T, bi, bj), tt, -1.f);
  named_bar_sync(kBarPrep, 128);
}

struct PrepParams {
  const float* g;  // [B][T][Hv] log decay
  const float* beta;
  int64_t gs_b, gs_t;
  unsigned char* ws;  // records [B][Hv][nblk]
  int T;
  int Hv;
  int group;  // value heads per key head
  int c0;     // first chunk of this block
  int nblk;   // records per (sequence, head) in the workspace
  unsigned int* err;
};

__global__ void __launch_bounds__(128, 4)
    gdn_chunk_prep_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmW,
                          const PrepParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int cl = blockIdx.x;
  const int c = p.c0 + cl;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / p.group;
  const int lt = threadIdx.x;
  const int warp = lt >> 5;
  uint64_t* tma_qk = reinterpret_cast<uint64_t*>(smem + kPBar);
  uint64_t* tma_v = tma_qk + 1;
  uint64_t* mma = tma_qk + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kPBar + 24);
  float* gam = reinterpret_cast<float*>(smem + kPGam);  // gamma * log2(e)
  float* bet = reinterpret_cast<float*>(smem + kPBet);
  float* sq = reinterpret_cast<float*>(smem + kPSq);
  float* sk = reinterpret_cast<float*>(smem + kPSk);
  float* graw = reinterpret_cast<float*>(smem + kPGraw);
  float* ebk = reinterpret_cast<float*>(smem + kPEbk);  // beta e^gamma s_k per column
  const uint32_t sbase = smem_u32(smem);
  const int64_t rec_idx = static_cast<int64_t>(b * p.Hv + h) * p.nblk + cl;
  unsigned char* rec = p.ws + rec_idx * static_cast<int64_t>(kRecBytes);
  const int32_t rec_row = static_cast<int32_t>(rec_idx * kRecRows);

  if (lt == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmW);
    mbar_init(tma_qk, 1);
    mbar_init(tma_v, 1);
    mbar_init(mma, 1);
    mbar_fence_init();
    mbar_arrive_expect_tx(tma_qk, 4 * kBox);
    tma_load_3d(smem + kPX, &tmQ, hk * kDK, c * kC, b, tma_qk);
    tma_load_3d(smem + kPX + kBox, &tmK, hk * kDK, c * kC, b, tma_qk);
    tma_load_3d(smem + kPY, &tmQ, hk * kDK + 64, c * kC, b, tma_qk);
    tma_load_3d(smem + kPY + kBox, &tmK, hk * kDK + 64, c * kC, b, tma_qk);
  }
  if (warp == 1) {  // beside thread 0's barrier set-up and TMA issue
    tc::tmem_alloc(tslot, 128);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *tslot;
  const uint32_t my_lane = tm + (static_cast<uint32_t>(warp * 32) << 16);
  constexpr uint32_t kTmG = 0, kTmW = 0, kTmU = 0;  // G, then U^T, then W (128 columns)

  // gates: inclusive scan of the chunk's log decays inside each of the two warps
  float gscan = 0.f, bv = 0.f;
  if (lt < kC) {
    const int t = c * kC + lt;
    const bool ok = t < p.T;
    const int64_t gi = static_cast<int64_t>(b) * p.gs_b + static_cast<int64_t>(t) * p.gs_t + h;
    gscan = ok ? p.g[gi] : 0.f;
    bv = ok ? p.beta[gi] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, gscan, o);
      if ((lt & 31) >= o) gscan += up;
    }
    if (lt == 31) graw[0] = gscan;  // warp 0 total
  }
  mbar_wait_bounded(tma_qk, 0, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
  // ---- G = [Q;K] [Q;K]^T (raw q, k; N = 128 costs the M = 128 UMMA no more
  // time than N = 64): columns 64 + j hold q_i.k_j and k_i.k_j, and the
  // diagonal gives the squared row norms of q and k.
  if (lt == 0) {
    tc::fence_after_sync();
    const uint32_t id = tc::idesc_bf16(128, 128, false, false);
    for (int ks = 0; ks < 8; ++ks) {
      const uint64_t d = tc::sdesc_sw128(sbase + (ks < 4 ? kPX : kPY) + (ks & 3) * 32, 16, 1024);
      tc::mma_bf16(tm + kTmG, d, d, id, ks > 0);
    }
    tc::commit(mma);
  }
  if (lt < kC) {
    named_bar_sync(kBarPrep + 1, 64);  // warp 0's total is in graw
    gam[lt] = (lt >= 32 ? gscan + graw[0] : gscan) * kLog2e;
    bet[lt] = bv;
  }
  mbar_wait_bounded(mma, 0, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
  tc::fence_after_sync();
  {  // row lt's squared norm sits in column lt (warp w: columns 32w .. 32w + 31)
    float v[32];
    tc::ld32(my_lane + kTmG + 32 * warp, v);
    tc::wait_ld();
    // v[lane] by halving selects (static register indices only)
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
      const bool hi = (lt & w) != 0;
#pragma unroll
      for (int e = 0; e < w; ++e) v[e] = hi ? v[e + w] : v[e];
    }
    const float rn = rsqrtf(v[0] + 1e-6f);
    if (lt < 64) sq[lt] = rn; else sk[lt - 64] = rn;
  }
  named_bar_sync(kBarPrep, 128);
  if (lt < kC) ebk[lt] = bet[lt] * exp2f(gam[lt]) * sk[lt];

  // ---- P rows (lanes 0-63) to the record, A rows (lanes 64-127) to SMEM,
  // 32 columns per TMEM load.  Rows 0-31 have no entries in columns 32-63
  // (causal), so warps 0 and 2 load one half only (warp 0 stores zeros for
  // its P row's second half; A keeps lower blocks only).
  {
    const bool is_p = lt < 64;
    const int i = lt & 63;
    const int bi = i >> 4;
    const float gi = gam[i];
    const float si = is_p ? sq[i] * kQScale : bet[i] * sk[i];
    const int halves = (lt & 32) ? 2 : 1;
    float* Ab = reinterpret_cast<float*>(smem + kPA);

#pragma unroll 1
    for (int hf = 0; hf < halves; ++hf) {
      const int j0 = 32 * hf;
      float v[32];
      tc::ld32(my_lane + kTmG + 64 + j0, v);
      tc::wait_ld();
#pragma unroll
      for (int e4 = 0; e4 < 32; e4 += 4) {
        const float4 sk4 = *reinterpret_cast<const float4*>(sk + j0 + e4);
        const float4 gm4 = *reinterpret_cast<const float4*>(gam + j0 + e4);
        const float skv[4] = {sk4.x, sk4.y, sk4.z, sk4.w}, gmv[4] = {gm4.x, gm4.y, gm4.z, gm4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = j0 + e4 + e;
          const bool keep = is_p ? j <= i : j < i;
          v[e4 + e] = keep ? v[e4 + e] * si * skv[e] * ex2_approx(gi - gmv[e]) : 0.f;
        }
      }
      if (is_p) {
        store_row<false, 32>(smem + kPX, i, j0, v);
      } else {
#pragma unroll
        for (int gq = 0; gq < 2; ++gq) {
          const int bj = 2 * hf + gq;
          if (bj <= bi) {
            float* dst = Ab + tri_blk(bi, bj) * 16 * kBl + (i & 15) * kBl;
#pragma unroll
            for (int e = 0; e < 16; ++e) dst[e] = v[16 * gq + e];
          }
        }
      }
    }
    if (lt < 32) {
#pragma unroll
      for (int c8 = 32; c8 < 64; c8 += 8)
        *reinterpret_cast<uint4*>(smem + kPX + tc::sw128_off(i, c8)) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  fence_proxy_async_smem();
  tc::fence_before_sync();
  named_bar_sync(kBarPrep, 128);  // G consumed, A complete, P staged over the first Q box
  // P to the record; once the store has read the staging tile, V comes in
  // over the Q boxes (dims 0-63, 64-127).  Thread 64 issues both while
  // threads 0-63 run the diagonal-block substitution.
  if (lt == 64) {
    tma_store_2d(&tmW, smem + kPX, 0, rec_row + kRecP / 128);
    bulk_commit_group();
    bulk_wait_read0();
    mbar_arrive_expect_tx(tma_v, 2 * kBox);
    tma_load_3d(smem + kPX, &tmV, h * kDV, c * kC, b, tma_v);
    tma_load_3d(smem + kPY, &tmV, h * kDV + 64, c * kC, b, tma_v);
  }
  invert_unit_lower64(reinterpret_cast<float*>(smem + kPA), reinterpret_cast<float*>(smem + kPT), lt);
  {  // TW = T diag(beta e^gamma s_k) (lanes 0-63, bf16), TU = T diag(beta) (lanes 64-127, fp16);
     // T's row i is zero past its diagonal block.  All of T is read before
     // the tiles are written over A and T.
    const int i = lt & 63;
    const int bi = i >> 4;
    const float* Tb = reinterpret_cast<const float*>(smem + kPT);
    const float* cs = lt < 64 ? ebk : bet;
    uint32_t pk[32];
#pragma unroll
    for (int bj = 0; bj < 4; ++bj) {
      const float* trow = Tb + tri_blk(bi, bj) * 16 * kBl + (i & 15) * kBl;
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        float x0 = 0.f, x1 = 0.f;
        if (bj <= bi) {
          x0 = trow[e] * cs[16 * bj + e];
          x1 = trow[e + 1] * cs[16 * bj + e + 1];
        }
        pk[8 * bj + e / 2] = pack16x2(lt >= 64, x0, x1);
      }
    }
    named_bar_sync(kBarPrep, 128);
    unsigned char* dst = smem + kPTw + (lt < 64 ? 0 : kBox);
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8)
      *reinterpret_cast<uint4*>(dst + tc::sw128_off(i, 8 * c8)) =
          make_uint4(pk[4 * c8], pk[4 * c8 + 1], pk[4 * c8 + 2], pk[4 * c8 + 3]);
  }
  // V (loaded during the inverse) to fp16 in place
  mbar_wait_bounded(tma_v, 0, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
  bf16_to_f16_inplace(smem + kPX, kBox / 16, lt, 128);
  bf16_to_f16_inplace(smem + kPY, kBox / 16, lt, 128);
  fence_proxy_async_smem();
  tc::fence_before_sync();
  named_bar_sync(kBarPrep, 128);
  tc::fence_after_sync();

  // ---- U^T = V^T TU^T (A = V, MN-major over the Q boxes), into G's columns
  if (lt == 0) {
    tc::fence_after_sync();
    const uint32_t id = tc::idesc_f16(128, 64, true, false);
    for (int ks = 0; ks < 4; ++ks)
      tc::mma_bf16(tm + kTmU, tc::sdesc_sw128(sbase + kPX + ks * 2048, kPY - kPX, 1024),
                   tc::sdesc_sw128(sbase + kPTw + kBox + ks * 32, 16, 1024), id, ks > 0);
    tc::commit(mma);
  }
  {
    float* scal = reinterpret_cast<float*>(rec + kRecScal);
    const float gC = gam[kC - 1];
    if (lt < kC) {
      scal[4 + lt] = sk[lt] * exp2f(gC - gam[lt]);
      scal[68 + lt] = exp2f(gam[lt]) * sq[lt] * kQScale;
    }
    if (lt < 4) scal[lt] = lt == 0 ? exp2f(gC) : 0.f;
  }
  mbar_wait_bounded(mma, 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
  tc::fence_after_sync();
  {  // U^T row lt (dv) staged over V (consumed): rows 0-63 in the first Q box, 64-127 in the second
    unsigned char* tile = smem + (lt < 64 ? kPX : kPY);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float v[32];
      tc::ld32(my_lane + kTmU + 32 * hf, v);
      tc::wait_ld();
      store_row<true, 32>(tile, lt & 63, 32 * hf, v);
    }
  }
  fence_proxy_async_smem();
  tc::fence_before_sync();
  named_bar_sync(kBarPrep, 128);  // U^T is read out of TMEM and staged
  if (lt == 64) {
    tma_store_2d(&tmW, smem + kPX, 0, rec_row + kRecUT / 128);
    tma_store_2d(&tmW, smem + kPY, 0, rec_row + kRecUT / 128 + 64);
    bulk_commit_group();
  }
  // ---- W = TW K, token-major: A = [TW; TU] (the TU rows give unused rows
  // 64-127), B = the K tile (MN-major, dk across the two boxes), N = 128 dk
  if (lt == 0) {
    tc::fence_after_sync();
    const uint32_t id = tc::idesc_bf16(128, 128, false, true);
    for (int ks = 0; ks < 4; ++ks)
      tc::mma_bf16(tm + kTmW, tc::sdesc_sw128(sbase + kPTw + ks * 32, 16, 1024),
                   tc::sdesc_sw128(sbase + kPX + kBox + ks * 2048, kPY - kPX, 1024), id, ks > 0);
    tc::commit(mma);
  }
  mbar_wait_bounded(mma, 0, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
  tc::fence_after_sync();
  if (lt < 64) {  // W row lt (token) staged over TW | TU (consumed): dk 0-63 and dk 64-127 boxes
#pragma unroll
    for (int q32 = 0; q32 < 4; ++q32) {
      float v[32];
      tc::ld32(my_lane + kTmW + 32 * q32, v);
      tc::wait_ld();
      store_row<false, 32>(smem + kPTw + (q32 >> 1) * kBox, lt, 32 * (q32 & 1), v);
    }
  }
  fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  if (lt == 0) {
    tma_store_2d(&tmW, smem + kPTw, 0, rec_row + kRecW / 128);
    tma_store_2d(&tmW, smem + kPTw + kBox, 0, rec_row + kRecW / 128 + 64);
    bulk_commit_group();
    bulk_wait_read0();  // the stores have read SMEM; their writes complete with the grid
  }
  if (lt == 64) bulk_wait_read0();  // the U^T stores
  if (warp == 1) tc::tmem_dealloc(tm, 128);
}

struct RecParams {
  const unsigned char* ws;
  const float* init_state;  // [B][Hv][128 k][128 v] or null (zeros)
  float* final_state;
  int T;
  int Hv;
  int group;
  int c0;
  int nblk;
  unsigned int* err;
};

__device__ __forceinline__ void pack16(const float* v, uint32_t* pk) {
#pragma unroll
  for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
}

__global__ void __launch_bounds__(512, 1)
    gdn_chunk_recurrence_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                                const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmO,
                                const RecParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int hk = h / p.group;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int wg = tid >> 7;   // column quarter handled by this warpgroup
  const int lt = tid & 127;  // TMEM lane = dv
  const int lane = tid & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRBar);
  uint64_t* bar_x = full + kSlots;
  uint64_t* bar_s = bar_x + 1;
  uint64_t* bar_o = bar_x + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_x + 3);
  const uint32_t sbase = smem_u32(smem);
  const int nchunks = (p.T + kC - 1) / kC;
  const int n = min(p.nblk, nchunks - p.c0);
  const int64_t rec0 = static_cast<int64_t>(b * p.Hv + h) * p.nblk;
  constexpr int kStoreTid = 128;  // issues output stores and refills (warp 4)

  // TMA of block-local chunk j's operands into slot j % 3 (one thread).
  auto issue = [&](int j) {
    const int s = j % kSlots;
    unsigned char* slot = smem + s * kSlotBytes;
    const int c = p.c0 + j;
    const int32_t row = static_cast<int32_t>((rec0 + j) * kRecRows);
    mbar_arrive_expect_tx(&full[s], kChunkTx);
    tma_load_3d(slot + kSlWQ + kBox, &tmQ, hk * kDK, c * kC, b, &full[s]);
    tma_load_3d(slot + kSlWQ + 3 * kBox, &tmQ, hk * kDK + 64, c * kC, b, &full[s]);
    tma_load_3d(slot + kSlK, &tmK, hk * kDK, c * kC, b, &full[s]);
    tma_load_3d(slot + kSlK + kBox, &tmK, hk * kDK + 64, c * kC, b, &full[s]);
    tma_load_2d(slot + kSlWQ, &tmW, 0, row + kRecW / 128, &full[s]);
    tma_load_2d(slot + kSlWQ + 2 * kBox, &tmW, 0, row + kRecW / 128 + 64, &full[s]);
    tma_load_2d(slot + kSlUT, &tmW, 0, row + kRecUT / 128, &full[s]);
    tma_load_2d(slot + kSlUT + kBox, &tmW, 0, row + kRecUT / 128 + 64, &full[s]);
    tma_load_2d(slot + kSlP, &tmW, 0, row + kRecP / 128, &full[s]);
    bulk_g2s(slot + kSlScal, p.ws + (rec0 + j) * static_cast<int64_t>(kRecBytes) + kRecScal, kScalBytes, &full[s]);
  };

  if (tid == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmO);
    for (int i = 0; i < kSlots; ++i) mbar_init(&full[i], 1);
    mbar_init(bar_x, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_fence_init();
    for (int j = 0; j < min(n, kSlots); ++j) issue(j);
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *tslot;
  const uint32_t my_lane = tm + (static_cast<uint32_t>((warp & 3) * 32) << 16);

  {  // initial state: warpgroup wg loads dk columns [64 wg, 64 wg + 64)
    const float* s0 = p.init_state ? p.init_state + static_cast<int64_t>(b * p.Hv + h) * kDK * kDV : nullptr;
    {
      const int k0 = 32 * wg;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = s0 ? s0[(k0 + i) * kDV + lt] : 0.f;
      tc::st32(my_lane + kTS + k0, v);
    }
    tc::wait_st();
  }

  // Output of block-local chunk j, step 1 (all threads): O^T (lane = dv) from
  // TMEM buffer j & 1 into a [64 tokens][128 dv] bf16 staging tile (two
  // 128-byte-swizzled 64-dv boxes) in the W^T region of chunk j's slot, whose
  // MMAs are then all complete.  Lane pairs swap halves so that every SMEM
  // store is a bf16 pair.
  auto stage_output = [&](int j) {
    mbar_wait_bounded(bar_o, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
    tc::fence_after_sync();
    float o[16];
    tc::ld16(my_lane + kTD + 128 * (j & 1) + 64 + 16 * wg, o);
    tc::wait_ld();
    unsigned char* stg = smem + (j % kSlots) * kSlotBytes + kSlWQ + (lt >> 6) * kBox;
    const bool odd = lane & 1;
    const int col = (lt & 63) & ~1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = odd ? o[2 * i] : o[2 * i + 1];
      const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
      const int t = 16 * wg + 2 * i + (odd ? 1 : 0);
      const uint32_t pk = odd ? pack_bf16x2(recv, o[2 * i + 1]) : pack_bf16x2(o[2 * i], recv);
      *reinterpret_cast<uint32_t*>(stg + tc::sw128_off(t, col)) = pk;
    }
    fence_proxy_async_smem();
  };
  // Step 2 (one thread, after a barrier): TMA tensor stores of the staging
  // tile (rows past the prompt end are clipped by the tensor map); once the
  // stores have read it, the slot is refilled with chunk j + 3.
  auto store_output = [&](int j) {
    const unsigned char* stg = smem + (j % kSlots) * kSlotBytes + kSlWQ;
    const int c = p.c0 + j;
    tma_store_3d(&tmO, stg, h * kDV, c * kC, b);
    tma_store_3d(&tmO, stg + kBox, h * kDV + 64, c * kC, b);
    bulk_commit_group();
    bulk_wait_read0();
    if (j + kSlots < n) issue(j + kSlots);
  };

  for (int j = 0; j < n; ++j) {
    const int s = j % kSlots;
    unsigned char* slot = smem + s * kSlotBytes;
    const uint32_t aslot = sbase + s * kSlotBytes;
    const float* scal = reinterpret_cast<const float*>(slot + kSlScal);
    const uint32_t sb = kTSb;                  // bf16 S^T
    const uint32_t dd = kTD + 128 * (j & 1);  // this chunk's [X | O]
    mbar_wait_bounded(&full[s], (j / kSlots) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
    const float eC = scal[0];

    // ---- bf16 S^T into TMEM (A operand of X and O), S^T *= e^gamma_C; Q rows -> Qr
    {
      const int k0 = 32 * wg;
      float v[32];
      uint32_t pk[16];
      tc::ld32(my_lane + kTS + k0, v);
      tc::wait_ld();
      pack16(v, pk);
      tc::st16(my_lane + sb + k0 / 2, pk);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= eC;
      tc::st32(my_lane + kTS + k0, v);
    }
    {  // Qr = diag(output scale) Q: thread -> (row, 64-dim box, half of the row)
      const int r = tid & 63;
      unsigned char* rowp = slot + kSlWQ + (((tid >> 6) & 1) ? 3 : 1) * kBox + r * 128;
      const float sc = scal[68 + r];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int ch = (2 * (tid >> 7) + c) ^ (r & 7);
        uint4 u = *reinterpret_cast<uint4*>(rowp + ch * 16);
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h2[e]);
          h2[e] = __floats2bfloat162_rn(f.x * sc, f.y * sc);
        }
        *reinterpret_cast<uint4*>(rowp + ch * 16) = u;
      }
    }
    // K to fp16 in place (the B operand of the state update)
    bf16_to_f16_inplace(slot + kSlK, 2 * kBox / 16, tid, 512);
    tc::wait_st();
    fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    // ---- [X | O] = S^T [W | Qr]^T; meanwhile the previous chunk's output goes to staging
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t idXO = tc::idesc_bf16(128, 128, false, false);
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_bf16_ts(tm + dd, tm + sb + ks * 8,
                        tc::sdesc_sw128(aslot + kSlWQ + (ks >> 2) * (2 * kBox) + (ks & 3) * 32, 16, 1024), idXO,
                        ks > 0);
      tc::commit(bar_x);
    }
    if (j > 0) stage_output(j - 1);

    // ---- V'^T = U^T - X: raw (bf16, for O) and column-scaled (fp16, for the state) into TMEM
    mbar_wait_bounded(bar_x, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
    tc::fence_after_sync();
    {
      float x[16], u[16];
      uint32_t pk[8];
      tc::ld16(my_lane + dd + 16 * wg, x);
      load_row_f16<16>(slot + kSlUT, lt, 16 * wg, u);
      tc::wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) u[i] -= x[i];
#pragma unroll
      for (int i = 0; i < 8; ++i) pk[i] = pack_bf16x2(u[2 * i], u[2 * i + 1]);
      tc::st8(my_lane + kTV + 8 * wg, pk);
#pragma unroll
      for (int i = 0; i < 16; ++i) u[i] *= scal[4 + 16 * wg + i];
#pragma unroll
      for (int i = 0; i < 8; ++i) pk[i] = pack_f16x2(u[2 * i], u[2 * i + 1]);
      tc::st8(my_lane + kTVs + 8 * wg, pk);
      tc::wait_st();
    }
    tc::fence_before_sync();
    __syncthreads();

    // ---- S^T += V's^T K first (the next chunk waits only for it), then O += V'^T P^T
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t idS = tc::idesc_f16(128, 128, false, true);
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16_ts(tm + kTS, tm + kTVs + ks * 8, tc::sdesc_sw128(aslot + kSlK + ks * 2048, kBox, 1024), idS,
                        true);
      tc::commit(bar_s);
      const uint32_t idO = tc::idesc_bf16(128, 64, false, false);
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16_ts(tm + dd + 64, tm + kTV + ks * 8, tc::sdesc_sw128(aslot + kSlP + ks * 32, 16, 1024), idO,
                        true);
      tc::commit(bar_o);
    }
    if (tid == kStoreTid && j > 0) store_output(j - 1);
    mbar_wait_bounded(bar_s, j & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
    tc::fence_after_sync();
  }
  if (n > 0) {
    stage_output(n - 1);
    __syncthreads();
    if (tid == kStoreTid) store_output(n - 1);
  }
  if (tid == kStoreTid) bulk_wait_all0();
  {
    float* sf = p.final_state + static_cast<int64_t>(b * p.Hv + h) * kDK * kDV;
    {
      const int k0 = 32 * wg;
      float v[32];
      tc::ld32(my_lane + kTS + k0, v);
      tc::wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) sf[(k0 + i) * kDV + lt] = v[i];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 512);
}

}  // namespace

extern "C" int64_t ria_gdn_chunk_prefill_workspace_bytes(int32_t batch, int32_t seq_len, int32_t num_v_heads) {
  if (batch <= 0 || seq_len <= 0 || num_v_heads <= 0) return 0;
  return static_cast<int64_t>(batch) * num_v_heads * ((seq_len + kC - 1) / kC) * kRecBytes;
}

extern "C" int ria_gdn_chunk_prefill(const void* q, int64_t q_stride_b, int64_t q_stride_t, const void* k,
                                     int64_t k_stride_b, int64_t k_stride_t, const void* v, int64_t v_stride_b,
                                     int64_t v_stride_t, const float* g, const float* beta, int64_t gb_stride_b,
                                     int64_t gb_stride_t, const float* initial_state, float* final_state, void* out,
                                     int64_t o_stride_b, int64_t o_stride_t, void* workspace, int64_t workspace_bytes,
                                     int32_t batch, int32_t seq_len, int32_t num_k_heads, int32_t num_v_heads,
                                     ria_stream_t stream) {
  if (batch < 0 || seq_len < 0) return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: negative size");
  if (batch == 0 || seq_len == 0) return RIA_OK;
  if (!q || !k || !v || !g || !beta || !final_state || !out || !workspace)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: null pointer argument");
  if (num_k_heads < 1 || num_v_heads < num_k_heads || num_v_heads % num_k_heads)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: %d value heads do not group over %d key heads",
                     num_v_heads, num_k_heads);
  if (batch > 65535 || num_v_heads > 65535) return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: grid too large");
  const int64_t qk_row = static_cast<int64_t>(num_k_heads) * kDK, v_row = static_cast<int64_t>(num_v_heads) * kDV;
  if (q_stride_t < qk_row || k_stride_t < qk_row || v_stride_t < v_row || o_stride_t < v_row ||
      gb_stride_t < num_v_heads)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: token stride smaller than the row width");
  if (!ria::aligned(q, 16) || !ria::aligned(k, 16) || !ria::aligned(v, 16) || (q_stride_t % 8) ||
      (k_stride_t % 8) || (v_stride_t % 8) || (q_stride_b % 8) || (k_stride_b % 8) || (v_stride_b % 8))
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: q/k/v must be 16-byte aligned with 16-byte strides");
  if (!ria::aligned(out, 16) || (o_stride_t % 8) || (o_stride_b % 8))
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: out must be 16-byte aligned with 16-byte strides");
  if (!ria::aligned(workspace, 16))
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: workspace must be 16-byte aligned");
  const int nchunks = (seq_len + kC - 1) / kC;
  const size_t per_chunk = static_cast<size_t>(batch) * num_v_heads * kRecBytes;
  // records per (sequence, head): as many chunks as the workspace holds, with
  // the workspace's row count inside the tensor map's 32-bit coordinates
  const size_t row_cap = static_cast<size_t>(INT32_MAX) / (static_cast<size_t>(batch) * num_v_heads * kRecRows);
  const size_t ws = workspace_bytes > 0 ? static_cast<size_t>(workspace_bytes) : 0;
  const int nblk = static_cast<int>(std::min<size_t>({static_cast<size_t>(nchunks), ws / per_chunk, row_cap}));
  if (nblk < 1)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_chunk_prefill: workspace of %zu bytes is below one chunk (%zu bytes)",
                     ws, per_chunk);

  CUtensorMap tmQ, tmK, tmV, tmW, tmO;
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
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(v_row), static_cast<uint64_t>(seq_len),
                              static_cast<uint64_t>(batch)};
    const uint64_t so[2] = {static_cast<uint64_t>(o_stride_t) * 2, static_cast<uint64_t>(o_stride_b) * 2};
    int rc = ria::encode_bf16_sw128_map(&tmO, out, 3, dims, so, box);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {64, static_cast<uint64_t>(batch) * num_v_heads * nblk * kRecRows};
    const uint64_t sw[1] = {128};
    int rc = ria::encode_bf16_sw128_map(&tmW, workspace, 2, dims, sw, box);
    if (rc) return rc;
  }

  PrepParams pp;
  pp.g = g;
  pp.beta = beta;
  pp.gs_b = gb_stride_b;
  pp.gs_t = gb_stride_t;
  pp.ws = static_cast<unsigned char*>(workspace);
  pp.T = seq_len;
  pp.Hv = num_v_heads;
  pp.group = num_v_heads / num_k_heads;
  pp.nblk = nblk;
  pp.err = ria::device_error_word();
  RecParams rp;
  rp.ws = static_cast<const unsigned char*>(workspace);
  rp.final_state = final_state;
  rp.T = seq_len;
  rp.Hv = num_v_heads;
  rp.group = pp.group;
  rp.nblk = nblk;
  rp.err = pp.err;

  cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gdn_chunk_recurrence_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRSmem);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_gdn_chunk_prefill: smem attribute: %s", cudaGetErrorString(e));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int c0 = 0; c0 < nchunks; c0 += nblk) {
    const int nc = std::min(nblk, nchunks - c0);
    pp.c0 = c0;
    gdn_chunk_prep_kernel<<<dim3(nc, num_v_heads, batch), 128, kPSmem, st>>>(tmQ, tmK, tmV, tmW, pp);
    int rc = ria::check_launch("ria_gdn_chunk_prefill (prep)");
    if (rc) return rc;
    rp.c0 = c0;
    rp.init_state = c0 == 0 ? initial_state : final_state;
    gdn_chunk_recurrence_kernel<<<dim3(num_v_heads, batch), 512, kRSmem, st>>>(tmQ, tmK, tmW, tmO, rp);
    rc = ria::check_launch("ria_gdn_chunk_prefill (recurrence)");
    if (rc) return rc;
  }
  return RIA_OK;
}

