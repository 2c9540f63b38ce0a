// K1: fused Gated DeltaNet decode step (one token per sequence, B sequences).
//
// Reference semantics (router-ia v2/src/router_ia/qwen36_attention_cache.py):
//   conv:   history = [state(4), x]; state' = history[-4:]; y = silu(sum w*state')
//           computed in the conv weight dtype (bf16)                      :176-221
//   split:  q = y[0:2048], k = y[2048:4096], v = y[4096:8192]; value head h
//           reads key head h/2 (repeat_interleave(2))                     :237-240
//   gates:  beta = sigmoid(b); g = -exp(A_log) * softplus(a + dt_bias)     :242-250
//   norms:  q,k <- x * rsqrt(sum x^2 + 1e-6); q *= 128^-0.5                :252-254
//   update: S *= exp(g); r = S^T k; d = beta (v - r); S += k d^T; o = S^T q :256-266
//   out:    gated_rmsnorm(o, z, norm_w)  (qwen36_gated_norm_probe.py:19-36)
//
// B200 design
//   * Work unit = (sequence, key head j): value heads 2j and 2j+1 share q/k, so
//     the conv of the q/k channels, the L2 norms and the conv-state write happen
//     exactly once per unit with no cross-CTA traffic.
//   * Persistent grid (one 256-thread CTA per SM).  Each head's 64 KiB fp32
//     state tile is streamed HBM -> SMEM by the TMA engine (cp.async.bulk,
//     mbarrier completion) through a 3-stage ring, so the next tiles are in
//     flight while the current one is reduced and written back.
//   * One read and one write of the state: r = S^T k and S^T q are reduced in a
//     single sweep of SMEM; o is rebuilt as decay*S^T q + d (k.q) so the update
//     and the output need no second reduction; the updated tile is stored with
//     16-byte coalesced st.global.v4 (512 contiguous bytes per warp row).
#include <algorithm>

#include "ria_capi_internal.h"
#include "ria_common.cuh"

namespace {

constexpr int kHv = 32;
constexpr int kHk = 16;
constexpr int kD = 128;
constexpr int kConvDim = 8192;
constexpr int kKeyDim = 2048;
constexpr int kValDim = 4096;
constexpr int kThreads = 256;
constexpr int kStages = 3;
constexpr int kTileFloats = kD * kD;
constexpr uint32_t kTileBytes = kTileFloats * 4;
constexpr int kCopyChunks = 8;  // bulk copies per tile (8 KiB each)

struct GdnParams {
  const __nv_bfloat16* mixed;
  int64_t mixed_stride;
  const __nv_bfloat16* z;
  int64_t z_stride;
  const __nv_bfloat16* bgate;
  int64_t b_stride;
  const __nv_bfloat16* agate;
  int64_t a_stride;
  const __nv_bfloat16* conv_w;
  const float* a_log;
  const float* dt_bias;
  const float* norm_w;
  __nv_bfloat16* conv_state;
  float* rec_state;
  const int32_t* slots;
  __nv_bfloat16* out;
  int64_t out_stride;
  int batch;
  int num_slots;
  unsigned int* err;
};

// Shared-memory map (bytes).
constexpr int kOffStage = 0;
constexpr int kOffRed = kOffStage + kStages * kTileBytes;  // [8 warps][2][128] f32
constexpr int kOffQ = kOffRed + 8 * 2 * kD * 4;            // [128] f32
constexpr int kOffK = kOffQ + kD * 4;                      // [128] f32
constexpr int kOffV = kOffK + kD * 4;                      // [2][128] f32
constexpr int kOffDelta = kOffV + 2 * kD * 4;              // [128] f32
constexpr int kOffScal = kOffDelta + kD * 4;               // [32] f32
constexpr int kOffWred = kOffScal + 32 * 4;                // [8][4] f32
constexpr int kOffBar = kOffWred + 32 * 4;                 // kStages x u64
constexpr int kSmemBytes = kOffBar + kStages * 8;

// scal[] slots
constexpr int kSBeta = 0;    // [2]
constexpr int kSDecay = 2;   // [2]

__device__ __forceinline__ float silu_bf16(float acc) {
  // conv1d output and SiLU both materialise in bf16 in the reference.
  float y = bf16_round(acc);
  return bf16_round(y / (1.0f + expf(-y)));
}

__device__ __forceinline__ float conv_channel(const GdnParams& p, int b, int slot, bool write, int ch) {
  const __nv_bfloat16* st = p.conv_state + (static_cast<int64_t>(slot) * kConvDim + ch) * 4;
  uint2 sraw = *reinterpret_cast<const uint2*>(st);
  uint2 wraw = *reinterpret_cast<const uint2*>(p.conv_w + static_cast<int64_t>(ch) * 4);
  __nv_bfloat16 x = p.mixed[static_cast<int64_t>(b) * p.mixed_stride + ch];
  const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&sraw);
  const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wraw);
  float2 s01 = __bfloat1622float2(s2[0]);
  float2 s23 = __bfloat1622float2(s2[1]);
  float2 w01 = __bfloat1622float2(w2[0]);
  float2 w23 = __bfloat1622float2(w2[1]);
  float xf = __bfloat162float(x);
  // history = [s0 s1 s2 s3 x]; last output reads history[1..4].
  float acc = w01.x * s01.y;
  acc = fmaf(w01.y, s23.x, acc);
  acc = fmaf(w23.x, s23.y, acc);
  acc = fmaf(w23.y, xf, acc);
  // new state = [s1 s2 s3 x]
  __nv_bfloat162 n0 = __halves2bfloat162(s2[0].y, s2[1].x);
  __nv_bfloat162 n1 = __halves2bfloat162(s2[1].y, x);
  uint2 nraw;
  nraw.x = *reinterpret_cast<uint32_t*>(&n0);
  nraw.y = *reinterpret_cast<uint32_t*>(&n1);
  if (write) *reinterpret_cast<uint2*>(const_cast<__nv_bfloat16*>(st)) = nraw;
  return silu_bf16(acc);
}

__device__ __forceinline__ float softplus_torch(float x) {
  // torch.nn.functional.softplus, beta=1, threshold=20.
  return x > 20.0f ? x : log1pf(expf(x));
}

__global__ void __launch_bounds__(kThreads, 1) gdn_decode_kernel(const GdnParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  float* stage = reinterpret_cast<float*>(smem + kOffStage);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* qs = reinterpret_cast<float*>(smem + kOffQ);
  float* ks = reinterpret_cast<float*>(smem + kOffK);
  float* vs = reinterpret_cast<float*>(smem + kOffV);
  float* ds = reinterpret_cast<float*>(smem + kOffDelta);
  float* scal = reinterpret_cast<float*>(smem + kOffScal);
  float* wred = reinterpret_cast<float*>(smem + kOffWred);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int units = p.batch * kHk;
  if (static_cast<int>(blockIdx.x) >= units) return;
  const int my_units = (units - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1;
  const int my_tiles = 2 * my_units;

  auto tile_unit = [&](int n) { return static_cast<int>(blockIdx.x) + (n >> 1) * static_cast<int>(gridDim.x); };
  // Out-of-range slots read slot 0 (always mapped) and skip every write; the
  // error word records the bad entry.
  auto slot_of = [&](int b) {
    const int s = p.slots ? p.slots[b] : b;
    return (s >= 0 && s < p.num_slots) ? s : 0;
  };
  auto slot_ok = [&](int b) {
    const int s = p.slots ? p.slots[b] : b;
    return s >= 0 && s < p.num_slots;
  };

  // Producer: lanes 0..7 of warp 0 each issue one 8 KiB slice of the tile.
  auto issue = [&](int n) {
    const int u = tile_unit(n);
    const int b = u / kHk;
    const int h = 2 * (u % kHk) + (n & 1);
    const int s = n % kStages;
    const float* src = p.rec_state + (static_cast<int64_t>(slot_of(b)) * kHv + h) * kTileFloats;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], kTileBytes);
    __syncwarp();
    if (lane < kCopyChunks) {
      constexpr int chunk_floats = kTileFloats / kCopyChunks;
      bulk_g2s(stage + s * kTileFloats + lane * chunk_floats, src + lane * chunk_floats, kTileBytes / kCopyChunks,
               &full[s]);
    }
  };

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) {
    for (int n = 0; n < kStages && n < my_tiles; ++n) issue(n);
  }

  const int row0 = warp * 16;  // rows of S owned by this warp (k index)
  float kq = 0.f;

  for (int n = 0; n < my_tiles; ++n) {
    const int u = tile_unit(n);
    const int b = u / kHk;
    const int j = u % kHk;
    const int hp = n & 1;  // 0: head 2j, 1: head 2j+1
    const int h = 2 * j + hp;
    const int slot = slot_of(b);
    const bool wr = slot_ok(b);
    if (!wr && hp == 0 && tid == 0) ria_set_error(p.err, RIA_DEVERR_BAD_SLOT);

    if (hp == 0) {
      // ---- per-unit prologue: conv + SiLU for 128 q, 128 k and 256 v channels,
      // L2 norms, gates for both value heads.
      const int ch_qk = (tid < 128) ? (j * kD + tid) : (kKeyDim + j * kD + (tid - 128));
      const float yqk = conv_channel(p, b, slot, wr, ch_qk);
      const float yv = conv_channel(p, b, slot, wr, 2 * kKeyDim + j * 2 * kD + tid);
      vs[tid] = yv;
      if (tid < 128) qs[tid] = yqk; else ks[tid - 128] = yqk;
      if (tid < 2) {
        const int hh = 2 * j + tid;
        const float bb = __bfloat162float(p.bgate[static_cast<int64_t>(b) * p.b_stride + hh]);
        const float aa = __bfloat162float(p.agate[static_cast<int64_t>(b) * p.a_stride + hh]);
        const float beta = 1.0f / (1.0f + expf(-bb));
        const float g = -expf(p.a_log[hh]) * softplus_torch(aa + p.dt_bias[hh]);
        scal[kSBeta + tid] = beta;
        scal[kSDecay + tid] = expf(g);
      }
      __syncthreads();
      if (tid < 128) {
        const float qv = qs[tid], kv = ks[tid];
        float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv), sqk = warp_sum(qv * kv);
        if (lane == 0) {
          wred[warp * 4 + 0] = sq;
          wred[warp * 4 + 1] = sk;
          wred[warp * 4 + 2] = sqk;
        }
      }
      __syncthreads();
      {
        float sq = 0.f, sk = 0.f, sqk = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          sq += wred[w * 4 + 0];
          sk += wred[w * 4 + 1];
          sqk += wred[w * 4 + 2];
        }
        const float rq = rsqrtf(sq + 1e-6f);
        const float rk = rsqrtf(sk + 1e-6f);
        const float qscale = 0.08838834764831845f;  // 128 ** -0.5
        kq = sqk * rq * rk * qscale;
        __syncthreads();  // everyone has read qs/ks raw values
        if (tid < 128) {
          qs[tid] = qs[tid] * rq * qscale;
          ks[tid] = ks[tid] * rk;
        }
      }
      __syncthreads();
    }

    // ---- wait for this tile
    const int s = n % kStages;
    mbar_wait_bounded(&full[s], (n / kStages) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_GDN);
    const float* tile = stage + s * kTileFloats;
    const float decay = scal[kSDecay + hp];
    const float beta = scal[kSBeta + hp];

    // ---- phase 1: partial S^T k and S^T q over this warp's 16 rows
    float4 racc = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 oacc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const int row = row0 + r;
      const float4 sv = reinterpret_cast<const float4*>(tile + row * kD)[lane];
      const float kk = ks[row];
      const float qq = qs[row];
      racc.x = fmaf(sv.x, kk, racc.x);
      racc.y = fmaf(sv.y, kk, racc.y);
      racc.z = fmaf(sv.z, kk, racc.z);
      racc.w = fmaf(sv.w, kk, racc.w);
      oacc.x = fmaf(sv.x, qq, oacc.x);
      oacc.y = fmaf(sv.y, qq, oacc.y);
      oacc.z = fmaf(sv.z, qq, oacc.z);
      oacc.w = fmaf(sv.w, qq, oacc.w);
    }
    reinterpret_cast<float4*>(red + (warp * 2 + 0) * kD)[lane] = racc;
    reinterpret_cast<float4*>(red + (warp * 2 + 1) * kD)[lane] = oacc;
    __syncthreads();

    // ---- reduce over the 8 warps: delta and the head output
    float o = 0.f;
    if (tid < kD) {
      float rr = 0.f, oo = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        rr += red[(w * 2 + 0) * kD + tid];
        oo += red[(w * 2 + 1) * kD + tid];
      }
      const float delta = beta * (vs[hp * kD + tid] - decay * rr);
      o = fmaf(decay, oo, delta * kq);
      ds[tid] = delta;
      const float so = warp_sum(o * o);
      if (lane == 0) wred[16 + warp] = so;
    }
    __syncthreads();

    // ---- epilogue: gated RMSNorm -> bf16 output row
    if (tid < kD) {
      const float ss = wred[16] + wred[17] + wred[18] + wred[19];
      const float on = o * rsqrtf(ss * (1.0f / kD) + 1e-6f);
      const float zz = __bfloat162float(p.z[static_cast<int64_t>(b) * p.z_stride + h * kD + tid]);
      const float gate = zz / (1.0f + expf(-zz));
      if (wr)
        p.out[static_cast<int64_t>(b) * p.out_stride + h * kD + tid] = __float2bfloat16_rn(p.norm_w[tid] * on * gate);
    }

    // ---- phase 2: S' = decay*S + k d^T, streamed back to HBM
    {
      float* dst = p.rec_state + (static_cast<int64_t>(slot) * kHv + h) * kTileFloats;
      const float4 d4 = reinterpret_cast<const float4*>(ds)[lane];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int row = row0 + r;
        const float4 sv = reinterpret_cast<const float4*>(tile + row * kD)[lane];
        const float kk = ks[row];
        float4 nv;
        nv.x = fmaf(decay, sv.x, kk * d4.x);
        nv.y = fmaf(decay, sv.y, kk * d4.y);
        nv.z = fmaf(decay, sv.z, kk * d4.z);
        nv.w = fmaf(decay, sv.w, kk * d4.w);
        if (wr) reinterpret_cast<float4*>(dst + row * kD)[lane] = nv;
      }
    }
    __syncthreads();  // stage s, ds and wred are free again
    if (warp == 0 && n + kStages < my_tiles) issue(n + kStages);
  }
}

}  // namespace

extern "C" int ria_gdn_decode_step(const void* mixed, int64_t mixed_stride, const void* z, int64_t z_stride,
                                   const void* b, int64_t b_stride, const void* a, int64_t a_stride,
                                   const void* conv_weight, const float* a_log, const float* dt_bias,
                                   const float* norm_weight, void* conv_state, float* rec_state, const int32_t* slots,
                                   int32_t num_slots, void* out, int64_t out_stride, int32_t batch,
                                   ria_stream_t stream) {
  if (batch < 0) return ria::fail(RIA_ERR_INVALID, "ria_gdn_decode_step: batch=%d < 0", batch);
  if (batch == 0) return RIA_OK;
  if (!mixed || !z || !b || !a || !conv_weight || !a_log || !dt_bias || !norm_weight || !conv_state || !rec_state ||
      !out)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_decode_step: null pointer argument");
  if (mixed_stride < kConvDim || z_stride < kValDim || b_stride < kHv || a_stride < kHv || out_stride < kValDim)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_decode_step: row stride smaller than the row width");
  if (!ria::aligned(rec_state, 16))
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_decode_step: rec_state must be 16-byte aligned");
  if (!ria::aligned(conv_state, 8) || !ria::aligned(conv_weight, 8))
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_decode_step: conv_state/conv_weight must be 8-byte aligned");
  if (!slots && num_slots < batch)
    return ria::fail(RIA_ERR_INVALID, "ria_gdn_decode_step: num_slots=%d < batch=%d", num_slots, batch);
  if (num_slots < 1) return ria::fail(RIA_ERR_INVALID, "ria_gdn_decode_step: num_slots=%d < 1", num_slots);

  GdnParams p;
  p.mixed = static_cast<const __nv_bfloat16*>(mixed);
  p.mixed_stride = mixed_stride;
  p.z = static_cast<const __nv_bfloat16*>(z);
  p.z_stride = z_stride;
  p.bgate = static_cast<const __nv_bfloat16*>(b);
  p.b_stride = b_stride;
  p.agate = static_cast<const __nv_bfloat16*>(a);
  p.a_stride = a_stride;
  p.conv_w = static_cast<const __nv_bfloat16*>(conv_weight);
  p.a_log = a_log;
  p.dt_bias = dt_bias;
  p.norm_w = norm_weight;
  p.conv_state = static_cast<__nv_bfloat16*>(conv_state);
  p.rec_state = rec_state;
  p.slots = slots;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.batch = batch;
  p.num_slots = num_slots;
  p.err = ria::device_error_word();

  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gdn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess)
      return ria::fail(RIA_ERR_CUDA, "ria_gdn_decode_step: smem attribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  const int units = batch * kHk;
  const int grid = std::min(units, ria::num_sms());
  gdn_decode_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(p);
  return ria::check_launch("ria_gdn_decode_step");
}
