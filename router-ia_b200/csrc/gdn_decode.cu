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
//   * Persistent grid, two 256-thread CTAs per SM.  Each head's 64 KiB fp32
//     state tile arrives as two 32 KiB halves by cp.async.bulk (the TMA engine,
//     mbarrier completion) through a 3-slot ring per CTA; warps 0-3 own rows
//     0-63 (first half), warps 4-7 rows 64-127.  Each thread moves its 16x4
//     slice of the tile into registers, so a slot is handed back to the TMA
//     right after the first barrier and the next halves stream in while the
//     tile is reduced and written back.
//   * One read and one write of the state: S^T k and S^T q are reduced in one
//     sweep (with the raw, un-normalised q and k; the L2-norm scales are applied
//     to the reduced sums), o is rebuilt as decay*S^T q + d (k.q), and the new
//     tile is stored from registers with 16-byte coalesced stores.
//   * The next unit's conv state, conv weights, projections and gates are
//     loaded into registers one unit ahead, so the per-unit prologue never waits
//     on global memory.  Two barriers per tile, two per unit.
//   * Small batches (16 key-head units per sequence leave SMs idle) use one
//     unit per (sequence, value head) instead: twice the CTAs, each with one
//     tile's chain; the two value heads of a key head both compute its q / k
//     conv and norms (the even one writes its conv state) and each writes the
//     conv state of its own v channels.  The two are one 2-CTA cluster, and a
//     cluster barrier separates both CTAs' reads of a unit's conv state from
//     its write.  The per-tile arithmetic is the same in both forms, so their
//     results are bit-identical.
#include <algorithm>
#include <mutex>

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
constexpr int kSlots = 3;                      // ring of half tiles
constexpr int kTileFloats = kD * kD;           // 16384
constexpr int kHalfFloats = kTileFloats / 2;   // 8192 (64 rows)
constexpr uint32_t kHalfBytes = kHalfFloats * 4;
constexpr int kCopyChunks = 4;                 // bulk copies per half tile (8 KiB each)

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
  int per_vhead;  // units are (sequence, value head) instead of (sequence, key head)
  unsigned int* err;
};

// Shared-memory map (bytes).
constexpr int kOffStage = 0;
constexpr int kOffRed = kOffStage + kSlots * kHalfBytes;  // [8 warps][2][128] f32
constexpr int kOffQ = kOffRed + 8 * 2 * kD * 4;           // [128] f32 raw q
constexpr int kOffK = kOffQ + kD * 4;                     // [128] f32 raw k
constexpr int kOffV = kOffK + kD * 4;                     // [2][128] f32
constexpr int kOffDelta = kOffV + 2 * kD * 4;             // [128] f32
constexpr int kOffScal = kOffDelta + kD * 4;              // [8] f32: beta[2], decay[2]
constexpr int kOffWred = kOffScal + 8 * 4;                // [32] f32
constexpr int kOffBar = kOffWred + 32 * 4;                // kSlots x u64
constexpr int kSmemBytes = kOffBar + kSlots * 8;

// Global inputs of one unit, loaded one unit ahead.
struct Prefetch {
  uint2 st_qk, w_qk, st_v, w_v;  // conv state / weights of this thread's two channels
  __nv_bfloat16 x_qk, x_v;       // projection outputs of those channels
  __nv_bfloat16 z0, z1;          // z of value heads 2j, 2j+1 (threads < 128)
  __nv_bfloat16 bb, aa;          // b, a of value head 2j + tid (threads < 2)
  float a_log, dt_bias;
};

__device__ __forceinline__ float softplus_torch(float x) {
  // torch.nn.functional.softplus, beta=1, threshold=20.
  return x > 20.0f ? x : log1pf(expf(x));
}

// Causal conv over history [s0 s1 s2 s3 x] (last output reads s1..x), then the
// bf16 conv output and bf16 SiLU of the reference.  Returns y; writes the new
// state [s1 s2 s3 x] to *st when `write`.
__device__ __forceinline__ float conv_silu(uint2 sraw, uint2 wraw, __nv_bfloat16 x, __nv_bfloat16* st, bool write) {
  const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&sraw);
  const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wraw);
  const float2 s01 = __bfloat1622float2(s2[0]);
  const float2 s23 = __bfloat1622float2(s2[1]);
  const float2 w01 = __bfloat1622float2(w2[0]);
  const float2 w23 = __bfloat1622float2(w2[1]);
  float acc = w01.x * s01.y;
  acc = fmaf(w01.y, s23.x, acc);
  acc = fmaf(w23.x, s23.y, acc);
  acc = fmaf(w23.y, __bfloat162float(x), acc);
  if (write) {
    __nv_bfloat162 n0 = __halves2bfloat162(s2[0].y, s2[1].x);
    __nv_bfloat162 n1 = __halves2bfloat162(s2[1].y, x);
    uint2 nraw;
    nraw.x = *reinterpret_cast<uint32_t*>(&n0);
    nraw.y = *reinterpret_cast<uint32_t*>(&n1);
    *reinterpret_cast<uint2*>(st) = nraw;
  }
  const float y = bf16_round(acc);
  return bf16_round(y / (1.0f + expf(-y)));
}

__global__ void __launch_bounds__(kThreads, 2) gdn_decode_kernel(const GdnParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  pdl_wait();
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
  const int nt = p.per_vhead ? 1 : 2;  // tiles (value heads) per unit
  const int units = p.batch * kHk * (p.per_vhead ? 2 : 1);
  if (static_cast<int>(blockIdx.x) >= units) return;
  const int my_units = (units - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1;
  const int my_halves = 2 * nt * my_units;  // nt tiles x 2 halves per unit
  // unit -> sequence, key head, first value head offset (0 or 1) within the key head
  auto unit_b = [&](int u) { return p.per_vhead ? u / (2 * kHk) : u / kHk; };
  auto unit_j = [&](int u) { return p.per_vhead ? (u % (2 * kHk)) >> 1 : u % kHk; };
  auto unit_t0 = [&](int u) { return p.per_vhead ? u & 1 : 0; };

  auto unit_of = [&](int ui) { return static_cast<int>(blockIdx.x) + ui * static_cast<int>(gridDim.x); };
  // Out-of-range slots read slot 0 (always mapped) and skip every write; the
  // error word records the bad entry.
  auto raw_slot = [&](int b) { return p.slots ? p.slots[b] : b; };
  auto slot_of = [&](int b) {
    const int s = raw_slot(b);
    return (s >= 0 && s < p.num_slots) ? s : 0;
  };

  // Producer (warp 0): half tile jh -> ring slot jh % kSlots.
  auto issue = [&](int jh) {
    const int u = unit_of(jh / (2 * nt));
    const int b = unit_b(u);
    const int h = 2 * unit_j(u) + unit_t0(u) + ((jh >> 1) % nt);
    const int s = jh % kSlots;
    const float* src = p.rec_state + (static_cast<int64_t>(slot_of(b)) * kHv + h) * kTileFloats + (jh & 1) * kHalfFloats;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], kHalfBytes);
    __syncwarp();
    if (lane < kCopyChunks) {
      constexpr int chunk = kHalfFloats / kCopyChunks;
      bulk_g2s(stage + s * kHalfFloats + lane * chunk, src + lane * chunk, kHalfBytes / kCopyChunks, &full[s]);
    }
  };

  // Channels owned by this thread inside a unit: one of q/k, one of v.
  auto load_prefetch = [&](int ui, Prefetch& pf) {
    const int u = unit_of(ui);
    const int b = unit_b(u);
    const int j = unit_j(u);
    const int slot = slot_of(b);
    const int ch_qk = (tid < 128) ? (j * kD + tid) : (kKeyDim + j * kD + (tid - 128));
    const int ch_v = 2 * kKeyDim + j * 2 * kD + tid;
    const __nv_bfloat16* cs = p.conv_state + static_cast<int64_t>(slot) * kConvDim * 4;
    pf.st_qk = *reinterpret_cast<const uint2*>(cs + ch_qk * 4);
    pf.st_v = *reinterpret_cast<const uint2*>(cs + ch_v * 4);
    pf.w_qk = *reinterpret_cast<const uint2*>(p.conv_w + ch_qk * 4);
    pf.w_v = *reinterpret_cast<const uint2*>(p.conv_w + ch_v * 4);
    const __nv_bfloat16* mrow = p.mixed + static_cast<int64_t>(b) * p.mixed_stride;
    pf.x_qk = mrow[ch_qk];
    pf.x_v = mrow[ch_v];
    if (tid < 128) {
      const __nv_bfloat16* zrow = p.z + static_cast<int64_t>(b) * p.z_stride + 2 * j * kD + tid;
      pf.z0 = zrow[0];
      pf.z1 = zrow[kD];
    }
    if (tid < 2) {
      const int hh = 2 * j + tid;
      pf.bb = p.bgate[static_cast<int64_t>(b) * p.b_stride + hh];
      pf.aa = p.agate[static_cast<int64_t>(b) * p.a_stride + hh];
      pf.a_log = p.a_log[hh];
      pf.dt_bias = p.dt_bias[hh];
    }
  };

  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) {
    for (int jh = 0; jh < kSlots && jh < my_halves; ++jh) issue(jh);
  }

  Prefetch pf;
  load_prefetch(0, pf);

  const int half = warp >> 2;       // which half tile this warp reads
  const int lrow0 = (warp & 3) * 16;  // first row inside the half
  const int row0 = half * 64 + lrow0;  // first row of the tile (k index)

  for (int ui = 0; ui < my_units; ++ui) {
    const int u = unit_of(ui);
    const int b = unit_b(u);
    const int j = unit_j(u);
    const int t0 = unit_t0(u);
    const int slot = slot_of(b);
    const int rs = raw_slot(b);
    const bool wr = rs >= 0 && rs < p.num_slots;
    // conv-state writes: q / k channels by the even value head's unit, v
    // channels (threads 0-127: head 2j, 128-255: head 2j + 1) by their head's
    const bool wr_qk = wr && t0 == 0;
    const bool wr_v = wr && (!p.per_vhead || (tid >> 7) == t0);

    // ---- unit prologue from the prefetched registers
    if (p.per_vhead) {
      // both value heads' CTAs have read this unit's conv state (the loads
      // ordered before the release) before the even one overwrites it
      asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
    __syncthreads();  // previous unit's readers of qs/ks/vs/scal are done
    {
      __nv_bfloat16* cs = p.conv_state + static_cast<int64_t>(slot) * kConvDim * 4;
      const int ch_qk = (tid < 128) ? (j * kD + tid) : (kKeyDim + j * kD + (tid - 128));
      const int ch_v = 2 * kKeyDim + j * 2 * kD + tid;
      const float yqk = conv_silu(pf.st_qk, pf.w_qk, pf.x_qk, cs + ch_qk * 4, wr_qk);
      const float yv = conv_silu(pf.st_v, pf.w_v, pf.x_v, cs + ch_v * 4, wr_v);
      vs[tid] = yv;
      if (tid < 128) qs[tid] = yqk; else ks[tid - 128] = yqk;
      if (tid < 2) {
        const float bb = __bfloat162float(pf.bb);
        const float aa = __bfloat162float(pf.aa);
        scal[tid] = 1.0f / (1.0f + expf(-bb));
        scal[2 + tid] = expf(-expf(pf.a_log) * softplus_torch(aa + pf.dt_bias));
      }
      if (!wr && tid == 0) ria_set_error(p.err, RIA_DEVERR_BAD_SLOT);
    }
    const float z0 = (tid < 128) ? __bfloat162float(pf.z0) : 0.f;
    const float z1 = (tid < 128) ? __bfloat162float(pf.z1) : 0.f;
    if (ui + 1 < my_units) load_prefetch(ui + 1, pf);  // in flight during this unit
    __syncthreads();
    if (tid < 128) {
      const float qv = qs[tid], kv = ks[tid];
      const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv), sqk = warp_sum(qv * kv);
      if (lane == 0) {
        wred[warp * 4 + 0] = sq;
        wred[warp * 4 + 1] = sk;
        wred[warp * 4 + 2] = sqk;
      }
    }

    for (int tt = 0; tt < nt; ++tt) {
      const int t = t0 + tt;  // value head 2j + t
      const int n = nt * ui + tt;
      const int h = 2 * j + t;
      const int jh = 2 * n + half;
      const int s = jh % kSlots;
      mbar_wait_bounded(&full[s], (jh / kSlots) & 1, p.err, RIA_DEVERR_MBAR_TIMEOUT_GDN);
      const float* hs = stage + s * kHalfFloats;

      // ---- phase 1: this warp's 16 rows into registers; partial S^T k, S^T q
      float4 sreg[16];
      float4 racc = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 oacc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        sreg[r] = reinterpret_cast<const float4*>(hs + (lrow0 + r) * kD)[lane];
        const float kk = ks[row0 + r];
        const float qq = qs[row0 + r];
        racc.x = fmaf(sreg[r].x, kk, racc.x);
        racc.y = fmaf(sreg[r].y, kk, racc.y);
        racc.z = fmaf(sreg[r].z, kk, racc.z);
        racc.w = fmaf(sreg[r].w, kk, racc.w);
        oacc.x = fmaf(sreg[r].x, qq, oacc.x);
        oacc.y = fmaf(sreg[r].y, qq, oacc.y);
        oacc.z = fmaf(sreg[r].z, qq, oacc.z);
        oacc.w = fmaf(sreg[r].w, qq, oacc.w);
      }
      reinterpret_cast<float4*>(red + (warp * 2 + 0) * kD)[lane] = racc;
      reinterpret_cast<float4*>(red + (warp * 2 + 1) * kD)[lane] = oacc;
      __syncthreads();  // A: both halves of tile n are in registers
      if (warp == 0) {
        if (2 * n + kSlots < my_halves) issue(2 * n + kSlots);
        if (2 * n + 1 + kSlots < my_halves) issue(2 * n + 1 + kSlots);
      }

      // L2-norm scales from the prologue sums (every thread needs rk)
      float sq = 0.f, sk = 0.f, sqk = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        sq += wred[w * 4 + 0];
        sk += wred[w * 4 + 1];
        sqk += wred[w * 4 + 2];
      }
      const float qscale = 0.08838834764831845f;  // 128 ** -0.5
      const float rq = rsqrtf(sq + 1e-6f) * qscale;
      const float rk = rsqrtf(sk + 1e-6f);
      const float decay = scal[2 + t];

      // ---- reduce over the 8 warps: delta and the head output
      float o = 0.f;
      if (tid < kD) {
        float rr = 0.f, oo = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          rr += red[(w * 2 + 0) * kD + tid];
          oo += red[(w * 2 + 1) * kD + tid];
        }
        const float delta = scal[t] * (vs[t * kD + tid] - decay * (rr * rk));
        o = fmaf(decay, oo * rq, delta * (sqk * rq * rk));
        ds[tid] = delta;
        const float so = warp_sum(o * o);
        if (lane == 0) wred[16 + warp] = so;
      }
      __syncthreads();  // B

      // ---- phase 2: S' = decay*S + k d^T from registers to HBM
      {
        float* dst = p.rec_state + (static_cast<int64_t>(slot) * kHv + h) * kTileFloats;
        const float4 d4 = reinterpret_cast<const float4*>(ds)[lane];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const float kk = ks[row0 + r] * rk;
          float4 nv;
          nv.x = fmaf(decay, sreg[r].x, kk * d4.x);
          nv.y = fmaf(decay, sreg[r].y, kk * d4.y);
          nv.z = fmaf(decay, sreg[r].z, kk * d4.z);
          nv.w = fmaf(decay, sreg[r].w, kk * d4.w);
          if (wr) reinterpret_cast<float4*>(dst + (row0 + r) * kD)[lane] = nv;
        }
      }
      // ---- epilogue: gated RMSNorm -> bf16 output row
      if (tid < kD && wr) {
        const float ss = wred[16] + wred[17] + wred[18] + wred[19];
        const float on = o * rsqrtf(ss * (1.0f / kD) + 1e-6f);
        const float zz = t ? z1 : z0;
        const float gate = zz / (1.0f + expf(-zz));
        p.out[static_cast<int64_t>(b) * p.out_stride + h * kD + tid] = __float2bfloat16_rn(p.norm_w[tid] * on * gate);
      }
    }
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

  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static bool attr_set[64] = {false};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      cudaError_t e =
          cudaFuncSetAttribute(gdn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess)
        return ria::fail(RIA_ERR_CUDA, "ria_gdn_decode_step: smem attribute: %s", cudaGetErrorString(e));
      attr_set[dev] = true;
    }
  }
  // value-head units when the key-head units would leave SMs idle
  p.per_vhead = batch * kHk < ria::num_sms() ? 1 : 0;
  const int units = batch * kHk * (p.per_vhead ? 2 : 1);
  const int grid = std::min(units, 2 * ria::num_sms());  // even in the value-head form (units = 32 x batch)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.per_vhead ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, gdn_decode_kernel, p);
  if (le != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_gdn_decode_step: %s", cudaGetErrorString(le));
  return ria::check_launch("ria_gdn_decode_step");
}
