// Self-test of the tcgen05 operand layouts used by the prefill kernels:
// D[128 x N] = A[128 x K] * B[K x N] with bf16 (or, with a_mode bit 2, fp16)
// operands staged in shared
// memory in K-major or MN-major 128-byte-swizzled tiles, or A held in TMEM
// (a_mode 2: bf16 pairs packed into 32-bit columns), fp32 accumulation in
// TMEM, and the result read back with tcgen05.ld.  Every address the MMA reads
// lies inside the two 32 KiB operand regions or the 256-column TMEM
// allocation of this CTA.
#include "ria_capi_internal.h"
#include "ria_common.cuh"
#include "tcgen05.cuh"

namespace {

constexpr int kM = 128;
constexpr int kRegion = 32768;

__device__ __forceinline__ uint16_t to16(float x, bool f16) {
  if (f16) return __half_as_ushort(__float2half_rn(x));
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

__global__ void __launch_bounds__(128, 1) umma_selftest_kernel(int a_mode, int b_mn, int n, int k, const float* A,
                                                               const float* B, float* D, unsigned int* err) {
  const bool f16 = (a_mode & 4) != 0;
  a_mode &= 3;
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sa = smem;
  unsigned char* sb = smem + kRegion;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * kRegion);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 2 * kRegion + 8);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;

  const bool a_mn = a_mode == 1, a_tmem = a_mode == 2;
  constexpr uint32_t kAcol = 128;  // TMEM column of A in mode 2 (D uses 0..127)
  // Stage A (kM x k) and B (k x n) as bf16 in the requested layouts.
  for (int idx = tid; idx < (a_tmem ? 0 : kM * k); idx += blockDim.x) {
    const int m = idx / k, kk = idx % k;
    const uint16_t v = to16(A[idx], f16);
    uint32_t off;
    if (!a_mn)  // rows = m, 64-wide K boxes of kM rows each
      off = (kk >> 6) * (kM * 128) + tc::sw128_off(m, kk & 63);
    else  // rows = k, 64-wide M blocks of k rows each
      off = (m >> 6) * (k * 128) + tc::sw128_off(kk, m & 63);
    *reinterpret_cast<uint16_t*>(sa + off) = v;
  }
  for (int idx = tid; idx < k * n; idx += blockDim.x) {
    const int kk = idx / n, nn = idx % n;
    const uint16_t v = to16(B[idx], f16);
    uint32_t off;
    if (!b_mn)  // rows = n, 64-wide K boxes of n rows each
      off = (kk >> 6) * (n * 128) + tc::sw128_off(nn, kk & 63);
    else  // rows = k, 64-wide N blocks of k rows each
      off = (nn >> 6) * (k * 128) + tc::sw128_off(kk, nn & 63);
    *reinterpret_cast<uint16_t*>(sb + off) = v;
  }
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, 256);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  if (a_tmem) {  // thread = row m = TMEM lane; 16 packed columns per store
    for (int j0 = 0; j0 < k / 2; j0 += 16) {
      uint32_t r[16];
      for (int j = 0; j < 16; ++j)
        r[j] = f16 ? pack_f16x2(A[tid * k + 2 * (j0 + j)], A[tid * k + 2 * (j0 + j) + 1])
                   : pack_bf16x2(A[tid * k + 2 * (j0 + j)], A[tid * k + 2 * (j0 + j) + 1]);
      tc::st16(tc::taddr(tbase, warp * 32, kAcol + j0), r);
    }
    tc::wait_st();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }

  if (tid == 0) {
    const uint32_t idesc = f16 ? tc::idesc_f16(kM, n, a_mn, b_mn) : tc::idesc_bf16(kM, n, a_mn, b_mn);
    const uint32_t abase = smem_u32(sa), bbase = smem_u32(sb);
    for (int ks = 0; ks < k / 16; ++ks) {
      uint64_t ad, bd;
      if (!a_mn)
        ad = tc::sdesc_sw128(abase + (ks >> 2) * (kM * 128) + (ks & 3) * 32, 16, 1024);
      else
        ad = tc::sdesc_sw128(abase + ks * 2048, k * 128, 1024);
      if (!b_mn)
        bd = tc::sdesc_sw128(bbase + (ks >> 2) * (n * 128) + (ks & 3) * 32, 16, 1024);
      else
        bd = tc::sdesc_sw128(bbase + ks * 2048, k * 128, 1024);
      if (a_tmem)
        tc::mma_bf16_ts(tbase, tbase + kAcol + ks * 8, bd, idesc, ks > 0);
      else
        tc::mma_bf16(tbase, ad, bd, idesc, ks > 0);
    }
    tc::commit(bar);
  }
  mbar_wait_bounded(bar, 0, err, RIA_DEVERR_MBAR_TIMEOUT_PREFILL);
  tc::fence_after_sync();

  const int row = tid;  // TMEM lane = D row
  for (int c0 = 0; c0 < n; c0 += 32) {
    float v[32];
    tc::ld32(tc::taddr(tbase, warp * 32, c0), v);
    tc::wait_ld();
    for (int i = 0; i < 32; ++i) D[row * n + c0 + i] = v[i];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

}  // namespace

extern "C" int ria_umma_selftest(int32_t a_mn_major, int32_t b_mn_major, int32_t n, int32_t k, const float* a,
                                 const float* b, float* d, ria_stream_t stream) {
  if ((n != 64 && n != 128) || (k != 64 && k != 128))
    return ria::fail(RIA_ERR_INVALID, "ria_umma_selftest: n and k must be 64 or 128");
  if ((a_mn_major & 3) > 2 || (a_mn_major & ~7) != 0)
    return ria::fail(RIA_ERR_INVALID, "ria_umma_selftest: a_mode must be 0, 1 or 2, plus 4 for fp16 operands");
  if (!a || !b || !d) return ria::fail(RIA_ERR_INVALID, "ria_umma_selftest: null pointer");
  const int smem = 2 * kRegion + 64;
  cudaError_t e = cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_umma_selftest: %s", cudaGetErrorString(e));
  umma_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(a_mn_major, b_mn_major != 0, n, k, a,
                                                                           b, d, ria::device_error_word());
  return ria::check_launch("ria_umma_selftest");
}
