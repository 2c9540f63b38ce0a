// Shared device helpers for the router-ia B200 attention library.
//
// Everything here is sm_100a inline PTX or plain CUDA: mbarrier-tracked bulk
// copies (the TMA engine), tensor-map tiled copies, ldmatrix/movmatrix and the
// bf16 mma.sync shape used by the decode kernels.  Every wait on an mbarrier is
// bounded: after RIA_SPIN_LIMIT polls the kernel records an error code in
// the device error word and carries on, so a lost copy can never hang the GPU.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#ifndef RIA_SPIN_LIMIT
#define RIA_SPIN_LIMIT (1u << 26)
#endif

// Kernels report failures into a device error word (0 = no error) whose
// address the host passes in as a kernel argument (ria::device_error_word()).
// atomicCAS keeps the first error; ria_device_error() reads and clears it.

enum RiaDeviceError : unsigned int {
  RIA_DEVERR_NONE = 0,
  RIA_DEVERR_MBAR_TIMEOUT_GDN = 1,
  RIA_DEVERR_MBAR_TIMEOUT_GQA = 2,
  RIA_DEVERR_BAD_BLOCK = 3,
  RIA_DEVERR_MBAR_TIMEOUT_CHUNK = 4,
  RIA_DEVERR_MBAR_TIMEOUT_PREFILL = 5,
  RIA_DEVERR_BAD_SLOT = 6,
  RIA_DEVERR_SPLIT_PLAN = 7,  // a sequence needs more KV splits than were launched
  RIA_DEVERR_MOE_WAIT = 8,    // the MoE down phase gave up waiting for a unit's gate/up tiles
};

__device__ __forceinline__ void ria_set_error(unsigned int* err, unsigned int code) {
  if (err) atomicCAS(err, 0u, code);
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialisation attribute (ria::launch_pdl) may be scheduled before
// the kernel ahead of it in the stream has fully drained: it must call
// pdl_wait() before it reads anything that kernel (or any earlier one) wrote
// and before its first global write.  pdl_wait() returns once the preceding
// kernel has completed and its writes are visible; it is a no-op for a normal
// launch.  No kernel here triggers its dependents early: on the batch-1
// decode chain an early trigger let the next kernel's CTAs sit beside the
// weight-streaming GEMVs and slowed the step by 8%, while launching without
// it gained 1.6%.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok;
}

// Bounded wait.  Returns true when the phase completed, false on timeout (the
// error word is set; the caller finishes its work on whatever is in smem and
// the host reports the failure).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned int* err,
                                                  unsigned int code) {
  for (uint32_t i = 0; i < RIA_SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  ria_set_error(err, code);
  return false;
}

// ---------------------------------------------------------------- bulk copies (TMA engine)
// 1-D bulk copy global -> shared, completion counted on an mbarrier.  Both
// addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled tensor copy global -> shared (no multicast).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int32_t c0, int32_t c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled tensor copy global -> shared (no multicast).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, int32_t c0, int32_t c1, int32_t c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(smem_dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled tensor store shared -> global (bulk-group completion; no
// multicast).  Coordinates must be non-negative; rows past the tensor end are
// clipped.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* smem_src, int32_t c0, int32_t c1,
                                             int32_t c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(tmap),
               "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(smem_src))
               : "memory");
}
// 2-D tiled tensor store shared -> global (bulk-group completion), same rules.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap),
               "r"(c0), "r"(c1), "r"(smem_u32(smem_src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the shared-memory sources of all committed bulk stores were read.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until all committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Generic-proxy global writes made by this thread become visible to later
// async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- warp-level matrix ops
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// D = A(16x16, row) * B(16x8, col) + D, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a tile written
// by TMA with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows, 1024-byte atoms).
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
