// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "ria_attention.h"

namespace ria {

// Records a printf-style message for ria_last_error_string() and returns code.
int fail(int code, const char* fmt, ...);
// Converts a pending launch error into RIA_ERR_CUDA.
int check_launch(const char* what);
// SM count of the current device (cached per device).
int num_sms();
bool aligned(const void* p, size_t a);
// Device address of the error word on the current device (nullptr if the
// symbol lookup failed; kernels then skip error reporting).
unsigned int* device_error_word();
// Tiled bf16 tensor map with 128-byte swizzle (no multicast users): `rank`
// dims (innermost first), byte strides of dims 1..rank-1, box extents.
int encode_bf16_sw128_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box);

// Launch `kernel` as a programmatic dependent of the previous kernel in the
// stream (it overlaps that kernel's tail; the kernel calls pdl_wait() before
// touching data).  Stream capture records the dependency as a programmatic
// graph edge.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace ria
