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

}  // namespace ria
