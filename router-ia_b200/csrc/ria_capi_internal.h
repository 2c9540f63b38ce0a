// Host-side helpers shared by the C-ABI translation units.
#pragma once

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

}  // namespace ria
