// C-ABI plumbing shared by every entry point: status codes, the per-thread
// error string, the device error word and small device-property caches.
#include "ria_capi_internal.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

// The device error word (one per device, lives as long as the module).
static __device__ unsigned int g_ria_device_error = 0;

namespace ria {

static thread_local char t_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RIA_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return RIA_OK;
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static std::mutex mu;
  static int cache[64] = {0};
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

unsigned int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  static std::mutex mu;
  static unsigned int* cache[64] = {nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_ria_device_error) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cache[dev] = static_cast<unsigned int*>(ptr);
  }
  return cache[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_bf16_sw128_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box) {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
      void* ptr = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
          q == cudaDriverEntryPointSuccess)
        fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  }
  if (!fn) return fail(RIA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  if (rank < 1 || rank > 5) return fail(RIA_ERR_INVALID, "tensor map rank %d", rank);
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RIA_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return RIA_OK;
}

}  // namespace ria

extern "C" {

const char* ria_last_error_string(void) { return ria::t_last_error; }

int ria_abi_version(void) { return RIA_ABI_VERSION; }

int ria_device_error(int clear, unsigned int* code_out) {
  unsigned int code = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&code, g_ria_device_error, sizeof(code));
  if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_device_error: %s", cudaGetErrorString(e));
  if (clear && code != 0) {
    unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_ria_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return ria::fail(RIA_ERR_CUDA, "ria_device_error clear: %s", cudaGetErrorString(e));
  }
  if (code_out) *code_out = code;
  return RIA_OK;
}

}  // extern "C"
