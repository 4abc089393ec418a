// sa_capi.cu — error plumbing, version and device-error word of the C ABI.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "sa_common.cuh"

#ifndef SA_VERSION_STRING
#define SA_VERSION_STRING "sparseattentioninfer_b200 0.1.0 (sm_100a)"
#endif

// First device-side error recorded by any kernel of this library (0 = none).
__device__ int32_t g_sa_device_error = 0;

static thread_local char t_last_error[512] = {0};

int sa_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int sa_cuda_check(cudaError_t e, const char* what) {
  return sa_fail(SA_ERR_CUDA, "%s failed: %s", what, cudaGetErrorString(e));
}

int sa_num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return n;
}

int32_t* sa_device_error_ptr() {
  // Resolved once per device: a host-side symbol is not a device address.
  static int32_t* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sa_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int32_t*>(p);
  }
  return ptrs[dev];
}

extern "C" const char* sa_version(void) { return SA_VERSION_STRING; }

extern "C" const char* sa_last_error(void) { return t_last_error; }

extern "C" int sa_device_error(int32_t* code) {
  if (!code) return sa_fail(SA_ERR_INVALID, "code is NULL");
  SA_CHECK_CUDA(cudaDeviceSynchronize());
  int32_t v = 0;
  SA_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_sa_device_error, sizeof(v)));
  const int32_t zero = 0;
  SA_CHECK_CUDA(cudaMemcpyToSymbol(g_sa_device_error, &zero, sizeof(zero)));
  *code = v;
  return SA_OK;
}
