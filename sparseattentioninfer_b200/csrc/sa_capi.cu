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

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                      const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                      const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                      CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t get_encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(ptr);
  }
  return fn;
}

// 4-D bf16 map over [B, H, T, D] (innermost first: D, T, H, B), box (64, rows, 1, 1),
// SWIZZLE_128B, zero fill out of range.
int sa_make_map(CUtensorMap* m, const void* base, int B, int H, int T, int D,
                    const int64_t strides[3], int box_rows, const char* name) {
  PFN_encodeTiled_t enc = get_encode_fn();
  if (!enc) return sa_fail(SA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2,
                        (cuuint64_t)strides[0] * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, gstr, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return sa_fail(SA_ERR_INVALID, "tensor map for %s rejected (CUresult %d)", name, (int)r);
  return SA_OK;
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
