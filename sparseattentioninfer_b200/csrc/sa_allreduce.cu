// sa_allreduce.cu — tensor-parallel all-reduce over NVLink peer memory, fused
// with the residual add and the next RMSNorm of the decoder layer.
//
// Each rank's row-parallel GEMM (o_proj or down_proj) writes its partial sum y_r
// into its own slot of a buffer that every rank has mapped (CUDA IPC). One
// kernel then, per CTA:
//   1. barrier: stores the call's epoch into every rank's flag word for
//      (this CTA, this rank) with a system-scope release, and waits (bounded)
//      until its own flag words from every rank reach that epoch (acquire);
//   2. reads y_0 .. y_{N-1} for its rows straight from the peers' memory
//      (plain loads over NVLink, not cached in L1; every peer's 16 bytes are
//      requested before any is summed, so a thread waits for one NVLink round
//      trip, not one per peer), sums them in fp32 in rank order — the same
//      order on every rank, so all ranks hold identical residual streams —
//      and does x = bf16(x + sum), out = RMSNorm(x) * w. 512 threads cover a
//      4096-wide row in one pass.
// Calls alternate between two slots (o_proj, down_proj, o_proj, ...): a rank
// can only overwrite slot s after every peer entered the next call, i.e.
// finished reading s, so no exit barrier is needed. Epochs only grow, a peer
// may already show the next call's epoch, and waits test ">=".
//
// This replaces the NCCL all-reduce + separate add/RMSNorm for small (decode)
// messages; the tensor-parallel split itself follows Megatron (no counterpart
// in the reference, which runs on one device).
#include "sa_common.cuh"

namespace sa {

constexpr int kArMaxWorld = SA_AR_MAX_WORLD;
constexpr int kArThreads = 512;

struct ArParams {
  const __nv_bfloat16* data[kArMaxWorld];  // every rank's y for this call (slot already applied)
  uint32_t* flags[kArMaxWorld];            // every rank's flag words [max_ctas][kArMaxWorld]
  uint32_t* epoch;                         // this rank's per-CTA call counters [max_ctas]
  __nv_bfloat16* x;
  const __nv_bfloat16* w;
  __nv_bfloat16* out;
  int64_t rows, x_stride, out_stride;
  int n, rank, world;
  float eps;
  int32_t* err;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kArThreads) ar_add_rms_norm_kernel(const ArParams p) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_abort;
  __shared__ float s_red[kArThreads / 32];
  const int cta = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) {
    const uint32_t e = p.epoch[cta] + 1;
    p.epoch[cta] = e;
    s_epoch = e;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  if (tid < p.world) {
    __threadfence_system();  // this rank's y (written by the previous kernel) before the flag
    st_release_sys(p.flags[tid] + (int64_t)cta * kArMaxWorld + p.rank, e);
    const uint32_t* mine = p.flags[p.rank] + (int64_t)cta * kArMaxWorld + tid;
    const uint64_t t0 = globaltimer();
    uint32_t polls = 0;
    while ((int32_t)(ld_acquire_sys(mine) - e) < 0) {
      if ((++polls & 255u) == 0 && globaltimer() - t0 > SA_WAIT_LIMIT_NS) {
        record_error(p.err, SA_DEV_ERR_TIMEOUT);
        atomicExch(&s_abort, 1);
        break;
      }
    }
  }
  __syncthreads();
  if (s_abort) return;  // a peer never arrived: x is left unchanged, the error word is set

  for (int64_t r = cta; r < p.rows; r += gridDim.x) {
    __nv_bfloat16* xr = p.x + r * p.x_stride;
    float ss = 0.f;
    for (int i = tid * 8; i < p.n; i += kArThreads * 8) {
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
      uint4 v[kArMaxWorld];
#pragma unroll
      for (int q = 0; q < kArMaxWorld; ++q)
        if (q < p.world) v[q] = __ldcv(reinterpret_cast<const uint4*>(p.data[q] + r * p.n + i));
#pragma unroll
      for (int q = 0; q < kArMaxWorld; ++q) {
        if (q < p.world) {
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[q]);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(h[k]);
            acc[2 * k] += f.x;
            acc[2 * k + 1] += f.y;
          }
        }
      }
      uint4 xv = *reinterpret_cast<const uint4*>(xr + i);
      __nv_bfloat162* xh = reinterpret_cast<__nv_bfloat162*>(&xv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(xh[k]);
        xh[k] = __floats2bfloat162_rn(f.x + acc[2 * k], f.y + acc[2 * k + 1]);
        const float2 g = __bfloat1622float2(xh[k]);
        ss += g.x * g.x + g.y * g.y;
      }
      *reinterpret_cast<uint4*>(xr + i) = xv;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) s_red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kArThreads / 32; ++k) tot += s_red[k];
    __syncthreads();  // s_red is reused by the next row
    const float rs = rsqrtf(tot / p.n + p.eps);
    __nv_bfloat16* orow = p.out + r * p.out_stride;
    for (int i = tid * 8; i < p.n; i += kArThreads * 8) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + i);  // this thread's own stores
      const uint4 wv = *reinterpret_cast<const uint4*>(p.w + i);
      const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv);
      const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wv);
      uint4 ov;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = __bfloat1622float2(xh[k]), g = __bfloat1622float2(wh[k]);
        oh[k] = __floats2bfloat162_rn(a.x * rs * g.x, a.y * rs * g.y);
      }
      *reinterpret_cast<uint4*>(orow + i) = ov;
    }
  }
}

}  // namespace sa

using namespace sa;

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int sa_ar_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return sa_fail(SA_ERR_INVALID, "bad allocation request");
  *ptr = nullptr;
  SA_CHECK_CUDA(cudaMalloc(ptr, bytes));
  SA_CHECK_CUDA(cudaMemset(*ptr, 0, bytes));
  return SA_OK;
}

extern "C" int sa_ar_free(void* ptr) {
  if (ptr) SA_CHECK_CUDA(cudaFree(ptr));
  return SA_OK;
}

extern "C" int sa_ar_ipc_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  cudaIpcMemHandle_t h;
  SA_CHECK_CUDA(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle, &h, sizeof(h));
  return SA_OK;
}

extern "C" int sa_ar_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  SA_CHECK_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return SA_OK;
}

extern "C" int sa_ar_ipc_close(void* ptr) {
  if (ptr) SA_CHECK_CUDA(cudaIpcCloseMemHandle(ptr));
  return SA_OK;
}

extern "C" int sa_allreduce_add_rms_norm(const sa_ar_peers* peers, int64_t data_offset, void* x,
                                         const void* weight, void* out, int64_t rows, int32_t n,
                                         int64_t x_stride, int64_t out_stride, float eps, sa_stream_t stream) {
  if (!peers || !x || !weight || !out) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  const int world = peers->world;
  if (world < 1 || world > kArMaxWorld || peers->rank < 0 || peers->rank >= world)
    return sa_fail(SA_ERR_INVALID, "rank %d of world %d (at most %d ranks)", peers->rank, world, kArMaxWorld);
  if (rows <= 0 || n <= 0 || n % 8 || x_stride % 8 || out_stride % 8 || data_offset % 16 || !al16(x) ||
      !al16(weight) || !al16(out))
    return sa_fail(SA_ERR_INVALID, "rows=%lld n=%d: rows of a multiple of 8 elements on 16-byte boundaries",
                   (long long)rows, n);
  if (!peers->epoch || peers->max_ctas <= 0) return sa_fail(SA_ERR_INVALID, "no epoch counters");
  ArParams p;
  memset(&p, 0, sizeof(p));
  for (int q = 0; q < world; ++q) {
    if (!peers->data[q] || !peers->flags[q]) return sa_fail(SA_ERR_INVALID, "rank %d buffers missing", q);
    p.data[q] = reinterpret_cast<const __nv_bfloat16*>(static_cast<const char*>(peers->data[q]) + data_offset);
    p.flags[q] = peers->flags[q];
  }
  p.epoch = peers->epoch;
  p.x = static_cast<__nv_bfloat16*>(x);
  p.w = static_cast<const __nv_bfloat16*>(weight);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.rows = rows;
  p.x_stride = x_stride;
  p.out_stride = out_stride;
  p.n = n;
  p.rank = peers->rank;
  p.world = world;
  p.eps = eps;
  p.err = sa_device_error_ptr();
  const int64_t grid = rows < peers->max_ctas ? rows : peers->max_ctas;
  ar_add_rms_norm_kernel<<<(unsigned)grid, kArThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}
