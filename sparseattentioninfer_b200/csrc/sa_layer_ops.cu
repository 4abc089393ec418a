// sa_layer_ops.cu — the memory-bound decoder-layer steps around the attention
// kernels, each one launch:
//
// * sa_qk_norm_rope_append: per-head RMSNorm of q and k, rotate-half RoPE, and
//   the KV-cache append, from the fused q/k/v projection output. Replaces the
//   hook's q_norm / k_norm / apply_rotary_pos_emb / cache.update sequence
//   (sparse_llm/qwen3/integrations/modeling_sparse_qwen3.py:211-231), which is
//   a dozen elementwise launches plus a concatenating cache.
// * sa_add_rms_norm: residual add followed by the next RMSNorm (Qwen3RMSNorm
//   after each sub-block of the decoder layer).
// * sa_silu_mul: the SwiGLU activation silu(gate) * up over the fused
//   gate/up projection output (Qwen3MLP).
// * sa_linear_m8: the decoder's projections for at most 8 tokens (decode),
//   optionally with the SwiGLU activation fused into the gate/up projection.
//
// All arithmetic is fp32 with one bf16 rounding per stored value; the residual
// stream is stored in bf16 after each add, as the model keeps it.
#include "sa_common.cuh"

namespace sa {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int E>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, float (&x)[E]) {
  static_assert(E == 2 || E == 4, "2 or 4 elements per lane");
  if constexpr (E == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(b); x[3] = __high2float(b);
  } else {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(p);
    x[0] = __low2float(a); x[1] = __high2float(a);
  }
}

template <int E>
__device__ __forceinline__ void store_bf16(__nv_bfloat16* p, const float (&x)[E]) {
  if constexpr (E == 4) {
    uint2 u;
    *reinterpret_cast<__nv_bfloat162*>(&u.x) = __floats2bfloat162_rn(x[0], x[1]);
    *reinterpret_cast<__nv_bfloat162*>(&u.y) = __floats2bfloat162_rn(x[2], x[3]);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(x[0], x[1]);
  }
}

// One warp per (b, t, head) row of D = 32*E elements; lane l holds elements
// [E*l, E*l + E). Rotate-half pairs element d with d +- D/2, which sits in lane
// l ^ 16 at the same slot.
template <int E>
__global__ void __launch_bounds__(256) qk_norm_rope_append_kernel(sa_qkv_prologue_args a, int32_t* err) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int heads = a.Hq + 2 * a.Hkv;
  const int64_t rows = (int64_t)a.B * a.T * heads;
  if (row >= rows) return;
  const int j = (int)(row % heads);
  const int64_t bt = row / heads;
  const int t = (int)(bt % a.T), b = (int)(bt / a.T);
  const int pos0 = a.pos_dev ? __ldg(a.pos_dev) : a.pos;
  const int pos = pos0 + t;
  if (pos < 0 || pos >= a.capacity) {
    if (lane == 0) record_error(err, SA_DEV_ERR_INDEX);
    return;
  }
  const __nv_bfloat16* src =
      reinterpret_cast<const __nv_bfloat16*>(a.qkv) + (int64_t)b * a.qkv_sb + (int64_t)t * a.qkv_st + (int64_t)j * D;
  float x[E];
  load_bf16<E>(src + E * lane, x);
  if (j >= a.Hq + a.Hkv) {  // v: append as is
    const int h = j - a.Hq - a.Hkv;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.v_cache) + (int64_t)b * a.v_strides[0] +
                         (int64_t)h * a.v_strides[1] + (int64_t)pos * a.v_strides[2];
    store_bf16<E>(dst + E * lane, x);
    return;
  }
  const bool is_q = j < a.Hq;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss += x[e] * x[e];
  const float r = rsqrtf(warp_sum(ss) / D + a.eps);
  float w[E], c[E], s[E];
  load_bf16<E>(reinterpret_cast<const __nv_bfloat16*>(is_q ? a.q_weight : a.k_weight) + E * lane, w);
  load_bf16<E>(reinterpret_cast<const __nv_bfloat16*>(a.cos) + (int64_t)pos * D + E * lane, c);
  load_bf16<E>(reinterpret_cast<const __nv_bfloat16*>(a.sin) + (int64_t)pos * D + E * lane, s);
  float y[E], o[E];
#pragma unroll
  for (int e = 0; e < E; ++e) y[e] = x[e] * r * w[e];
  const float sign = lane < 16 ? -1.f : 1.f;  // first half: -x2 * sin; second half: +x1 * sin
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[e], 16);
    o[e] = y[e] * c[e] + sign * partner * s[e];
  }
  __nv_bfloat16* dst;
  if (is_q) {
    dst = reinterpret_cast<__nv_bfloat16*>(a.q_out) + (int64_t)b * a.q_strides[0] + (int64_t)j * a.q_strides[1] +
          (int64_t)t * a.q_strides[2];
  } else {
    dst = reinterpret_cast<__nv_bfloat16*>(a.k_cache) + (int64_t)b * a.k_strides[0] +
          (int64_t)(j - a.Hq) * a.k_strides[1] + (int64_t)pos * a.k_strides[2];
  }
  store_bf16<E>(dst + E * lane, o);
}

// One CTA per row: x = bf16(x + y); out = bf16(x * rsqrt(mean(x^2) + eps) * w).
// n % 8 == 0; rows 16-byte aligned.
__global__ void __launch_bounds__(256) add_rms_norm_kernel(__nv_bfloat16* __restrict__ x, const __nv_bfloat16* y,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           __nv_bfloat16* __restrict__ out, int n,
                                                           int64_t x_stride, int64_t y_stride, int64_t o_stride,
                                                           float eps) {
  __shared__ float s_red[8];
  const int64_t r = blockIdx.x;
  __nv_bfloat16* xr = x + r * x_stride;
  const __nv_bfloat16* yr = y ? y + r * y_stride : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < n; i += blockDim.x * 8) {
    uint4 xv = *reinterpret_cast<const uint4*>(xr + i);
    if (yr) {
      const uint4 yv = *reinterpret_cast<const uint4*>(yr + i);
      __nv_bfloat162* xp = reinterpret_cast<__nv_bfloat162*>(&xv);
      const __nv_bfloat162* yp = reinterpret_cast<const __nv_bfloat162*>(&yv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = __bfloat1622float2(xp[k]), b = __bfloat1622float2(yp[k]);
        xp[k] = __floats2bfloat162_rn(a.x + b.x, a.y + b.y);
      }
      *reinterpret_cast<uint4*>(xr + i) = xv;
    }
    const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = __bfloat1622float2(xp[k]);
      ss += a.x * a.x + a.y * a.y;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += s_red[k];
  const float rs = rsqrtf(tot / n + eps);
  __nv_bfloat16* orow = out + r * o_stride;
  for (int i = threadIdx.x * 8; i < n; i += blockDim.x * 8) {
    // re-read this thread's own stores (same thread, program order)
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + i);
    const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
    const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 ov;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = __bfloat1622float2(xp[k]), g = __bfloat1622float2(wp[k]);
      op[k] = __floats2bfloat162_rn(a.x * rs * g.x, a.y * rs * g.y);
    }
    *reinterpret_cast<uint4*>(orow + i) = ov;
  }
}

// out[r, i] = bf16(silu(g) * u), g = gu[r, i], u = gu[r, inter + i]; 8 elements per thread.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu,
                                                       __nv_bfloat16* __restrict__ out, int64_t rows, int inter,
                                                       int64_t gu_stride, int64_t o_stride) {
  const int per_row = inter / 8;
  const int64_t total = rows * per_row;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / per_row;
    const int i = (int)(v % per_row) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + r * gu_stride + i);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + r * gu_stride + inter + i);
    const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const __nv_bfloat162* up = reinterpret_cast<const __nv_bfloat162*>(&uv);
    uint4 ov;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 g = __bfloat1622float2(gp[k]), u = __bfloat1622float2(up[k]);
      const float a = g.x / (1.f + __expf(-g.x)), b = g.y / (1.f + __expf(-g.y));
      op[k] = __floats2bfloat162_rn(a * u.x, b * u.y);
    }
    *reinterpret_cast<uint4*>(out + r * o_stride + i) = ov;
  }
}

// ---------------------------------------------------------------------------
// Projections of M <= 8 tokens: out[m, n] = sum_k x[m, k] * W[n, k].
//
// At decode the weight matrix is the only large operand, so the kernel is a
// weight stream: one CTA per 16 weight rows, its 8 warps splitting K. A thread
// reads 16 contiguous bytes of two weight rows (g and g + 8) and of token row
// g of x per 32-wide K chunk, with eight chunks (GLU: four, for twice the
// rows) in flight before any math. The 32 K indices of a chunk are permuted
// consistently in A and B, which the sum over K does not see, so those 16-byte
// loads are exactly the mma.sync m16n8k16 fragments: weight rows are the
// M = 16 side, the 8 tokens the N = 8 side (tokens >= M read zeros). Warps
// are summed in a fixed order through shared memory (deterministic). With
// GLU the CTA also streams the matching up-projection rows (W rows N + n) and
// writes bf16(silu(g) * u) from the bf16-rounded g and u, the arithmetic of
// silu_mul_kernel.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int kLinWarps = 8;

template <bool GLU>
__global__ void __launch_bounds__(32 * kLinWarps) linear_m8_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                                                                   int64_t xs, const __nv_bfloat16* __restrict__ W,
                                                                   int64_t ws, int N, __nv_bfloat16* out,
                                                                   int64_t os) {
  constexpr int NT = GLU ? 2 : 1;  // weight tiles per CTA (gate, up)
  constexpr int U = GLU ? 4 : 8;   // K chunks in flight per thread
  __shared__ float red[NT][kLinWarps][16][9];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int n0 = blockIdx.x * 16;
  const int kw = K / kLinWarps;
  const int nch = kw / 32;
  const int64_t koff = (int64_t)warp * kw + 8 * c;
  const __nv_bfloat16* wr[NT][2];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    wr[t][0] = W + (int64_t)(n0 + t * N + g) * ws + koff;
    wr[t][1] = wr[t][0] + 8 * ws;
  }
  const bool xrow = g < M;
  const __nv_bfloat16* xp = x + (int64_t)(xrow ? g : 0) * xs + koff;
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
  for (int c0 = 0; c0 < nch; c0 += U) {
    uint4 wa[NT][U], wb[NT][U], xv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (c0 + u < nch) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          wa[t][u] = ld_stream16(wr[t][0] + (c0 + u) * 32);
          wb[t][u] = ld_stream16(wr[t][1] + (c0 + u) * 32);
        }
        xv[u] = xrow ? __ldg(reinterpret_cast<const uint4*>(xp + (c0 + u) * 32)) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (c0 + u < nch) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          mma_16816(acc[t], wa[t][u].x, wb[t][u].x, wa[t][u].y, wb[t][u].y, xv[u].x, xv[u].y);
          mma_16816(acc[t], wa[t][u].z, wb[t][u].z, wa[t][u].w, wb[t][u].w, xv[u].z, xv[u].w);
        }
      }
    }
  }
  // D fragment: acc[0..1] = rows g, tokens 2c, 2c+1; acc[2..3] = rows g + 8
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red[t][warp][g][2 * c] = acc[t][0];
    red[t][warp][g][2 * c + 1] = acc[t][1];
    red[t][warp][g + 8][2 * c] = acc[t][2];
    red[t][warp][g + 8][2 * c + 1] = acc[t][3];
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const int m = threadIdx.x >> 4, r = threadIdx.x & 15;
    if (m < M) {
      float sum[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        sum[t] = 0.f;
#pragma unroll
        for (int w = 0; w < kLinWarps; ++w) sum[t] += red[t][w][r][m];
      }
      float y;
      if constexpr (GLU) {
        const float gg = __bfloat162float(__float2bfloat16_rn(sum[0]));
        const float uu = __bfloat162float(__float2bfloat16_rn(sum[1]));
        y = gg / (1.f + __expf(-gg)) * uu;
      } else {
        y = sum[0];
      }
      out[(int64_t)m * os + n0 + r] = __float2bfloat16_rn(y);
    }
  }
}

}  // namespace sa

using namespace sa;

extern "C" int sa_linear_m8(const void* x, int32_t M, int32_t K, int64_t x_stride, const void* w, int32_t N,
                            int64_t w_stride, void* out, int64_t out_stride, int32_t glu, sa_stream_t stream) {
  if (!x || !w || !out) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  if (M < 1 || M > 8) return sa_fail(SA_ERR_UNSUPPORTED, "M=%d tokens (1..8)", M);
  if (K <= 0 || K % (32 * kLinWarps) || N <= 0 || N % 16)
    return sa_fail(SA_ERR_UNSUPPORTED, "K=%d (a multiple of %d), N=%d (a multiple of 16)", K, 32 * kLinWarps, N);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15u || x_stride % 8 || w_stride % 8 ||
      x_stride < K || w_stride < K || out_stride < N || (reinterpret_cast<uintptr_t>(out) & 1u))
    return sa_fail(SA_ERR_INVALID, "x and W rows must start on 16-byte boundaries (strides %% 8 == 0, >= K)");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  if (glu)
    linear_m8_kernel<true><<<N / 16, 32 * kLinWarps, 0, s>>>(xb, M, K, x_stride, wb, w_stride, N, ob, out_stride);
  else
    linear_m8_kernel<false><<<N / 16, 32 * kLinWarps, 0, s>>>(xb, M, K, x_stride, wb, w_stride, N, ob, out_stride);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int sa_qk_norm_rope_append(const sa_qkv_prologue_args* a, sa_stream_t stream) {
  if (!a) return sa_fail(SA_ERR_INVALID, "args is NULL");
  if (!a->qkv || !a->q_weight || !a->k_weight || !a->cos || !a->sin || !a->q_out || !a->k_cache || !a->v_cache)
    return sa_fail(SA_ERR_INVALID, "NULL pointer in prologue arguments");
  if (a->D != 64 && a->D != 128) return sa_fail(SA_ERR_UNSUPPORTED, "D=%d (64 or 128)", a->D);
  if (a->B <= 0 || a->T <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->Hq % a->Hkv || a->capacity <= 0)
    return sa_fail(SA_ERR_INVALID, "bad sizes B=%d T=%d Hq=%d Hkv=%d capacity=%d", a->B, a->T, a->Hq, a->Hkv,
                   a->capacity);
  if (!a->pos_dev && (a->pos < 0 || a->pos + a->T > a->capacity))
    return sa_fail(SA_ERR_INVALID, "positions [%d, %d) outside the cache capacity %d", a->pos, a->pos + a->T,
                   a->capacity);
  // every row starts on an 8-byte (D=128) / 4-byte (D=64) boundary for the vector loads
  const int64_t al = a->D == 128 ? 4 : 2;
  if ((a->qkv_sb | a->qkv_st | a->q_strides[0] | a->q_strides[1] | a->q_strides[2] | a->k_strides[0] |
       a->k_strides[1] | a->k_strides[2] | a->v_strides[0] | a->v_strides[1] | a->v_strides[2]) % al)
    return sa_fail(SA_ERR_INVALID, "strides must be multiples of %lld elements", (long long)al);
  const uintptr_t mis = (reinterpret_cast<uintptr_t>(a->qkv) | reinterpret_cast<uintptr_t>(a->q_weight) |
                         reinterpret_cast<uintptr_t>(a->k_weight) | reinterpret_cast<uintptr_t>(a->cos) |
                         reinterpret_cast<uintptr_t>(a->sin) | reinterpret_cast<uintptr_t>(a->q_out) |
                         reinterpret_cast<uintptr_t>(a->k_cache) | reinterpret_cast<uintptr_t>(a->v_cache)) &
                        (uintptr_t)(2 * al - 1);
  if (mis) return sa_fail(SA_ERR_INVALID, "pointers must be %lld-byte aligned", (long long)(2 * al));
  const int64_t rows = (int64_t)a->B * a->T * (a->Hq + 2 * a->Hkv);
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffff) return sa_fail(SA_ERR_INVALID, "too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a->D == 128)
    qk_norm_rope_append_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(*a, sa_device_error_ptr());
  else
    qk_norm_rope_append_kernel<2><<<(unsigned)blocks, 256, 0, s>>>(*a, sa_device_error_ptr());
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_add_rms_norm(void* x, const void* y, const void* weight, void* out, int64_t rows, int32_t n,
                               int64_t x_stride, int64_t y_stride, int64_t out_stride, float eps,
                               sa_stream_t stream) {
  if (!x || !weight || !out) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  if (rows <= 0 || rows > 0x7fffffff || n <= 0 || n % 8)
    return sa_fail(SA_ERR_INVALID, "rows=%lld n=%d (n a multiple of 8)", (long long)rows, n);
  if (!aligned16(x) || (y && !aligned16(y)) || !aligned16(weight) || !aligned16(out) || x_stride % 8 ||
      (y && y_stride % 8) || out_stride % 8)
    return sa_fail(SA_ERR_INVALID, "rows must start on 16-byte boundaries");
  add_rms_norm_kernel<<<(unsigned)rows, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y),
      static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out), n, x_stride, y_stride,
      out_stride, eps);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_silu_mul(const void* gate_up, void* out, int64_t rows, int32_t inter, int64_t gu_stride,
                           int64_t out_stride, sa_stream_t stream) {
  if (!gate_up || !out) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  if (rows <= 0 || inter <= 0 || inter % 8 || gu_stride % 8 || out_stride % 8 || !aligned16(gate_up) ||
      !aligned16(out))
    return sa_fail(SA_ERR_INVALID, "silu_mul needs 16-byte aligned rows and inter %% 8 == 0");
  const int64_t vec = rows * (inter / 8);
  const int64_t want = (vec + 255) / 256;
  const int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
  silu_mul_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), rows, inter, gu_stride,
      out_stride);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}
