// sa_topk.cu — data-dependent top-k attention (TopKPattern).
//
// The reference applies it in MaskedSdpaBackend (masked_sdpa.py:51-63): full
// scores q·k^T·scale, causal mask (bottom-right for decode), keep the top_k
// scores of each row (torch.topk), softmax over them, times V. The selection
// depends on every score of the row, so it cannot be a block-CSR schedule; the
// scores come from a library GEMM (fp32 accumulation) and this kernel does the
// rest of the row in one pass per CTA:
//   1. causal mask in place (keys past the row's absolute position -> -inf);
//   2. the k-th largest score by a 4-pass radix select (8 bits per pass) on
//      order-preserving unsigned keys, with per-CTA shared-memory histograms;
//   3. softmax over the scores >= that threshold and O = sum p_i v_i, gathering
//      only the selected rows of V (one warp per selected key, lanes over D).
// Ties exactly at a finite threshold are all kept (torch.topk keeps some of
// them); with continuous scores this does not occur. Rows whose valid keys are
// fewer than top_k keep them all, as torch.topk's extra -inf picks weigh 0.
#include "sa_common.cuh"

namespace sa {

constexpr int kTopkThreads = 256;

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct TopkParams {
  float* scores;            // [rows, T_k] fp32 (masked in place)
  int64_t s_row;            // row stride (elements)
  const __nv_bfloat16* v;   // [B, Hkv, T_k, D]
  int64_t v_sb, v_sh, v_st;
  void* out;                // [B, Hq, T_q, D] bf16 or fp32
  int64_t o_sb, o_sh, o_st;
  int out_f32;
  int B, Hkv, G, rows_per_head, t0, T_q, T_k, D, top_k;
};

// Row r of the score block = (b, kv head, g, t - t0) in that order (the layout
// of a [B, Hkv, G * rows_per_head, T_k] GEMM output).
__global__ void __launch_bounds__(kTopkThreads) topk_softmax_pv_kernel(const TopkParams p) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_need;
  __shared__ float s_max;
  __shared__ float s_red[kTopkThreads / 32];
  __shared__ float s_acc[kTopkThreads / 32][256];
  const int64_t r = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tl = (int)(r % p.rows_per_head);
  const int64_t rest = r / p.rows_per_head;
  const int g = (int)(rest % p.G);
  const int kvh = (int)((rest / p.G) % p.Hkv);
  const int b = (int)(rest / ((int64_t)p.G * p.Hkv));
  const int t = p.t0 + tl;
  const int q_abs = t + (p.T_k - p.T_q);
  float* srow = p.scores + r * p.s_row;

  // 1. causal mask + row max
  float mx = -INFINITY;
  for (int i = tid; i < p.T_k; i += kTopkThreads) {
    float s = srow[i];
    if (i > q_abs) {
      s = -INFINITY;
      srow[i] = s;
    }
    mx = fmaxf(mx, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  if (tid == 0) {
    s_prefix = 0u;
    s_need = (uint32_t)min(p.top_k, p.T_k);
  }
  __syncthreads();
  if (tid == 0) {
    float m = -INFINITY;
    for (int w = 0; w < kTopkThreads / 32; ++w) m = fmaxf(m, s_red[w]);
    s_max = m;
  }

  // 2. radix select: the largest key K such that #(key >= K) >= need
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t hi_mask = pass == 0 ? 0u : (0xffffffffu << (32 - 8 * pass));
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0u;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = tid; i < p.T_k; i += kTopkThreads) {
      const uint32_t k = fkey(srow[i]);
      if ((k & hi_mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t need = s_need, acc = 0u;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= need) break;
        acc += hist[d];
      }
      s_need = need - acc;  // still to take inside digit d
      s_prefix = prefix | ((uint32_t)d << shift);
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  const float m = s_max;
  const float m_use = m == -INFINITY ? 0.f : m;

  // 3. softmax over the selected keys and the gathered PV product
  const int D = p.D;
  const __nv_bfloat16* vbase = p.v + (int64_t)b * p.v_sb + (int64_t)kvh * p.v_sh;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  float lsum = 0.f;
  const int per_lane = D / 32;  // 2 (D=64) or 4 (D=128)
  for (int base = warp * 32; base < p.T_k; base += kTopkThreads) {
    const int i = base + lane;
    const float s = i < p.T_k ? srow[i] : -INFINITY;
    const bool sel = i < p.T_k && fkey(s) >= thr && s != -INFINITY;
    uint32_t bal = __ballot_sync(0xffffffffu, sel);
    while (bal) {
      const int src = __ffs(bal) - 1;
      bal &= bal - 1;
      const float ss = __shfl_sync(0xffffffffu, s, src);
      const float pv = __expf(ss - m_use);
      lsum += pv;  // every lane adds the same value; lane 0's copy is used
      const __nv_bfloat16* vr = vbase + (int64_t)(base + src) * p.v_st + lane * per_lane;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < per_lane) acc[e] += pv * __bfloat162float(vr[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (e < per_lane) s_acc[warp][lane * per_lane + e] = acc[e];
  if (lane == 0) s_red[warp] = lsum;
  __syncthreads();
  for (int d = tid; d < D; d += kTopkThreads) {
    float o = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kTopkThreads / 32; ++w) {
      o += s_acc[w][d];
      l += s_red[w];
    }
    const float val = l > 0.f ? o / l : 0.f;
    const int h = kvh * p.G + g;
    const int64_t off = (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)t * p.o_st + d;
    if (p.out_f32)
      static_cast<float*>(p.out)[off] = val;
    else
      static_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(val);
  }
}

}  // namespace sa

using namespace sa;

extern "C" int sa_topk_softmax_pv(const sa_topk_args* a, sa_stream_t stream) {
  if (!a || !a->scores || !a->v || !a->out) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  if (a->D != 64 && a->D != 128) return sa_fail(SA_ERR_UNSUPPORTED, "D=%d (64 or 128)", a->D);
  if (a->B <= 0 || a->Hkv <= 0 || a->G <= 0 || a->rows_per_head <= 0 || a->T_q <= 0 || a->T_k <= 0 ||
      a->top_k <= 0 || a->t0 < 0 || a->t0 + a->rows_per_head > a->T_q || a->T_q > a->T_k)
    return sa_fail(SA_ERR_INVALID, "topk: bad sizes (B=%d Hkv=%d G=%d rows=%d t0=%d T_q=%d T_k=%d k=%d)", a->B,
                   a->Hkv, a->G, a->rows_per_head, a->t0, a->T_q, a->T_k, a->top_k);
  if (a->s_row < a->T_k) return sa_fail(SA_ERR_INVALID, "topk: score row stride below T_k");
  TopkParams p;
  p.scores = static_cast<float*>(a->scores);
  p.s_row = a->s_row;
  p.v = static_cast<const __nv_bfloat16*>(a->v);
  p.v_sb = a->v_strides[0];
  p.v_sh = a->v_strides[1];
  p.v_st = a->v_strides[2];
  p.out = a->out;
  p.o_sb = a->o_strides[0];
  p.o_sh = a->o_strides[1];
  p.o_st = a->o_strides[2];
  p.out_f32 = a->out_f32;
  p.B = a->B;
  p.Hkv = a->Hkv;
  p.G = a->G;
  p.rows_per_head = a->rows_per_head;
  p.t0 = a->t0;
  p.T_q = a->T_q;
  p.T_k = a->T_k;
  p.D = a->D;
  p.top_k = a->top_k;
  const int64_t rows = (int64_t)a->B * a->Hkv * a->G * a->rows_per_head;
  if (rows > 0x7fffffff) return sa_fail(SA_ERR_INVALID, "topk: too many rows");
  topk_softmax_pv_kernel<<<(unsigned)rows, kTopkThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}
