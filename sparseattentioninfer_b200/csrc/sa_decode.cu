// sa_decode.cu — split-KV block-sparse decode (one query token per sequence).
//
// Replaces the decode use of _universal_sparse_attn_kernel
// (kernels/triton/universal_sparse_attn.py:45-160 with Q_OFFSET = T_k, :84-89),
// which spends a 1-row query block per (b, q-head) and re-reads K/V per head.
// Here one CTA serves a (b, kv-head, split): it reads each retained KV block of
// the group once for all Hq/Hkv query heads. The reference draws different
// random blocks per query head (bigbird_pattern.py:23-41), so the CTA walks the
// sorted union of the group's CSR rows with a per-head membership mask.
// Memory path: 128-bit loads, D/8 lanes per key row, 4 rows in flight per lane
// for K and for V; statistics in fp32 (log2 domain). A second kernel merges the
// splits (log-sum-exp) and writes bf16.
#include <cstring>

#include "sa_common.cuh"

namespace sa {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kMaxUnion = 2048;
constexpr int kUnroll = 4;

struct DecodeParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_sb, q_sh, k_sb, k_sh, k_st, v_sb, v_sh, v_st;
  const int32_t* pairs;
  const int32_t* offsets;
  int32_t pairs_stride;
  int32_t B, Hq, Hkv, T_k, bs, n_split;
  float scale_log2;
  float* part_o;   // [B, Hq, n_split, D]
  float* part_ml;  // [B, Hq, n_split, 2]
  int32_t* err;
};

__device__ __forceinline__ void bf16x8_to_f32(const uint4 u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int D, int G>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(const DecodeParams p) {
  constexpr int LPK = D / 8;          // lanes per key row (16 B each)
  constexpr int KPW = 32 / LPK;       // key rows per warp instruction
  __shared__ int s_kb[kMaxUnion];
  __shared__ uint8_t s_mask[kMaxUnion];
  __shared__ int s_n;
  __shared__ float s_m[kDecWarps][G], s_l[kDecWarps][G];
  __shared__ float s_o[kDecWarps][G][D];

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h0 = kvh * G;

  // Union of the G query heads' rows (single thread; rows are short).
  if (threadIdx.x == 0) {
    int ptr[G], end[G];
    const int32_t* prs[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int32_t* off = p.offsets + (int64_t)(h0 + j) * 2;
      ptr[j] = off[0];
      end[j] = off[1];
      prs[j] = p.pairs + (int64_t)(h0 + j) * p.pairs_stride;
    }
    int n = 0;
    while (true) {
      int best = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < G; ++j)
        if (ptr[j] < end[j]) best = min(best, prs[j][ptr[j]]);
      if (best == 0x7fffffff) break;
      uint32_t m = 0;
#pragma unroll
      for (int j = 0; j < G; ++j)
        if (ptr[j] < end[j] && prs[j][ptr[j]] == best) {
          m |= 1u << j;
          ++ptr[j];
        }
      if (n >= kMaxUnion) {
        record_error(p.err, SA_DEV_ERR_INDEX);
        break;
      }
      if (best < 0) m = 0;  // malformed index: contributes nothing
      s_kb[n] = best < 0 ? 0 : best;
      s_mask[n] = (uint8_t)m;
      ++n;
    }
    s_n = n;
  }
  __syncthreads();
  const int U = s_n;
  const int e_begin = (int)(((int64_t)U * split) / p.n_split);
  const int e_end = (int)(((int64_t)U * (split + 1)) / p.n_split);
  const int nkeys = (e_end - e_begin) * p.bs;

  // q slice of this lane, pre-scaled into the log2 domain.
  const int dsl = (lane % LPK) * 8;
  const int kr = lane / LPK;
  float qf[G][8];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const uint4 u = *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.q_sb + (int64_t)(h0 + j) * p.q_sh + dsl);
    bf16x8_to_f32(u, qf[j]);
#pragma unroll
    for (int e = 0; e < 8; ++e) qf[j][e] *= p.scale_log2;
  }
  float m[G], l[G], o[G][8];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[j][e] = 0.f;
  }
  const __nv_bfloat16* kbase = p.k + (int64_t)b * p.k_sb + (int64_t)kvh * p.k_sh + dsl;
  const __nv_bfloat16* vbase = p.v + (int64_t)b * p.v_sb + (int64_t)kvh * p.v_sh + dsl;

  constexpr int kBatch = kUnroll * KPW;  // keys per warp batch
  for (int f0 = warp * kBatch; f0 < nkeys; f0 += kDecWarps * kBatch) {
    uint4 ku[kUnroll], vu[kUnroll];
    int key[kUnroll];
    uint32_t hm[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int f = f0 + u * KPW + kr;
      key[u] = -1;
      hm[u] = 0;
      if (f < nkeys) {
        const int e = e_begin + f / p.bs;
        const int kk = s_kb[e] * p.bs + (f % p.bs);
        if (kk < p.T_k) {
          key[u] = kk;
          hm[u] = s_mask[e];
        }
      }
      const int kload = key[u] < 0 ? 0 : key[u];
      ku[u] = __ldg(reinterpret_cast<const uint4*>(kbase + (int64_t)kload * p.k_st));
      vu[u] = __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)kload * p.v_st));
    }
    float x[kUnroll][G];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float kf[8];
      bf16x8_to_f32(ku[u], kf);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d = fmaf(qf[j][e], kf[e], d);
#pragma unroll
        for (int off = LPK / 2; off >= 1; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        x[u][j] = (key[u] >= 0 && ((hm[u] >> j) & 1u)) ? d : -INFINITY;
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j) {
      float mb = m[j];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) mb = fmaxf(mb, x[u][j]);
      const float mu = mb == -INFINITY ? 0.f : mb;
      const float alpha = ex2(m[j] - mu);  // 0 when m = -inf
      l[j] *= alpha;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[j][e] *= alpha;
      m[j] = mb;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const float pj = ex2(x[u][j] - mu);
        l[j] += pj;
        float vf[8];
        bf16x8_to_f32(vu[u], vf);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[j][e] = fmaf(pj, vf[e], o[j][e]);
      }
    }
  }
  // Merge the KPW key rows of a warp (lanes with equal d-slice).
#pragma unroll
  for (int off = LPK; off < 32; off <<= 1) {
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[j], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l[j], off);
      const float mn = fmaxf(m[j], mo);
      const float mu = mn == -INFINITY ? 0.f : mn;
      const float a = ex2(m[j] - mu), c = ex2(mo - mu);
      l[j] = l[j] * a + lo * c;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float oo = __shfl_xor_sync(0xffffffffu, o[j][e], off);
        o[j][e] = o[j][e] * a + oo * c;
      }
      m[j] = mn;
    }
  }
  if (kr == 0) {
#pragma unroll
    for (int j = 0; j < G; ++j) {
#pragma unroll
      for (int e = 0; e < 8; ++e) s_o[warp][j][dsl + e] = o[j][e];
      if (lane == 0) {
        s_m[warp][j] = m[j];
        s_l[warp][j] = l[j];
      }
    }
  }
  __syncthreads();
  // Merge the warps: one thread per (head, d).
  for (int idx = threadIdx.x; idx < G * D; idx += kDecThreads) {
    const int j = idx / D, d = idx % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) mx = fmaxf(mx, s_m[w][j]);
    const float mu = mx == -INFINITY ? 0.f : mx;
    float lsum = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float c = ex2(s_m[w][j] - mu);
      lsum += s_l[w][j] * c;
      acc += s_o[w][j][d] * c;
    }
    const int64_t row = ((int64_t)b * p.Hq + h0 + j) * p.n_split + split;
    p.part_o[row * D + d] = acc;
    if (d == 0) {
      p.part_ml[row * 2] = mx;
      p.part_ml[row * 2 + 1] = lsum;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(D) decode_combine_kernel(const float* __restrict__ part_o,
                                                           const float* __restrict__ part_ml,
                                                           __nv_bfloat16* out, int64_t o_sb, int64_t o_sh,
                                                           int Hq, int n_split) {
  const int bh = blockIdx.x;
  const int b = bh / Hq, h = bh % Hq;
  const int d = threadIdx.x;
  const float* ml = part_ml + (int64_t)bh * n_split * 2;
  float mx = -INFINITY;
  for (int s = 0; s < n_split; ++s) mx = fmaxf(mx, ml[2 * s]);
  const float mu = mx == -INFINITY ? 0.f : mx;
  float lsum = 0.f, acc = 0.f;
  for (int s = 0; s < n_split; ++s) {
    const float c = ex2(ml[2 * s] - mu);
    lsum += ml[2 * s + 1] * c;
    acc += part_o[((int64_t)bh * n_split + s) * D + d] * c;
  }
  const float r = lsum > 0.f ? acc / lsum : 0.f;
  out[(int64_t)b * o_sb + (int64_t)h * o_sh + d] = __float2bfloat16_rn(r);
}

template <int D, int G>
static int launch_decode(const DecodeParams& prm, const sa_attn_args* a, cudaStream_t stream) {
  dim3 grid(prm.n_split, prm.Hkv, prm.B);
  decode_split_kernel<D, G><<<grid, kDecThreads, 0, stream>>>(prm);
  SA_CHECK_CUDA(cudaGetLastError());
  decode_combine_kernel<D><<<prm.B * prm.Hq, D, 0, stream>>>(
      prm.part_o, prm.part_ml, reinterpret_cast<__nv_bfloat16*>(a->out), a->o_strides[0],
      a->o_strides[1], prm.Hq, prm.n_split);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

}  // namespace sa

using namespace sa;

int sa_validate_attn_args(const sa_attn_args* a, bool decode);

// Fills DecodeParams from the C ABI arguments (shared with the no-scratch variant).
int sa_decode_prepare(const sa_attn_args* a, int32_t n_split, float* partial_o, float* partial_ml,
                      DecodeParams* prm) {
  int rc = sa_validate_attn_args(a, true);
  if (rc) return rc;
  if (a->T_q != 1) return sa_fail(SA_ERR_INVALID, "decode needs T_q == 1 (got %d)", a->T_q);
  const int G = a->Hq / a->Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return sa_fail(SA_ERR_UNSUPPORTED, "Hq/Hkv = %d unsupported for decode (1, 2, 4 or 8)", G);
  if (n_split < 1 || n_split > 64) return sa_fail(SA_ERR_INVALID, "n_split %d not in [1, 64]", n_split);
  if (!partial_o || !partial_ml) return sa_fail(SA_ERR_INVALID, "NULL scratch pointer");
  memset(prm, 0, sizeof(*prm));
  prm->q = reinterpret_cast<const __nv_bfloat16*>(a->q);
  prm->k = reinterpret_cast<const __nv_bfloat16*>(a->k);
  prm->v = reinterpret_cast<const __nv_bfloat16*>(a->v);
  prm->q_sb = a->q_strides[0];
  prm->q_sh = a->q_strides[1];
  prm->k_sb = a->k_strides[0];
  prm->k_sh = a->k_strides[1];
  prm->k_st = a->k_strides[2];
  prm->v_sb = a->v_strides[0];
  prm->v_sh = a->v_strides[1];
  prm->v_st = a->v_strides[2];
  prm->pairs = a->pairs;
  prm->offsets = a->offsets;
  prm->pairs_stride = a->pairs_stride;
  prm->B = a->B;
  prm->Hq = a->Hq;
  prm->Hkv = a->Hkv;
  prm->T_k = a->T_k;
  prm->bs = a->block_size;
  prm->n_split = n_split;
  prm->scale_log2 = a->scale * 1.4426950408889634f;
  prm->part_o = partial_o;
  prm->part_ml = partial_ml;
  prm->err = sa_device_error_ptr();
  return SA_OK;
}

int sa_decode_launch(const DecodeParams& prm, const sa_attn_args* a, cudaStream_t stream) {
  const int G = a->Hq / a->Hkv;
  switch (a->D * 100 + G) {
    case 12801: return launch_decode<128, 1>(prm, a, stream);
    case 12802: return launch_decode<128, 2>(prm, a, stream);
    case 12804: return launch_decode<128, 4>(prm, a, stream);
    case 12808: return launch_decode<128, 8>(prm, a, stream);
    case 6401: return launch_decode<64, 1>(prm, a, stream);
    case 6402: return launch_decode<64, 2>(prm, a, stream);
    case 6404: return launch_decode<64, 4>(prm, a, stream);
    case 6408: return launch_decode<64, 8>(prm, a, stream);
  }
  return sa_fail(SA_ERR_UNSUPPORTED, "no decode kernel for D=%d G=%d", a->D, G);
}

extern "C" int sa_decode_fwd(const sa_attn_args* a, int32_t n_split, float* partial_o,
                             float* partial_ml, sa_stream_t stream) {
  DecodeParams prm;
  int rc = sa_decode_prepare(a, n_split, partial_o, partial_ml, &prm);
  if (rc) return rc;
  return sa_decode_launch(prm, a, reinterpret_cast<cudaStream_t>(stream));
}
