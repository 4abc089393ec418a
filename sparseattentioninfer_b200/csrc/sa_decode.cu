// sa_decode.cu — split-KV block-sparse decode (one query token per sequence).
//
// Replaces the decode use of _universal_sparse_attn_kernel
// (kernels/triton/universal_sparse_attn.py:45-160 with Q_OFFSET = T_k, :84-89),
// which spends a 1-row query block per (b, q-head) and re-reads K/V per head.
// Here one CTA serves a (b, kv-head, split): it reads each retained KV block of
// the group once for all Hq/Hkv query heads. The reference draws different
// random blocks per query head (bigbird_pattern.py:23-41), so the CTA first
// builds the sorted union of the group's CSR rows in shared memory (a per-block
// head bitmask, filled in parallel and compacted), then takes its contiguous
// share of the union.
// Memory path: a ring of kDecStages stages of up to 64 keys of K and V, filled
// by untiled bulk copies (cp.async.bulk, mbarrier completion) issued by one
// thread, so a whole stage is in flight per instruction; four warps consume
// each stage from shared memory (D/8 lanes per key row, 16-byte reads).
// Statistics in fp32 (log2 domain). A second kernel merges the splits
// (log-sum-exp) and writes bf16.
#include <cstring>

#include "sa_common.cuh"

namespace sa {

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecStages = 3;
constexpr int kDecChunk = 64;        // keys per stage
constexpr int kMaxUnion = 2048;      // union entries per (b, kv head)
constexpr int kMaxNkbWords = 2048;   // membership bytes packed 4 per word: NKB <= 8192

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

template <int D>
struct DecodeCfg {
  static constexpr int kStageBytes = kDecChunk * D * 2;  // K (or V) of one stage
  static constexpr int kSmemBytes = 2 * kDecStages * kStageBytes + 128;
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

// Issue the bulk copies of one stage (rows [key0, key0+rows) of K and V).
template <int D>
__device__ __forceinline__ void issue_stage(const DecodeParams& p, int b, int kvh, int key0, int rows,
                                            uint32_t sk, uint32_t sv, uint32_t bar) {
  constexpr uint32_t kRow = D * 2;
  if (rows <= 0) {
    mbar_arrive(bar);
    return;
  }
  mbar_arrive_expect_tx(bar, 2u * rows * kRow);
  const __nv_bfloat16* kp = p.k + (int64_t)b * p.k_sb + (int64_t)kvh * p.k_sh + (int64_t)key0 * p.k_st;
  const __nv_bfloat16* vp = p.v + (int64_t)b * p.v_sb + (int64_t)kvh * p.v_sh + (int64_t)key0 * p.v_st;
  if (p.k_st == D) {
    bulk_load(sk, kp, rows * kRow, bar);
  } else {
    for (int r = 0; r < rows; ++r) bulk_load(sk + r * kRow, kp + (int64_t)r * p.k_st, kRow, bar);
  }
  if (p.v_st == D) {
    bulk_load(sv, vp, rows * kRow, bar);
  } else {
    for (int r = 0; r < rows; ++r) bulk_load(sv + r * kRow, vp + (int64_t)r * p.v_st, kRow, bar);
  }
}

template <int D, int G>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(const DecodeParams p) {
  using Cfg = DecodeCfg<D>;
  constexpr int LPK = D / 8;          // lanes per key row (16 B each)
  constexpr int KPW = 32 / LPK;       // key rows per warp instruction
  constexpr int KPWARP = kDecChunk / kDecWarps;  // keys of a stage per warp
  constexpr int IT = KPWARP / KPW;    // warp instructions per stage
  __shared__ int s_kb[kMaxUnion];
  __shared__ uint8_t s_hm[kMaxUnion];
  __shared__ int s_warp_cnt[kDecWarps + 1];
  __shared__ __align__(8) uint64_t bar_full[kDecStages], bar_empty[kDecStages];
  __shared__ float s_m[kDecWarps][G], s_l[kDecWarps][G];
  __shared__ int abort_flag;
  extern __shared__ __align__(128) uint8_t dsmem[];
  const uint32_t sbase = (smem_u32(dsmem) + 127u) & ~127u;
  // The stage ring is free before the first copy and after the drain: it holds
  // the membership words first and the per-warp partial outputs last.
  uint32_t* s_memb = reinterpret_cast<uint32_t*>(dsmem + (sbase - smem_u32(dsmem)));
  float(*s_o)[G][D] = reinterpret_cast<float(*)[G][D]>(dsmem + (sbase - smem_u32(dsmem)));
  static_assert(kMaxNkbWords * 4 <= 2 * kDecStages * DecodeCfg<D>::kStageBytes, "ring too small");
  static_assert(kDecWarps * G * D * 4 <= 2 * kDecStages * DecodeCfg<D>::kStageBytes, "ring too small");

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h0 = kvh * G;
  const int nkb = (p.T_k + p.bs - 1) / p.bs;
  const int nwords = (nkb + 3) >> 2;

  if (tid == 0) {
    for (int i = 0; i < kDecStages; ++i) {
      mbar_init(smem_u32(&bar_full[i]), 1);
      mbar_init(smem_u32(&bar_empty[i]), kDecWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (nwords > kMaxNkbWords) {  // block-uniform
    if (tid == 0) record_error(p.err, SA_DEV_ERR_INDEX);
    return;
  }
  for (int i = tid; i < nwords; i += kDecThreads) s_memb[i] = 0u;
  __syncthreads();
  // Membership bytes: bit j of byte kb = query head h0+j lists block kb.
#pragma unroll 1
  for (int j = 0; j < G; ++j) {
    const int32_t* off = p.offsets + (int64_t)(h0 + j) * 2;
    const int r0 = __ldg(off), r1 = __ldg(off + 1);
    const int32_t* row = p.pairs + (int64_t)(h0 + j) * p.pairs_stride;
    for (int i = r0 + tid; i < r1; i += kDecThreads) {
      const int kb = __ldg(row + i);
      if (kb >= 0 && kb < nkb) atomicOr(&s_memb[kb >> 2], (1u << j) << ((kb & 3) * 8));
    }
  }
  __syncthreads();
  // Compact to the sorted union: thread t owns words [t*per, (t+1)*per).
  const int per = (nwords + kDecThreads - 1) / kDecThreads;
  int cnt = 0;
  for (int w = tid * per; w < min(nwords, (tid + 1) * per); ++w) {
    const uint32_t x = s_memb[w];
    cnt += ((x & 0xffu) != 0) + ((x & 0xff00u) != 0) + ((x & 0xff0000u) != 0) + ((x >> 24) != 0);
  }
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp_cnt[warp] = incl;
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int w = 0; w < kDecWarps; ++w) {
      const int c = s_warp_cnt[w];
      s_warp_cnt[w] = acc;
      acc += c;
    }
    s_warp_cnt[kDecWarps] = acc;
  }
  __syncthreads();
  {
    int pos = s_warp_cnt[warp] + incl - cnt;
    for (int w = tid * per; w < min(nwords, (tid + 1) * per); ++w) {
      const uint32_t x = s_memb[w];
#pragma unroll
      for (int by = 0; by < 4; ++by) {
        const uint32_t m = (x >> (8 * by)) & 0xffu;
        if (m && pos < kMaxUnion) {
          s_kb[pos] = w * 4 + by;
          s_hm[pos] = (uint8_t)m;
          ++pos;
        }
      }
    }
  }
  __syncthreads();  // membership words no longer needed: the ring may be filled
  const int U = min(s_warp_cnt[kDecWarps], kMaxUnion);
  if (tid == 0 && s_warp_cnt[kDecWarps] > kMaxUnion) record_error(p.err, SA_DEV_ERR_INDEX);
  const int e_begin = (int)(((int64_t)U * split) / p.n_split);
  const int e_end = (int)(((int64_t)U * (split + 1)) / p.n_split);
  const int chk = min(p.bs, kDecChunk);      // keys per stage
  const int nsub = p.bs > kDecChunk ? p.bs / kDecChunk : 1;
  const int nst = (e_end - e_begin) * nsub;  // stages of this split

  auto stage_key0 = [&](int i) { return s_kb[e_begin + i / nsub] * p.bs + (i % nsub) * chk; };
  auto stage_rows = [&](int i) { return max(0, min(chk, p.T_k - stage_key0(i))); };
  auto sK = [&](int slot) { return sbase + slot * 2 * Cfg::kStageBytes; };
  auto sV = [&](int slot) { return sbase + slot * 2 * Cfg::kStageBytes + Cfg::kStageBytes; };

  if (tid == 0) {
    // generic-proxy writes (membership words) precede async-proxy writes here
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int i = 0; i < min(nst, kDecStages); ++i)
      issue_stage<D>(p, b, kvh, stage_key0(i), stage_rows(i), sK(i), sV(i), smem_u32(&bar_full[i]));
  }

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
  volatile int* abort_v = &abort_flag;
  bool ok = true;
  for (int i = 0; i < nst; ++i) {
    const int slot = i % kDecStages;
    ok = mbar_wait(smem_u32(&bar_full[slot]), (i / kDecStages) & 1, abort_v, p.err);
    if (!__all_sync(0xffffffffu, ok)) break;
    const int rows = stage_rows(i);
    const uint32_t hm = s_hm[e_begin + i / nsub];
    const uint8_t* kst = dsmem + (sK(slot) - smem_u32(dsmem));
    const uint8_t* vst = dsmem + (sV(slot) - smem_u32(dsmem));
    float x[IT][G];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int r = warp * KPWARP + it * KPW + kr;
      float kf[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(kst + r * D * 2 + dsl * 2), kf);
      const bool valid = r < rows;
#pragma unroll
      for (int j = 0; j < G; ++j) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d = fmaf(qf[j][e], kf[e], d);
#pragma unroll
        for (int off = LPK / 2; off >= 1; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        x[it][j] = (valid && ((hm >> j) & 1u)) ? d : -INFINITY;
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j) {
      float mb = m[j];
#pragma unroll
      for (int it = 0; it < IT; ++it) mb = fmaxf(mb, x[it][j]);
      const float mu = mb == -INFINITY ? 0.f : mb;
      const float alpha = ex2(m[j] - mu);
      l[j] *= alpha;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[j][e] *= alpha;
      m[j] = mb;
    }
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int r = warp * KPWARP + it * KPW + kr;
      float vf[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(vst + r * D * 2 + dsl * 2), vf);
      if (r >= rows) {  // rows past T_k were not copied this time: never multiply them
#pragma unroll
        for (int e = 0; e < 8; ++e) vf[e] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const float mu = m[j] == -INFINITY ? 0.f : m[j];
        const float pj = ex2(x[it][j] - mu);
        l[j] += pj;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[j][e] = fmaf(pj, vf[e], o[j][e]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&bar_empty[slot]));
    if (tid == 0 && i + kDecStages < nst) {
      // refill this slot once every warp has consumed it
      ok = mbar_wait(smem_u32(&bar_empty[slot]), (i / kDecStages) & 1, abort_v, p.err);
      if (ok)
        issue_stage<D>(p, b, kvh, stage_key0(i + kDecStages), stage_rows(i + kDecStages), sK(slot), sV(slot),
                       smem_u32(&bar_full[slot]));
    }
  }
  // Drain (bounded) copies still in flight before the ring is reused or the CTA exits.
  if (tid == 0) {
    int zero = 0;
    for (int i = max(0, nst - kDecStages); i < nst; ++i)
      mbar_wait(smem_u32(&bar_full[i % kDecStages]), (i / kDecStages) & 1, &zero, nullptr);
  }
  __syncthreads();  // ring idle: reuse it for the per-warp partials
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
  for (int idx = tid; idx < G * D; idx += kDecThreads) {
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
    const int64_t rowi = ((int64_t)b * p.Hq + h0 + j) * p.n_split + split;
    p.part_o[rowi * D + d] = acc;
    if (d == 0) {
      p.part_ml[rowi * 2] = mx;
      p.part_ml[rowi * 2 + 1] = lsum;
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
  SA_CHECK_CUDA(cudaFuncSetAttribute(decode_split_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     DecodeCfg<D>::kSmemBytes));
  decode_split_kernel<D, G><<<grid, kDecThreads, DecodeCfg<D>::kSmemBytes, stream>>>(prm);
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

// ---------------------------------------------------------------------------
// Allocation-free decode: split partials in a library-owned device array.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_sa_decode_scratch[SA_DECODE_SCRATCH_FLOATS];

// Device address of g_sa_decode_scratch on the current device, looked up once
// per device (the host-side symbol is not a device address).
static int decode_scratch_ptr(float** out) {
  static float* ptrs[64] = {nullptr};
  int dev = 0;
  SA_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return sa_fail(SA_ERR_UNSUPPORTED, "device index %d out of range", dev);
  if (!ptrs[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_sa_decode_scratch);
    if (e != cudaSuccess) return sa_cuda_check(e, "cudaGetSymbolAddress(g_sa_decode_scratch)");
    ptrs[dev] = static_cast<float*>(p);
  }
  *out = ptrs[dev];
  return SA_OK;
}

extern "C" int sa_decode_fwd_noalloc(const sa_attn_args* a, int32_t n_split, sa_stream_t stream) {
  if (!a) return sa_fail(SA_ERR_INVALID, "args is NULL");
  if (n_split < 1 || n_split > 64) return sa_fail(SA_ERR_INVALID, "n_split %d not in [1, 64]", n_split);
  if (a->B <= 0 || a->Hq <= 0 || (a->D != 64 && a->D != 128))
    return sa_fail(SA_ERR_INVALID, "bad B/Hq/D (B=%d Hq=%d D=%d)", a->B, a->Hq, a->D);
  const int64_t rows = (int64_t)a->B * a->Hq * n_split;
  const int64_t need = rows * (a->D + 2);
  if (need > (int64_t)SA_DECODE_SCRATCH_FLOATS)
    return sa_fail(SA_ERR_INVALID,
                   "decode scratch needs %lld floats (B*Hq*n_split*(D+2)), the built-in array holds %d; "
                   "lower n_split or use sa_decode_fwd with caller scratch",
                   (long long)need, (int)SA_DECODE_SCRATCH_FLOATS);
  float* base = nullptr;
  int rc = decode_scratch_ptr(&base);
  if (rc) return rc;
  DecodeParams prm;
  rc = sa_decode_prepare(a, n_split, base, base + rows * a->D, &prm);
  if (rc) return rc;
  return sa_decode_launch(prm, a, reinterpret_cast<cudaStream_t>(stream));
}
