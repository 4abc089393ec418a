// sa_decode.cu — split-KV block-sparse decode (one query token per sequence).
//
// Replaces the decode use of _universal_sparse_attn_kernel
// (kernels/triton/universal_sparse_attn.py:45-160 with Q_OFFSET = T_k, :84-89),
// which spends a 1-row query block per (b, q-head) and re-reads K/V per head.
// Here one CTA serves a (b, kv-head, split): it reads each retained KV block of
// the group once for all G = Hq/Hkv query heads. The reference draws different
// random blocks per query head (bigbird_pattern.py:23-41), so the CTA first
// builds the sorted union of the group's CSR rows in shared memory (a per-block
// head bitmask, filled in parallel and compacted), then takes its contiguous
// share of the union.
//
// Pipeline: a producer warp streams stages of up to 64 keys of K and V with TMA
// (4-D tensor maps, SWIZZLE_128B, zero fill past T_k) into a 3-stage ring; four
// consumer warps take 16 keys each and do both products on the tensor cores
// with mma.sync m16n8k16 (bf16 in, fp32 accumulate): the group's G query rows
// are padded to the 16-row A operand, K fragments come from ldmatrix on the
// swizzled rows, V fragments from ldmatrix.trans, and P goes from the S
// accumulators straight into the A operand of PV. Online softmax per warp in
// fp32 (log2 domain); warps and splits are merged by log-sum-exp (a second tiny
// kernel when n_split > 1; the split kernel writes bf16 directly otherwise).
#include <cstring>

#include "sa_common.cuh"

namespace sa {

constexpr int kDecConsumers = 4;                  // consumer warps
constexpr int kDecThreads = 32 * (kDecConsumers + 1);
constexpr int kDecStages = 3;
constexpr int kDecChunk = 64;        // max keys per stage
constexpr int kMaxUnion = 2048;      // union entries per (b, kv head)
constexpr int kMaxNkbWords = 2048;   // membership bytes packed 4 per word: NKB <= 8192

struct DecodeParams {
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh;
  const int32_t* pairs;
  const int32_t* offsets;
  int32_t pairs_stride;
  int32_t B, Hq, Hkv, T_k, bs, n_split, chk;
  const int32_t* T_k_dev;  // live key count in device memory (<= T_k), or NULL
  float scale_log2;
  float* part_o;   // [B, Hq, n_split, D]
  float* part_ml;  // [B, Hq, n_split, 2]
  __nv_bfloat16* out;  // written directly when n_split == 1
  int64_t o_sb, o_sh;
  int32_t* err;
};

template <int D>
struct DecodeCfg {
  static constexpr int kRegions = D / 64;
  static constexpr int kHalfBytes = kDecChunk * D * 2;          // K (or V) of one stage
  static constexpr int kStageBytes = 2 * kHalfBytes;
  static constexpr int kSmemBytes = kDecStages * kStageBytes;
};

#ifdef SA_PHASE_TRACE
__device__ unsigned long long g_dec_trace[4096 * 4];
#define DEC_TRACE(slot)                                                                                   \
  do {                                                                                                    \
    const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);                       \
    if (threadIdx.x == 0 && cta_ < 4096) {                                                                \
      unsigned long long t_;                                                                              \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                             \
      g_dec_trace[cta_ * 4 + (slot)] = t_;                                                                \
    }                                                                                                     \
  } while (0)
#else
#define DEC_TRACE(slot) \
  do {                  \
  } while (0)
#endif

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D = A(16x16, row) * B(16x8, col) + D, bf16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Shared address of 16-byte chunk `c` (of 8 per 128-byte row) of row `r` in a
// SWIZZLE_128B region (1024-byte aligned): TMA stored it XOR-permuted by r%8.
__device__ __forceinline__ uint32_t sw128(uint32_t region, int r, int c) {
  return region + r * 128 + ((c ^ (r & 7)) << 4);
}

template <int D, int G>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(const __grid_constant__ DecodeParams p) {
  using Cfg = DecodeCfg<D>;
  constexpr int R = Cfg::kRegions;
  constexpr int NT = D / 8;  // n-tiles of the PV product
  __shared__ int s_kb[kMaxUnion];
  __shared__ uint8_t s_hm[kMaxUnion];
  __shared__ int s_warp_cnt[kDecThreads / 32 + 1];
  __shared__ __align__(8) uint64_t bar_full[kDecStages], bar_empty[kDecStages];
  __shared__ float s_m[kDecConsumers][8], s_l[kDecConsumers][8];
  __shared__ int abort_flag;
  extern __shared__ __align__(1024) uint8_t dsmem[];
  const uint32_t sbase = smem_u32(dsmem);
  // The stage ring is free before the first copy and after the drain: it holds
  // the membership words first and the per-warp partial outputs last.
  uint32_t* s_memb = reinterpret_cast<uint32_t*>(dsmem);
  float(*s_o)[8][D] = reinterpret_cast<float(*)[8][D]>(dsmem);
  static_assert(kMaxNkbWords * 4 <= kDecStages * Cfg::kStageBytes, "ring too small");
  static_assert(kDecConsumers * 8 * D * 4 <= kDecStages * Cfg::kStageBytes, "ring too small");
  static_assert(G <= 8, "at most 8 query heads per KV group");

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h0 = kvh * G;
  // Keys [0, T_k): the live length from device memory when given (graph replays
  // of a growing cache), else the host value; the tensor maps span p.T_k rows.
  const int T_k = p.T_k_dev ? max(0, min(__ldg(p.T_k_dev), p.T_k)) : p.T_k;
  const int nkb = (T_k + p.bs - 1) / p.bs;
  const int nwords = (nkb + 3) >> 2;
  DEC_TRACE(0);

  if (tid == 0) {
    if (sbase & 1023u) record_error(p.err, SA_DEV_ERR_INDEX);
    for (int i = 0; i < kDecStages; ++i) {
      mbar_init(smem_u32(&bar_full[i]), 1);
      mbar_init(smem_u32(&bar_empty[i]), kDecConsumers);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (nwords > kMaxNkbWords || (sbase & 1023u)) {  // block-uniform
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
    for (int w = 0; w < kDecThreads / 32; ++w) {
      const int c = s_warp_cnt[w];
      s_warp_cnt[w] = acc;
      acc += c;
    }
    s_warp_cnt[kDecThreads / 32] = acc;
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
  DEC_TRACE(1);
  const int U = min(s_warp_cnt[kDecThreads / 32], kMaxUnion);
  if (tid == 0 && s_warp_cnt[kDecThreads / 32] > kMaxUnion) record_error(p.err, SA_DEV_ERR_INDEX);
  const int e_begin = (int)(((int64_t)U * split) / p.n_split);
  const int e_end = (int)(((int64_t)U * (split + 1)) / p.n_split);
  const int chk = p.chk;                                    // keys per stage (= TMA box rows)
  const int nsub = p.bs > chk ? p.bs / chk : 1;
  const int nst = (e_end - e_begin) * nsub;                 // stages of this split
  volatile int* abort_v = &abort_flag;

  auto stage_key0 = [&](int i) { return s_kb[e_begin + i / nsub] * p.bs + (i % nsub) * chk; };

  float m_run = -INFINITY, l_run = 0.f;
  float o_acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o_acc[j][0] = o_acc[j][1] = o_acc[j][2] = o_acc[j][3] = 0.f;
  const int row = lane >> 2;  // query head of this thread's accumulator rows 0..7

  if (warp == kDecConsumers) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // membership words were generic writes
      bool ok = true;
      for (int i = 0; i < nst && ok; ++i) {
        const int slot = i % kDecStages;
        if (i >= kDecStages &&
            !(ok = mbar_wait(smem_u32(&bar_empty[slot]), ((i / kDecStages) - 1) & 1, abort_v, p.err)))
          break;
        const int key0 = min(stage_key0(i), T_k);  // past T_k: masked below
        const uint32_t st = sbase + slot * Cfg::kStageBytes;
        mbar_arrive_expect_tx(smem_u32(&bar_full[slot]), 2u * chk * D * 2);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          tma_load_4d(st + r * kDecChunk * 128, &p.tm_k, smem_u32(&bar_full[slot]), r * 64, key0, kvh, b);
          tma_load_4d(st + Cfg::kHalfBytes + r * kDecChunk * 128, &p.tm_v, smem_u32(&bar_full[slot]), r * 64,
                      key0, kvh, b);
        }
      }
      int zero = 0;  // drain (bounded) copies still in flight
      for (int i = max(0, nst - kDecStages); i < nst; ++i)
        mbar_wait(smem_u32(&bar_full[i % kDecStages]), (i / kDecStages) & 1, &zero, nullptr);
    }
  } else {
    // ------------------------------------------------------------ consumers
    // Q of the group as the A operand: rows 0..G-1 = heads, rows G..15 zero.
    uint32_t qa[D / 16][2];
    {
      const __nv_bfloat16* qrow = p.q + (int64_t)b * p.q_sb + (int64_t)(h0 + row) * p.q_sh;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int d = kk * 16 + 2 * (lane & 3);
        qa[kk][0] = row < G ? *reinterpret_cast<const uint32_t*>(qrow + d) : 0u;
        qa[kk][1] = row < G ? *reinterpret_cast<const uint32_t*>(qrow + d + 8) : 0u;
      }
    }
    const int k_lo = warp * 16;  // this warp's 16 keys of each stage
    for (int i = 0; i < nst; ++i) {
      const int slot = i % kDecStages;
      bool ok = mbar_wait(smem_u32(&bar_full[slot]), (i / kDecStages) & 1, abort_v, p.err);
      if (!__all_sync(0xffffffffu, ok)) break;
      const int key0 = stage_key0(i);
      const int rows = max(0, min(chk, T_k - key0));
      const uint32_t hm = s_hm[e_begin + i / nsub];
      if (k_lo < rows) {
        const uint32_t sk = sbase + slot * Cfg::kStageBytes;
        const uint32_t sv = sk + Cfg::kHalfBytes;
        // S = Q K^T for this warp's two 8-key n-tiles.
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
        const int kr = k_lo + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int reg = kk >> 2;
          const int ch = ((kk & 3) << 1) + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sw128(sk + reg * kDecChunk * 128, kr, ch), b0, b1, b2, b3);
          mma_bf16(s0, qa[kk][0], 0u, qa[kk][1], 0u, b0, b1);
          mma_bf16(s1, qa[kk][0], 0u, qa[kk][1], 0u, b2, b3);
        }
        // mask + online softmax (rows = heads; keys 2*(lane&3)+{0,1} of each tile)
        const bool head_ok = row < G && ((hm >> row) & 1u);
        const int c0 = k_lo + 2 * (lane & 3);
        float x[4];
        x[0] = (head_ok && c0 < rows) ? s0[0] * p.scale_log2 : -INFINITY;
        x[1] = (head_ok && c0 + 1 < rows) ? s0[1] * p.scale_log2 : -INFINITY;
        x[2] = (head_ok && c0 + 8 < rows) ? s1[0] * p.scale_log2 : -INFINITY;
        x[3] = (head_ok && c0 + 9 < rows) ? s1[1] * p.scale_log2 : -INFINITY;
        float mb = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
        mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
        const float m_new = fmaxf(m_run, mb);
        const float mu = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = ex2(m_run - mu);
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[e] = ex2(x[e] - mu);
        l_run = l_run * alpha + (pr[0] + pr[1]) + (pr[2] + pr[3]);
        m_run = m_new;
        const uint32_t pa0 = pack_bf16(pr[0], pr[1]), pa2 = pack_bf16(pr[2], pr[3]);
        // O = alpha * O + P V over this warp's 16 keys.
        const int vr = k_lo + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
          const int dch = j + (lane >> 4);  // 16-byte chunk index over D
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(sw128(sv + (dch >> 3) * kDecChunk * 128, vr, dch & 7), v0, v1, v2, v3);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            o_acc[j][e] *= alpha;
            o_acc[j + 1][e] *= alpha;
          }
          mma_bf16(o_acc[j], pa0, 0u, pa2, 0u, v0, v1);
          mma_bf16(o_acc[j + 1], pa0, 0u, pa2, 0u, v2, v3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar_empty[slot]));
    }
  }
  DEC_TRACE(2);
  __syncthreads();  // ring idle (producer drained): reuse it for the per-warp partials
  if (warp < kDecConsumers) {
    float l_row = l_run;
    l_row += __shfl_xor_sync(0xffffffffu, l_row, 1);
    l_row += __shfl_xor_sync(0xffffffffu, l_row, 2);
    if ((lane & 3) == 0) {
      s_m[warp][row] = m_run;
      s_l[warp][row] = l_row;
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      s_o[warp][row][j * 8 + 2 * (lane & 3)] = o_acc[j][0];
      s_o[warp][row][j * 8 + 2 * (lane & 3) + 1] = o_acc[j][1];
    }
  }
  __syncthreads();
  // Merge the consumer warps: one thread per (head, d).
  for (int idx = tid; idx < G * D; idx += kDecThreads) {
    const int j = idx / D, d = idx % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecConsumers; ++w) mx = fmaxf(mx, s_m[w][j]);
    const float mu = mx == -INFINITY ? 0.f : mx;
    float lsum = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kDecConsumers; ++w) {
      const float c = ex2(s_m[w][j] - mu);
      lsum += s_l[w][j] * c;
      acc += s_o[w][j][d] * c;
    }
    if (p.n_split == 1) {
      p.out[(int64_t)b * p.o_sb + (int64_t)(h0 + j) * p.o_sh + d] = __float2bfloat16_rn(lsum > 0.f ? acc / lsum : 0.f);
    } else {
      const int64_t rowi = ((int64_t)b * p.Hq + h0 + j) * p.n_split + split;
      p.part_o[rowi * D + d] = acc;
      if (d == 0) {
        p.part_ml[rowi * 2] = mx;
        p.part_ml[rowi * 2 + 1] = lsum;
      }
    }
  }
  DEC_TRACE(3);
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
  if (prm.n_split > 1) {
    decode_combine_kernel<D><<<prm.B * prm.Hq, D, 0, stream>>>(
        prm.part_o, prm.part_ml, reinterpret_cast<__nv_bfloat16*>(a->out), a->o_strides[0],
        a->o_strides[1], prm.Hq, prm.n_split);
    SA_CHECK_CUDA(cudaGetLastError());
  }
  return SA_OK;
}

}  // namespace sa

using namespace sa;

int sa_validate_attn_args(const sa_attn_args* a, bool decode);

// Host-side checks shared by every decode entry point (before any CUDA call).
static int decode_check(const sa_attn_args* a, int32_t n_split) {
  int rc = sa_validate_attn_args(a, true);
  if (rc) return rc;
  if (a->T_q != 1) return sa_fail(SA_ERR_INVALID, "decode needs T_q == 1 (got %d)", a->T_q);
  const int G = a->Hq / a->Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return sa_fail(SA_ERR_UNSUPPORTED, "Hq/Hkv = %d unsupported for decode (1, 2, 4 or 8)", G);
  if (n_split < 1 || n_split > 64) return sa_fail(SA_ERR_INVALID, "n_split %d not in [1, 64]", n_split);
  // Shared-memory limits of one CTA: the membership words cover NKB <= 8192 key
  // blocks and the union list holds kMaxUnion blocks; the union of a group's G
  // rows has at most min(NKB, G * pairs_stride) blocks.
  const int64_t nkb = ((int64_t)a->T_k + a->block_size - 1) / a->block_size;
  if (nkb > (int64_t)kMaxNkbWords * 4)
    return sa_fail(SA_ERR_UNSUPPORTED, "decode supports ceil(T_k / block_size) <= %d (got %lld)", kMaxNkbWords * 4,
                   (long long)nkb);
  const int64_t ub = nkb < (int64_t)G * a->pairs_stride ? nkb : (int64_t)G * a->pairs_stride;
  if (ub > kMaxUnion)
    return sa_fail(SA_ERR_UNSUPPORTED,
                   "decode unions up to %d blocks per KV group; min(ceil(T_k / block_size), (Hq/Hkv) * "
                   "pairs_stride) = %lld",
                   kMaxUnion, (long long)ub);
  return SA_OK;
}

// Fills DecodeParams from the C ABI arguments (shared with the no-scratch variant).
int sa_decode_prepare(const sa_attn_args* a, int32_t n_split, float* partial_o, float* partial_ml,
                      DecodeParams* prm) {
  int rc = decode_check(a, n_split);
  if (rc) return rc;
  if (!partial_o || !partial_ml) return sa_fail(SA_ERR_INVALID, "NULL scratch pointer");
  memset(prm, 0, sizeof(*prm));
  prm->chk = a->block_size < kDecChunk ? a->block_size : kDecChunk;
  if ((rc = sa_make_map(&prm->tm_k, a->k, a->B, a->Hkv, a->T_k, a->D, a->k_strides, prm->chk, "k"))) return rc;
  if ((rc = sa_make_map(&prm->tm_v, a->v, a->B, a->Hkv, a->T_k, a->D, a->v_strides, prm->chk, "v"))) return rc;
  prm->q = reinterpret_cast<const __nv_bfloat16*>(a->q);
  prm->q_sb = a->q_strides[0];
  prm->q_sh = a->q_strides[1];
  prm->out = reinterpret_cast<__nv_bfloat16*>(a->out);
  prm->o_sb = a->o_strides[0];
  prm->o_sh = a->o_strides[1];
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

extern "C" int sa_decode_fwd_seqlen(const sa_attn_args* a, const int32_t* seq_len, int32_t n_split,
                                    float* partial_o, float* partial_ml, sa_stream_t stream) {
  if (!seq_len) return sa_fail(SA_ERR_INVALID, "seq_len is NULL");
  DecodeParams prm;
  int rc = sa_decode_prepare(a, n_split, partial_o, partial_ml, &prm);
  if (rc) return rc;
  prm.T_k_dev = seq_len;
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
  int rc = decode_check(a, n_split);  // same checks and error codes as sa_decode_fwd
  if (rc) return rc;
  // With one split the kernel writes the output directly and never touches the
  // scratch array, so only n_split > 1 is bounded by its size.
  const int64_t rows = (int64_t)a->B * a->Hq * n_split;
  const int64_t need = rows * (a->D + 2);
  if (n_split > 1 && need > (int64_t)SA_DECODE_SCRATCH_FLOATS)
    return sa_fail(SA_ERR_INVALID,
                   "decode scratch needs %lld floats (B*Hq*n_split*(D+2)), the built-in array holds %d; "
                   "lower n_split or use sa_decode_fwd with caller scratch",
                   (long long)need, (int)SA_DECODE_SCRATCH_FLOATS);
  float* base = nullptr;
  if ((rc = decode_scratch_ptr(&base))) return rc;
  DecodeParams prm;
  // n_split == 1: the partial pointers are unused; point both at the array start.
  rc = sa_decode_prepare(a, n_split, base, n_split > 1 ? base + rows * a->D : base, &prm);
  if (rc) return rc;
  return sa_decode_launch(prm, a, reinterpret_cast<cudaStream_t>(stream));
}

#ifdef SA_PHASE_TRACE
extern "C" SA_API int sa_debug_dec_trace_read(unsigned long long* host, int n) {
  SA_CHECK_CUDA(cudaDeviceSynchronize());
  SA_CHECK_CUDA(cudaMemcpyFromSymbol(host, sa::g_dec_trace, sizeof(unsigned long long) * (n < 16384 ? n : 16384)));
  return SA_OK;
}
#endif
