// sa_prefill_sm100.cu — block-sparse FlashAttention forward for B200 (sm_100a).
//
// Computes what _universal_sparse_attn_kernel computes
// (kernels/triton/universal_sparse_attn.py:45-160): for every query row, online
// softmax over the key blocks listed in its CSR row, causal + bounds masked,
// fp32 statistics, P rounded to bf16 before the PV product, empty rows -> 0.
//
// Design (one persistent CTA per SM, 6 warps, warp-specialised):
//   warp 0      TMA producer: Q tile once per tile, then a ring of K/V chunk
//               stages (4-D tensor maps over [B, H, T, D], SWIZZLE_128B).
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//                 S = Q K^T    (SS form, M=128, N=chunk, K=D) into TMEM
//                 O += P V     (TS form, P read straight from TMEM)
//   warps 2..5  softmax warpgroup: one thread per query row = one TMEM lane.
//               Reads S with tcgen05.ld, masks, keeps the running max/sum in
//               registers, writes P (bf16x2) back over S with tcgen05.st,
//               rescales O in TMEM only when the row max grew by > 2^8
//               (exact: the same stale max is used for P, l and O), and runs
//               the epilogue (O / l -> bf16 -> global).
// A tile is 128 query rows of one (b, q-head). For block size bs < 128 a tile
// holds 128/bs consecutive query blocks; their CSR rows are merged on the fly
// into one sorted chunk stream with a per-block membership mask. For bs > 128
// each key block is split into 128-key chunks.
// TMEM: O at columns [0, D), two S/P buffers at [128, 256) and [256, 384).
// Tiles are visited heaviest-first (last query tiles first) with a static
// stride over the persistent grid.
#include <cstdio>
#include <cstring>

#include "sa_common.cuh"

namespace sa {

struct PrefillParams {
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_st;
  const int32_t* pairs;
  const int32_t* offsets;
  int32_t pairs_stride;
  int32_t B, Hq, Hkv, T_q, T_k, bs, nqb, nqt, group;
  float scale_log2;
  int32_t* err;
};

constexpr int kThreads = 192;
constexpr int kTileM = 128;
constexpr int kMaxSeg = 8;  // 128 / 16

template <int D, int N>
struct PrefillCfg {
  static constexpr int kRegions = D / 64;               // 64-column (128 B) slabs
  static constexpr int kQBytes = kTileM * D * 2;
  static constexpr int kKVBytes = N * D * 2;            // one K (or V) chunk
  static constexpr int kSmemBudget = 227 * 1024 - 2048;
  static constexpr int kStagesFit = (kSmemBudget - 1024 - kQBytes) / (2 * kKVBytes);
  static constexpr int kStages = kStagesFit > 4 ? 4 : kStagesFit;
  static constexpr int kSmemBytes = 1024 + kQBytes + kStages * 2 * kKVBytes;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage pipeline");
};

// Chunk stream of one tile: sorted union of up to kMaxSeg CSR rows, each key
// block expanded into `nsub` chunks of N keys.
struct ChunkStream {
  const int32_t* pairs;
  int ptr[kMaxSeg];
  int end[kMaxSeg];
  int nseg;
  int nsub;
  int sub;
  int kb;
  uint32_t mask;

  __device__ void init(const PrefillParams& p, int h, int qb0, int nseg_, int nsub_) {
    pairs = p.pairs + (int64_t)h * p.pairs_stride;
    const int32_t* off = p.offsets + (int64_t)h * (p.nqb + 1);
    nseg = nseg_;
    nsub = nsub_;
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s) {
      if (s < nseg) {
        ptr[s] = __ldg(off + qb0 + s);
        end[s] = __ldg(off + qb0 + s + 1);
      } else {
        ptr[s] = end[s] = 0;
      }
    }
    sub = nsub;  // forces an advance on the first next()
    kb = -1;
    mask = 0;
  }
  // Advance to the next chunk; false when exhausted.
  __device__ bool next() {
    if (sub + 1 < nsub) {
      ++sub;
      return true;
    }
    int best = 0x7fffffff;
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s)
      if (s < nseg && ptr[s] < end[s]) best = min(best, __ldg(pairs + ptr[s]));
    if (best == 0x7fffffff) return false;
    uint32_t m = 0;
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s)
      if (s < nseg && ptr[s] < end[s] && __ldg(pairs + ptr[s]) == best) {
        m |= 1u << s;
        ++ptr[s];
      }
    kb = best;
    mask = m;
    sub = 0;
    return true;
  }
};

struct TileCoord {
  int b, h, q0, qb0, nseg, nsub;
};

__device__ __forceinline__ TileCoord tile_coord(const PrefillParams& p, int t) {
  const int bh_total = p.B * p.Hq;
  const int qt = p.nqt - 1 - t / bh_total;  // heaviest (last) query tiles first
  const int bh = t % bh_total;
  TileCoord c;
  c.b = bh / p.Hq;
  c.h = bh % p.Hq;
  c.q0 = qt * kTileM;
  if (p.bs <= kTileM) {
    c.qb0 = c.q0 / p.bs;
    c.nseg = min(kTileM / p.bs, p.nqb - c.qb0);
    c.nsub = 1;
  } else {
    c.qb0 = c.q0 / p.bs;
    c.nseg = 1;
    c.nsub = p.bs / kTileM;
  }
  return c;
}

template <int D, int N>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  using Cfg = PrefillCfg<D, N>;
  constexpr int NST = Cfg::kStages;
  constexpr int R = Cfg::kRegions;

  __shared__ __align__(8) uint64_t bar_q_full, bar_q_empty, bar_o_empty, bar_drain;
  __shared__ __align__(8) uint64_t bar_k_full[NST], bar_v_full[NST], bar_kv_empty[NST];
  __shared__ __align__(8) uint64_t bar_s_full[2], bar_p_full[2], bar_pv_done[2];
  __shared__ int meta_key0[NST];
  __shared__ uint32_t meta_mask[NST];
  __shared__ int meta_last[NST];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = smem_base;
  const uint32_t sK = sQ + Cfg::kQBytes;
  const uint32_t sV = sK + NST * Cfg::kKVBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntiles = p.nqt * p.B * p.Hq;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar_q_full), 1);
    mbar_init(smem_u32(&bar_q_empty), 1);
    mbar_init(smem_u32(&bar_o_empty), 128);
    mbar_init(smem_u32(&bar_drain), 1);
    for (int i = 0; i < NST; ++i) {
      mbar_init(smem_u32(&bar_k_full[i]), 1);
      mbar_init(smem_u32(&bar_v_full[i]), 1);
      mbar_init(smem_u32(&bar_kv_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bar_s_full[i]), 1);
      mbar_init(smem_u32(&bar_p_full[i]), 128);
      mbar_init(smem_u32(&bar_pv_done[i]), 1);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base_sh), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  volatile int* abort_v = &abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t g = 0;  // chunks issued by this CTA
      int it = 0;
      int q_issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
        const TileCoord c = tile_coord(p, t);
        const int kvh = c.h / p.group;
        if (it > 0 && !(ok = mbar_wait(smem_u32(&bar_q_empty), (it - 1) & 1, abort_v, p.err))) break;
        mbar_arrive_expect_tx(smem_u32(&bar_q_full), Cfg::kQBytes);
#pragma unroll
        for (int r = 0; r < R; ++r)
          tma_load_4d(sQ + r * kTileM * 128, &p.tm_q, smem_u32(&bar_q_full), r * 64, c.q0, c.h, c.b);
        ++q_issued;

        ChunkStream cs;
        cs.init(p, c.h, c.qb0, c.nseg, c.nsub);
        bool have = cs.next();
        int cur_kb = have ? cs.kb : 0;
        uint32_t cur_mask = have ? cs.mask : 0u;  // empty tile: one fully masked chunk
        int cur_sub = have ? cs.sub : 0;
        while (true) {
          const bool more = have && cs.next();
          const int st = g % NST;
          if (g >= (uint32_t)NST &&
              !(ok = mbar_wait(smem_u32(&bar_kv_empty[st]), ((g / NST) - 1) & 1, abort_v, p.err)))
            break;
          int key0 = cur_kb * p.bs + cur_sub * N;
          if (cur_kb < 0 || key0 < 0 || cur_kb >= (0x7fffffff / max(p.bs, 1)) ) {
            // malformed index: load block 0, mask everything
            record_error(p.err, SA_DEV_ERR_INDEX);
            key0 = 0;
            cur_mask = 0;
          }
          meta_key0[st] = key0;
          meta_mask[st] = cur_mask;
          meta_last[st] = more ? 0 : 1;
          const int kcoord = min(key0, p.T_k);  // fully out-of-range chunks read zeros
          mbar_arrive_expect_tx(smem_u32(&bar_k_full[st]), Cfg::kKVBytes);
#pragma unroll
          for (int r = 0; r < R; ++r)
            tma_load_4d(sK + st * Cfg::kKVBytes + r * N * 128, &p.tm_k, smem_u32(&bar_k_full[st]),
                        r * 64, kcoord, kvh, c.b);
          mbar_arrive_expect_tx(smem_u32(&bar_v_full[st]), Cfg::kKVBytes);
#pragma unroll
          for (int r = 0; r < R; ++r)
            tma_load_4d(sV + st * Cfg::kKVBytes + r * N * 128, &p.tm_v, smem_u32(&bar_v_full[st]),
                        r * 64, kcoord, kvh, c.b);
          ++g;
          if (!more) break;
          cur_kb = cs.kb;
          cur_mask = cs.mask;
          cur_sub = cs.sub;
        }
      }
      // Drain: wait (bounded, ignoring the abort flag) for copies still in flight.
      int zero = 0;
      volatile int* never = &zero;
      const uint32_t n_recent = g < (uint32_t)NST ? g : (uint32_t)NST;
      for (uint32_t i = 0; i < n_recent; ++i) {
        const uint32_t gi = g - 1 - i;
        const int st = gi % NST;
        mbar_wait(smem_u32(&bar_k_full[st]), (gi / NST) & 1, never, nullptr);
        mbar_wait(smem_u32(&bar_v_full[st]), (gi / NST) & 1, never, nullptr);
      }
      if (q_issued > 0) mbar_wait(smem_u32(&bar_q_full), (q_issued - 1) & 1, never, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, N, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, D, true);
      uint32_t g = 0;
      int it = 0;
      bool ok = true;
      auto issue_s = [&](uint32_t gg) {
        const int st = gg % NST;
        const uint32_t d = tmem + 128 + (gg & 1) * 128;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int r = k >> 2, kk = k & 3;
          const uint64_t a = smem_desc_sw128(sQ + r * kTileM * 128 + kk * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(sK + st * Cfg::kKVBytes + r * N * 128 + kk * 32, 16, 1024);
          mma_ss(d, a, b, idesc_s, k > 0 ? 1u : 0u);
        }
      };
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
        if (!(ok = mbar_wait(smem_u32(&bar_q_full), it & 1, abort_v, p.err))) break;
        tc_fence_after();
        int st = g % NST;
        if (!(ok = mbar_wait(smem_u32(&bar_k_full[st]), (g / NST) & 1, abort_v, p.err))) break;
        tc_fence_after();
        int last = meta_last[st];
        issue_s(g);
        mma_commit(smem_u32(&bar_s_full[g & 1]));
        if (last) mma_commit(smem_u32(&bar_q_empty));
        bool first = true;
        while (true) {
          const bool cur_last = last;
          const uint32_t gn = g + 1;
          if (!cur_last) {
            const int stn = gn % NST;
            if (!(ok = mbar_wait(smem_u32(&bar_k_full[stn]), (gn / NST) & 1, abort_v, p.err))) break;
            tc_fence_after();
            last = meta_last[stn];
            issue_s(gn);
            mma_commit(smem_u32(&bar_s_full[gn & 1]));
            if (last) mma_commit(smem_u32(&bar_q_empty));
          }
          if (!(ok = mbar_wait(smem_u32(&bar_p_full[g & 1]), (g >> 1) & 1, abort_v, p.err))) break;
          if (first && it > 0 &&
              !(ok = mbar_wait(smem_u32(&bar_o_empty), (it - 1) & 1, abort_v, p.err)))
            break;
          if (!(ok = mbar_wait(smem_u32(&bar_v_full[st]), (g / NST) & 1, abort_v, p.err))) break;
          tc_fence_after();
          const uint32_t pbuf = tmem + 128 + (g & 1) * 128;
#pragma unroll
          for (int k = 0; k < N / 16; ++k) {
            const uint64_t b = smem_desc_sw128(sV + st * Cfg::kKVBytes + k * 2048, N * 128, 1024);
            mma_ts(tmem, pbuf + k * 8, b, idesc_pv, (!first || k > 0) ? 1u : 0u);
          }
          mma_commit(smem_u32(&bar_kv_empty[st]));
          mma_commit(smem_u32(&bar_pv_done[g & 1]));
          g = gn;
          st = g % NST;
          first = false;
          if (cur_last) break;
        }
      }
      // Drain this thread's outstanding MMAs before TMEM is released.
      mma_commit(smem_u32(&bar_drain));
      int zero = 0;
      mbar_wait(smem_u32(&bar_drain), 0, &zero, nullptr);
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int wr = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = wr * 32 + lane;
    const uint32_t lane_base = (uint32_t)(wr * 32) << 16;
    const unsigned FULL = 0xffffffffu;
    uint32_t g = 0;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
      const TileCoord c = tile_coord(p, t);
      const int q_local = c.q0 + row;
      const int q_abs = q_local + (p.T_k - p.T_q);
      const bool row_ok = q_local < p.T_q;
      const int seg = p.bs < kTileM ? row / p.bs : 0;
      float m_ref = -INFINITY;
      float l = 0.f;
      bool first = true;
      while (true) {
        const int st = g % NST;
        ok = mbar_wait(smem_u32(&bar_k_full[st]), (g / NST) & 1, abort_v, p.err);
        if (!__all_sync(FULL, ok)) { ok = false; break; }
        const int key0 = meta_key0[st];
        const uint32_t mask = meta_mask[st];
        const int last = meta_last[st];
        ok = mbar_wait(smem_u32(&bar_s_full[g & 1]), (g >> 1) & 1, abort_v, p.err);
        if (!__all_sync(FULL, ok)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sbuf = tmem + lane_base + 128 + (g & 1) * 128;
        float s[N];
        if constexpr (N >= 32) {
#pragma unroll
          for (int cc = 0; cc < N / 32; ++cc) {
            uint32_t r32[32];
            tmem_ld32(sbuf + cc * 32, r32);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) s[cc * 32 + i] = __uint_as_float(r32[i]);
          }
        } else {
          uint32_t r16[16];
          tmem_ld16(sbuf, r16);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) s[i] = __uint_as_float(r16[i]);
        }
        const bool mine = row_ok && ((mask >> seg) & 1u);
        const bool full_ok = mine && (key0 + N - 1 <= q_abs) && (key0 + N <= p.T_k);
        float mblk = -INFINITY;
        if (full_ok) {
#pragma unroll
          for (int i = 0; i < N; ++i) {
            s[i] *= p.scale_log2;
            mblk = fmaxf(mblk, s[i]);
          }
        } else {
          const int lim = min(q_abs, p.T_k - 1) - key0;  // valid columns: i <= lim
#pragma unroll
          for (int i = 0; i < N; ++i) {
            const bool v = mine && (i <= lim);
            s[i] = v ? s[i] * p.scale_log2 : -INFINITY;
            mblk = fmaxf(mblk, s[i]);
          }
        }
        const float m_new = fmaxf(m_ref, mblk);
        if (first) {
          m_ref = m_new;
        } else {
          const bool need = m_new > m_ref + 8.0f;
          if (__any_sync(FULL, need)) {
            // O still holds the previous chunk's PV: wait for it, then rescale.
            ok = mbar_wait(smem_u32(&bar_pv_done[(g - 1) & 1]), ((g - 1) >> 1) & 1, abort_v, p.err);
            if (!__all_sync(FULL, ok)) { ok = false; break; }
            tc_fence_after();
            const float alpha = need ? ex2(m_ref - m_new) : 1.0f;
#pragma unroll
            for (int cc = 0; cc < D / 32; ++cc) {
              uint32_t o32[32];
              tmem_ld32(tmem + lane_base + cc * 32, o32);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o32[i] = __float_as_uint(__uint_as_float(o32[i]) * alpha);
              tmem_st32(tmem + lane_base + cc * 32, o32);
            }
            tmem_wait_st();
            if (need) {
              l *= alpha;
              m_ref = m_new;
            }
          }
        }
        const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
        uint32_t pk[N / 2];
        float rs = 0.f;
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
          const float p0 = ex2(s[2 * i] - m_use);
          const float p1 = ex2(s[2 * i + 1] - m_use);
          rs += p0 + p1;
          pk[i] = pack_bf16(p0, p1);
        }
        l += rs;
        // P (bf16 pairs) overwrites the first N/2 columns of this S buffer.
        if constexpr (N / 2 >= 32) {
#pragma unroll
          for (int cc = 0; cc < N / 64; ++cc) {
            uint32_t w32[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) w32[i] = pk[cc * 32 + i];
            tmem_st32(sbuf + cc * 32, w32);
          }
        } else if constexpr (N / 2 == 16) {
          uint32_t w16[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w16[i] = pk[i];
          tmem_st16(sbuf, w16);
        } else {
          uint32_t w8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w8[i] = pk[i];
          tmem_st8(sbuf, w8);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&bar_p_full[g & 1]));
        ++g;
        first = false;
        if (last) break;
      }
      if (!ok) break;
      // ---------------------------------------------------------------- epilogue
      ok = mbar_wait(smem_u32(&bar_pv_done[(g - 1) & 1]), ((g - 1) >> 1) & 1, abort_v, p.err);
      if (!__all_sync(FULL, ok)) { ok = false; break; }
      tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __nv_bfloat16* orow = p.out + (int64_t)c.b * p.o_sb + (int64_t)c.h * p.o_sh + (int64_t)q_local * p.o_st;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o32[32];
        tmem_ld32(tmem + lane_base + cc * 32, o32);
        tmem_wait_ld();
        if (row_ok) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16(__uint_as_float(o32[2 * i]) * inv, __uint_as_float(o32[2 * i + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&bar_o_empty));
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
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

// 4-D bf16 map over [B, H, T, D] (innermost first: D, T, H, B), box (64, rows, 1, 1).
static int make_map(CUtensorMap* m, const void* base, int B, int H, int T, int D,
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

template <int D, int N>
static int launch_prefill(const PrefillParams& prm, int grid, cudaStream_t stream) {
  using Cfg = PrefillCfg<D, N>;
  static bool attr_set = false;  // per process; the attribute is per function and device-independent
  if (!attr_set) {
    SA_CHECK_CUDA(cudaFuncSetAttribute(prefill_kernel<D, N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Cfg::kSmemBytes));
    attr_set = true;
  }
  prefill_kernel<D, N><<<grid, kThreads, Cfg::kSmemBytes, stream>>>(prm);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

}  // namespace sa

using namespace sa;

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int sa_validate_attn_args(const sa_attn_args* a, bool decode) {
  if (!a) return sa_fail(SA_ERR_INVALID, "args is NULL");
  if (!a->q || !a->k || !a->v || !a->out || !a->pairs || !a->offsets)
    return sa_fail(SA_ERR_INVALID, "NULL tensor pointer");
  if (a->D != 64 && a->D != 128) return sa_fail(SA_ERR_UNSUPPORTED, "head_dim %d unsupported (64 or 128)", a->D);
  if (a->B <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->T_q <= 0 || a->T_k <= 0)
    return sa_fail(SA_ERR_INVALID, "non-positive size (B=%d Hq=%d Hkv=%d T_q=%d T_k=%d)", a->B, a->Hq,
                   a->Hkv, a->T_q, a->T_k);
  if (a->Hq % a->Hkv != 0) return sa_fail(SA_ERR_INVALID, "Hq=%d not a multiple of Hkv=%d", a->Hq, a->Hkv);
  const int bs = a->block_size;
  if (bs < 16 || bs > 512 || (bs & (bs - 1)))
    return sa_fail(SA_ERR_INVALID, "block_size %d must be a power of 2 in [16, 512]", bs);
  if (a->T_q > a->T_k) return sa_fail(SA_ERR_INVALID, "T_q=%d > T_k=%d", a->T_q, a->T_k);
  if (a->pairs_stride <= 0) return sa_fail(SA_ERR_INVALID, "pairs_stride must be positive");
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
    return sa_fail(SA_ERR_INVALID, "q/k/v/out must be 16-byte aligned");
  const int64_t* st[4] = {a->q_strides, a->k_strides, a->v_strides, a->o_strides};
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 3; ++j)
      if (st[i][j] < 0 || (st[i][j] % 8) != 0)
        return sa_fail(SA_ERR_INVALID, "strides must be non-negative multiples of 8 elements (16 B)");
  (void)decode;
  return SA_OK;
}

extern "C" int sa_prefill_fwd(const sa_attn_args* a, sa_stream_t stream_) {
  int rc = sa_validate_attn_args(a, false);
  if (rc) return rc;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int bs = a->block_size;
  const int N = bs >= 128 ? 128 : bs;
  PrefillParams prm;
  memset(&prm, 0, sizeof(prm));
  if ((rc = make_map(&prm.tm_q, a->q, a->B, a->Hq, a->T_q, a->D, a->q_strides, kTileM, "q"))) return rc;
  if ((rc = make_map(&prm.tm_k, a->k, a->B, a->Hkv, a->T_k, a->D, a->k_strides, N, "k"))) return rc;
  if ((rc = make_map(&prm.tm_v, a->v, a->B, a->Hkv, a->T_k, a->D, a->v_strides, N, "v"))) return rc;
  prm.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  prm.o_sb = a->o_strides[0];
  prm.o_sh = a->o_strides[1];
  prm.o_st = a->o_strides[2];
  prm.pairs = a->pairs;
  prm.offsets = a->offsets;
  prm.pairs_stride = a->pairs_stride;
  prm.B = a->B;
  prm.Hq = a->Hq;
  prm.Hkv = a->Hkv;
  prm.T_q = a->T_q;
  prm.T_k = a->T_k;
  prm.bs = bs;
  prm.nqb = (a->T_q + bs - 1) / bs;
  prm.nqt = (a->T_q + kTileM - 1) / kTileM;
  prm.group = a->Hq / a->Hkv;
  prm.scale_log2 = a->scale * 1.4426950408889634f;
  prm.err = sa_device_error_ptr();
  const int64_t ntiles = (int64_t)prm.nqt * a->B * a->Hq;
  if (ntiles > 0x7fffffff) return sa_fail(SA_ERR_INVALID, "too many tiles");
  int sms = a->num_sms > 0 ? a->num_sms : sa_num_sms();
  if (sms <= 0) return sa_fail(SA_ERR_CUDA, "cannot query SM count");
  const int grid = (int)(ntiles < sms ? ntiles : sms);
  switch (a->D * 1000 + N) {
    case 128128: return launch_prefill<128, 128>(prm, grid, stream);
    case 128064: return launch_prefill<128, 64>(prm, grid, stream);
    case 128032: return launch_prefill<128, 32>(prm, grid, stream);
    case 128016: return launch_prefill<128, 16>(prm, grid, stream);
    case 64128: return launch_prefill<64, 128>(prm, grid, stream);
    case 64064: return launch_prefill<64, 64>(prm, grid, stream);
    case 64032: return launch_prefill<64, 32>(prm, grid, stream);
    case 64016: return launch_prefill<64, 16>(prm, grid, stream);
  }
  return sa_fail(SA_ERR_UNSUPPORTED, "no kernel for D=%d chunk=%d", a->D, N);
}
