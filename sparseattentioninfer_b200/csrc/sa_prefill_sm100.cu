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
#include <cstdlib>
#include <cstring>

#include "sa_common.cuh"

namespace sa {

// Lanes per transpose group of the epilogue stores (4 or 8; 4 measured faster:
// 997 against 980 TFLOP/s on config 2 in the same run).
#ifndef SA_EPI_GROUP
#define SA_EPI_GROUP 4
#endif

#ifdef SA_PHASE_TRACE
// Debug-only phase timestamps (clock64) of CTA 0: 16 slots per chunk step.
__device__ unsigned long long g_sa_trace[16 * 512];
#define SA_TRACE(step, slot)                                                           \
  do {                                                                                 \
    if (blockIdx.x == 0 && (step) < 512) g_sa_trace[(step) * 16 + (slot)] = clock64(); \
  } while (0)
__device__ unsigned long long g_sa_cta_trace[1024 * 2];
#else
#define SA_TRACE(step, slot) \
  do {                       \
  } while (0)
#endif

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
  int32_t qt_tail;   // (b, head) pairs at the end visited query-tile-major (see tile_coord)
  float scale_log2;
  int32_t* err;
  uint32_t* sched;  // {next tile, CTAs finished} of this launch's scheduler slot
};

constexpr int kTileRing = 4;  // warp 0 producer, warp 1 MMA issuer, warps 2..5 softmax
constexpr int kTileM = 128;
constexpr int kMaxSeg = 8;  // 128 / 16
// Chunk metadata ring. The producer runs at most kKStages chunks ahead of the
// S=QK^T MMA, which runs at most 2 chunks ahead of the softmax, so a slot is
// never rewritten before the softmax has read it.
constexpr int kMetaRing = 16;

template <int D, int N, int CTAS, int LANES>
struct PrefillCfg {
  static constexpr int kRegions = D / 64;               // 64-column (128 B) slabs
  static constexpr int kQBytes = kTileM * D * 2;
  static constexpr int kKVBytes = N * D * 2;            // one K (or V) chunk
  // TMEM per lane: O in columns [0, D), then kSBufs S/P buffers of kSStride
  // columns. With two lanes each lane has one S buffer: the other lane's MMAs
  // fill the tensor core while this lane's softmax runs.
  static constexpr int kSBufs = LANES == 1 ? 2 : 1;
  static constexpr int kSStride = N < 32 ? 32 : N;
  static constexpr int kLaneNeed = D + kSBufs * kSStride;
  static constexpr int kLaneCols = kLaneNeed <= 32 ? 32 : kLaneNeed <= 64 ? 64 : kLaneNeed <= 128 ? 128
                                   : kLaneNeed <= 256 ? 256 : 512;
  static constexpr int kTmemCols = kLaneCols * LANES;
  static_assert(kTmemCols * CTAS <= 512, "TMEM over-subscribed");
  // 228 KB of shared memory per SM, of which 1 KB per resident CTA is reserved
  // by the hardware; static shared data is kept under LANES KB.
  static constexpr int kSmemBudget = (233472 / CTAS) - 1024 - 1024 * LANES;
  static constexpr int kLaneBudget = kSmemBudget / LANES;
  static constexpr int kBufs = (kLaneBudget - kQBytes) / kKVBytes;  // K + V chunk buffers per lane
  // V is consumed a whole softmax later than K (PV after P, S as soon as K
  // lands), so the odd buffer goes to V: measured 2 K + 3 V at 64-key chunks
  // against 3 K + 2 V, period 1,964 -> 1,673 cycles per chunk.
  static constexpr int kKHalf = kBufs / 2;
  static constexpr int kKStages = kKHalf > 4 ? 4 : kKHalf;
  static constexpr int kVStages = (kBufs - kKStages) > 4 ? 4 : (kBufs - kKStages);
  static constexpr int kLaneBytes = kQBytes + (kKStages + kVStages) * kKVBytes;
  static constexpr int kSmemBytes = kLaneBytes * LANES;
  static_assert(kVStages >= 1 && kKStages >= 1, "not enough shared memory for the K/V rings");
  // With two S buffers the MMA issuer puts S of chunk g+1 in before PV of chunk
  // g, which needs K of g+1 resident while K of g is still being consumed.
  static_assert(kSBufs == 1 || kKStages >= 2, "two S buffers need two K stages");
  static_assert(kKStages + 3 < kMetaRing, "meta ring too short");
  static constexpr int kThreads = LANES * 192;  // per lane: producer, MMA issuer, 4 softmax warps
};

// Chunk stream of one tile: sorted union of up to kMaxSeg CSR rows, each key
// block expanded into `nsub` chunks of N keys. Each segment keeps its current
// and next index in registers and the load of the one after is issued a whole
// chunk before it is needed (unconditional, at a clamped index: a select on a
// load result would stall the producer on every chunk).
struct ChunkStream {
  const int32_t* pairs;
  int ptr[kMaxSeg];
  int end[kMaxSeg];
  int headv[kMaxSeg];
  int nextv[kMaxSeg];
  int nseg;
  int nsub;
  int sub;
  int kb;
  uint32_t mask;

  __device__ __forceinline__ static int clamp_idx(int i, int e) { return max(0, min(i, e - 1)); }

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
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s) {
      headv[s] = __ldg(pairs + clamp_idx(ptr[s], end[s]));
      nextv[s] = __ldg(pairs + clamp_idx(ptr[s] + 1, end[s]));
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
      if (s < nseg && ptr[s] < end[s]) best = min(best, headv[s]);
    if (best == 0x7fffffff) return false;
    uint32_t m = 0;
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s)
      if (s < nseg && ptr[s] < end[s] && headv[s] == best) {
        m |= 1u << s;
        ++ptr[s];
        headv[s] = nextv[s];
        nextv[s] = __ldg(pairs + clamp_idx(ptr[s] + 1, end[s]));
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

// Head-major order (consecutive tiles share one (b, head), so its K/V stays in
// L2), heaviest (last) query tile of each head first — except for the last
// qt_tail (b, head) pairs, which are visited query-tile-major: the heaviest
// tiles of all of them first, the lightest last. Otherwise the heavy tiles of
// the last heads would start when the other CTAs are running dry and set the
// launch's tail. Their K/V (qt_tail heads) is sized to stay in L2.
template <int N>
__device__ __forceinline__ TileCoord tile_coord(const PrefillParams& p, int t) {
  const int nbh = p.B * p.Hq;
  const int head_tiles = (nbh - p.qt_tail) * p.nqt;
  int bh, qt;
  if (t < head_tiles) {
    bh = t / p.nqt;
    qt = p.nqt - 1 - t % p.nqt;
  } else {
    const int u = t - head_tiles;
    bh = nbh - p.qt_tail + u % p.qt_tail;
    qt = p.nqt - 1 - u / p.qt_tail;
  }
  TileCoord c;
  c.b = bh / p.Hq;
  c.h = bh % p.Hq;
  c.q0 = qt * kTileM;
  c.qb0 = c.q0 / p.bs;
  c.nseg = p.bs < kTileM ? min(kTileM / p.bs, p.nqb - c.qb0) : 1;
  c.nsub = p.bs > N ? p.bs / N : 1;
  return c;
}

// One lane = one tile at a time through its own producer, K/V rings, MMA
// issuer and softmax warpgroup. Warps of lane L: 6L producer, 6L+1 MMA issuer,
// 6L+2 .. 6L+5 softmax (their warp index mod 4 covers the four TMEM lane
// quadrants). With LANES = 2 the two lanes' MMAs interleave on the tensor core.
template <int D, int N, int CTAS, int LANES>
__global__ void __launch_bounds__(LANES * 192, CTAS) prefill_kernel(const __grid_constant__ PrefillParams p) {
  using Cfg = PrefillCfg<D, N, CTAS, LANES>;
  constexpr uint32_t SB = D;                  // first S/P buffer column (within a lane)
  constexpr uint32_t SS = Cfg::kSStride;      // S/P buffer stride (columns)
  constexpr int NSB = Cfg::kSBufs;
  constexpr int NSK = Cfg::kKStages;
  constexpr int NSV = Cfg::kVStages;
  constexpr int R = Cfg::kRegions;

  __shared__ __align__(8) uint64_t bar_q_full[LANES], bar_q_empty[LANES], bar_o_empty[LANES], bar_drain[LANES];
  __shared__ __align__(8) uint64_t bar_k_full[LANES][NSK], bar_k_empty[LANES][NSK];
  __shared__ __align__(8) uint64_t bar_v_full[LANES][NSV], bar_v_empty[LANES][NSV];
  __shared__ __align__(8) uint64_t bar_p_full[LANES][2];
  __shared__ __align__(8) uint64_t bar_meta[LANES][kMetaRing];
  __shared__ __align__(8) uint64_t bar_tile[LANES][kTileRing];
  __shared__ int meta_key0[LANES][kMetaRing];
  __shared__ uint32_t meta_mask[LANES][kMetaRing];
  __shared__ int meta_last[LANES][kMetaRing];
  __shared__ int tile_ring[LANES][kTileRing];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  // Dynamic shared memory per lane: Q | K ring | V ring, 1024-byte aligned for SWIZZLE_128B.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int L = warp / 6;        // tile lane of this warp
  const int role = warp % 6;     // 0 producer, 1 MMA issuer, 2..5 softmax
  const uint32_t sQ = smem_u32(smem_raw) + L * Cfg::kLaneBytes;
  const uint32_t sK = sQ + Cfg::kQBytes;
  const uint32_t sV = sK + NSK * Cfg::kKVBytes;
  const int ntiles = p.nqt * p.B * p.Hq;
  const bool misaligned = (smem_u32(smem_raw) & 1023u) != 0;
#ifdef SA_PHASE_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) {
    unsigned long long t_;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));
    g_sa_cta_trace[blockIdx.x * 2] = t_;
  }
#endif

  if (threadIdx.x == 0) {
    if (misaligned) record_error(p.err, SA_DEV_ERR_INDEX);
    for (int l = 0; l < LANES; ++l) {
      mbar_init(smem_u32(&bar_q_full[l]), 1);
      mbar_init(smem_u32(&bar_q_empty[l]), 1);
      mbar_init(smem_u32(&bar_o_empty[l]), 128);
      mbar_init(smem_u32(&bar_drain[l]), 1);
      for (int i = 0; i < NSK; ++i) {
        mbar_init(smem_u32(&bar_k_full[l][i]), 1);
        mbar_init(smem_u32(&bar_k_empty[l][i]), 1);
      }
      for (int i = 0; i < NSV; ++i) {
        mbar_init(smem_u32(&bar_v_full[l][i]), 1);
        mbar_init(smem_u32(&bar_v_empty[l][i]), 1);
      }
      for (int i = 0; i < kMetaRing; ++i) mbar_init(smem_u32(&bar_meta[l][i]), 1);
      for (int i = 0; i < kTileRing; ++i) mbar_init(smem_u32(&bar_tile[l][i]), 1);
      for (int i = 0; i < 2; ++i) mbar_init(smem_u32(&bar_p_full[l][i]), 128);
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
    tmem_alloc(smem_u32(&tmem_base_sh), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh + L * Cfg::kLaneCols;
  volatile int* abort_v = &abort_flag;

  if (misaligned) {
    // dynamic shared memory not 1024-byte aligned (recorded above): do nothing
  } else if (role == 0) {
    // ------------------------------------------------------------------ producer
    // One thread. Dynamic schedule: tiles come in order from the launch's
    // counter (head-major, heaviest tile of a head first) and are published to
    // this lane's MMA and softmax warps through the tile ring; -1 ends the lane.
    // Per chunk: metadata (+ its barrier), K into the K ring once its slot's
    // S=QK^T retired, V into the V ring once its slot's PV retired.
    if (lane == 0) {
      uint32_t g = 0;
      int it = 0, q_issued = 0;
      bool ok = true;
      for (;; ++it) {
        int t = (int)atomicAdd(&p.sched[0], 1u);
        if (t >= ntiles) t = -1;
        tile_ring[L][it % kTileRing] = t;
        mbar_arrive(smem_u32(&bar_tile[L][it % kTileRing]));
        if (t < 0) break;
        const TileCoord c = tile_coord<N>(p, t);
        const int kvh = c.h / p.group;
        if (it > 0 && !(ok = mbar_wait(smem_u32(&bar_q_empty[L]), (it - 1) & 1, abort_v, p.err))) break;
        mbar_arrive_expect_tx(smem_u32(&bar_q_full[L]), Cfg::kQBytes);
#pragma unroll
        for (int r = 0; r < R; ++r)
          tma_load_4d(sQ + r * kTileM * 128, &p.tm_q, smem_u32(&bar_q_full[L]), r * 64, c.q0, c.h, c.b);
        if (L == 0) SA_TRACE(g, 15);
        ++q_issued;
        ChunkStream cs;
        cs.init(p, c.h, c.qb0, c.nseg, c.nsub);
        bool have = cs.next();
        int cur_kb = have ? cs.kb : 0;
        uint32_t cur_mask = have ? cs.mask : 0u;  // empty tile: one fully masked chunk
        int cur_sub = have ? cs.sub : 0;
        while (true) {
          const bool more = have && cs.next();
          int key0 = cur_kb * p.bs + cur_sub * N;
          if (cur_kb < 0 || cur_kb >= (0x7fffffff / max(p.bs, 1))) {
            record_error(p.err, SA_DEV_ERR_INDEX);  // malformed index: load block 0, mask all
            key0 = 0;
            cur_mask = 0;
          }
          const int kcoord = min(key0, p.T_k);  // fully out-of-range chunks read zeros
          const int ks = g % NSK, vs = g % NSV, ms = g % kMetaRing;
          if (g >= (uint32_t)NSK &&
              !(ok = mbar_wait(smem_u32(&bar_k_empty[L][ks]), ((g / NSK) - 1) & 1, abort_v, p.err)))
            break;
          meta_key0[L][ms] = key0;
          meta_mask[L][ms] = cur_mask;
          meta_last[L][ms] = more ? 0 : 1;
          mbar_arrive(smem_u32(&bar_meta[L][ms]));
          mbar_arrive_expect_tx(smem_u32(&bar_k_full[L][ks]), Cfg::kKVBytes);
#pragma unroll
          for (int r = 0; r < R; ++r)
            tma_load_4d(sK + ks * Cfg::kKVBytes + r * N * 128, &p.tm_k, smem_u32(&bar_k_full[L][ks]), r * 64,
                        kcoord, kvh, c.b);
          if (L == 0) SA_TRACE(g, 13);
          if (g >= (uint32_t)NSV &&
              !(ok = mbar_wait(smem_u32(&bar_v_empty[L][vs]), ((g / NSV) - 1) & 1, abort_v, p.err)))
            break;
          mbar_arrive_expect_tx(smem_u32(&bar_v_full[L][vs]), Cfg::kKVBytes);
#pragma unroll
          for (int r = 0; r < R; ++r)
            tma_load_4d(sV + vs * Cfg::kKVBytes + r * N * 128, &p.tm_v, smem_u32(&bar_v_full[L][vs]), r * 64,
                        kcoord, kvh, c.b);
          if (L == 0) SA_TRACE(g, 14);
          ++g;
          if (!more) break;
          cur_kb = cs.kb;
          cur_mask = cs.mask;
          cur_sub = cs.sub;
        }
        if (!ok) break;
      }
      // Drain: wait (bounded, ignoring the abort flag) for copies still in flight.
      int zero = 0;
      volatile int* never = &zero;
      for (uint32_t i = 0; i < (g < (uint32_t)NSK ? g : (uint32_t)NSK); ++i) {
        const uint32_t gi = g - 1 - i;
        mbar_wait(smem_u32(&bar_k_full[L][gi % NSK]), (gi / NSK) & 1, never, nullptr);
      }
      for (uint32_t i = 0; i < (g < (uint32_t)NSV ? g : (uint32_t)NSV); ++i) {
        const uint32_t gi = g - 1 - i;
        mbar_wait(smem_u32(&bar_v_full[L][gi % NSV]), (gi / NSV) & 1, never, nullptr);
      }
      if (q_issued > 0) mbar_wait(smem_u32(&bar_q_full[L]), (q_issued - 1) & 1, never, nullptr);
    }
  } else if (role == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, N, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, D, true);
      // Descriptors are built once; an operand's start address is a constant
      // offset (16-byte units) added to the base descriptor.
      const uint64_t q_desc = smem_desc_sw128(sQ, 16, 1024);
      const uint64_t k_desc = smem_desc_sw128(sK, 16, 1024);
      const uint64_t v_desc = smem_desc_sw128(sV, N * 128, 1024);
      uint32_t g = 0;
      int it = 0;
      bool ok = true;
      // S = Q K^T for chunk gg. Its commit on the K slot both frees the slot
      // and tells the softmax that S is in TMEM.
      auto issue_s = [&](uint32_t gg) {
        const int ks = gg % NSK;
        const uint32_t d = tmem + SB + (gg % NSB) * SS;
        const uint64_t kst = k_desc + (uint64_t)((ks * Cfg::kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int r = k >> 2, kk = k & 3;
          mma_ss(d, q_desc + ((r * kTileM * 128 + kk * 32) >> 4), kst + ((r * N * 128 + kk * 32) >> 4), idesc_s,
                 k > 0 ? 1u : 0u);
        }
        mma_commit(smem_u32(&bar_k_empty[L][ks]));
        if (L == 0) SA_TRACE(gg, 5);
      };
      // Wait for K of chunk gg, then issue its S (and release Q after the tile's last S).
      auto next_s = [&](uint32_t gg, int& last) -> bool {
        if (!mbar_wait(smem_u32(&bar_k_full[L][gg % NSK]), (gg / NSK) & 1, abort_v, p.err)) return false;
        tc_fence_after();
        last = meta_last[L][gg % kMetaRing];
        issue_s(gg);
        if (last) mma_commit(smem_u32(&bar_q_empty[L]));
        return true;
      };
      for (;; ++it) {
        if (!(ok = mbar_wait(smem_u32(&bar_tile[L][it % kTileRing]), (it / kTileRing) & 1, abort_v, p.err))) break;
        if (tile_ring[L][it % kTileRing] < 0) break;
        if (!(ok = mbar_wait(smem_u32(&bar_q_full[L]), it & 1, abort_v, p.err))) break;
        if (L == 0) SA_TRACE(g, 12);
        tc_fence_after();
        int last = 0;
        const uint32_t g0 = g;
        if (!(ok = next_s(g0, last))) break;
        while (true) {
          const bool cur_last = last;
          // Two S buffers: S of the next chunk goes in before this chunk's PV.
          if (NSB == 2 && !cur_last && !(ok = next_s(g + 1, last))) break;
          if (!(ok = mbar_wait(smem_u32(&bar_p_full[L][g & 1]), (g >> 1) & 1, abort_v, p.err))) break;
          if (L == 0) SA_TRACE(g, 6);
          if (g == g0 && it > 0 &&
              !(ok = mbar_wait(smem_u32(&bar_o_empty[L]), (it - 1) & 1, abort_v, p.err)))
            break;
          const int vs = g % NSV;
          if (!(ok = mbar_wait(smem_u32(&bar_v_full[L][vs]), (g / NSV) & 1, abort_v, p.err))) break;
          tc_fence_after();
          const uint32_t pbuf = tmem + SB + (g % NSB) * SS;
          const uint64_t vst = v_desc + (uint64_t)((vs * Cfg::kKVBytes) >> 4);
          const uint32_t acc0 = g != g0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < N / 16; ++k)
            mma_ts(tmem, pbuf + k * 8, vst + ((k * 2048) >> 4), idesc_pv, k > 0 ? 1u : acc0);
          mma_commit(smem_u32(&bar_v_empty[L][vs]));  // PV_g retired: V slot free, O holds chunk g
          if (L == 0) SA_TRACE(g, 7);
          // One S buffer: the next S reuses it once this PV (reading P) is issued.
          if (NSB == 1 && !cur_last && !(ok = next_s(g + 1, last))) break;
          ++g;
          if (cur_last) break;
        }
        if (!ok) break;
      }
      // Drain this thread's outstanding MMAs before TMEM is released.
      mma_commit(smem_u32(&bar_drain[L]));
      int zero = 0;
      mbar_wait(smem_u32(&bar_drain[L]), 0, &zero, nullptr);
    }
  } else {
    // ------------------------------------------------------------------ softmax
    // "S_j in TMEM" is completion of K slot j%NSK and "PV_j retired" that of V
    // slot j%NSV: neither can advance a second phase before this warpgroup has
    // consumed chunk j, so the parity waits are exact.
    // S is read in two passes of 64-column halves (row max, then exponentials
    // and P) so that no thread holds a whole 128-column row in registers.
    constexpr int HALF = N >= 64 ? 64 : N;  // columns per pass step
    const int wr = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = wr * 32 + lane;
    const uint32_t lane_base = (uint32_t)(wr * 32) << 16;
    const unsigned FULL = 0xffffffffu;
    uint32_t g = 0;
    int it = 0;
    bool ok = true;
    for (;; ++it) {
      ok = mbar_wait(smem_u32(&bar_tile[L][it % kTileRing]), (it / kTileRing) & 1, abort_v, p.err);
      if (!__all_sync(FULL, ok)) break;
      const int t = tile_ring[L][it % kTileRing];
      if (t < 0) break;
      const TileCoord c = tile_coord<N>(p, t);
      const int q_local = c.q0 + row;
      const int q_abs = q_local + (p.T_k - p.T_q);
      const bool row_ok = q_local < p.T_q;
      const int seg = p.bs < kTileM ? row / p.bs : 0;
      float m_ref = -INFINITY;
      float l = 0.f;
      bool first = true;
      while (true) {
        const int ms = g % kMetaRing;
        if (L == 0 && threadIdx.x == 64) SA_TRACE(g, 8);
        ok = mbar_wait(smem_u32(&bar_meta[L][ms]), (g / kMetaRing) & 1, abort_v, p.err);
        if (L == 0 && threadIdx.x == 64) SA_TRACE(g, 9);
        if (!__all_sync(FULL, ok)) { ok = false; break; }
        const int key0 = meta_key0[L][ms];
        const uint32_t mask = meta_mask[L][ms];
        const int last = meta_last[L][ms];
        if (L == 0 && threadIdx.x == 64) SA_TRACE(g, 0);
        ok = mbar_wait(smem_u32(&bar_k_empty[L][g % NSK]), (g / NSK) & 1, abort_v, p.err);
        if (L == 0 && threadIdx.x == 64) SA_TRACE(g, 1);
        if (!__all_sync(FULL, ok)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sbuf = tmem + lane_base + SB + (g % NSB) * SS;
        const bool mine = row_ok && ((mask >> seg) & 1u);
        const bool full_ok = mine && (key0 + N - 1 <= q_abs) && (key0 + N <= p.T_k);
        const int lim = min(q_abs, p.T_k - 1) - key0;  // valid columns: i <= lim
        // Load columns [h0, h0 + HALF) of S, masked when needed.
        auto load_half = [&](int h0, float (&s)[HALF]) {
          if constexpr (HALF >= 32) {
            uint32_t r32[HALF / 32][32];
#pragma unroll
            for (int cc = 0; cc < HALF / 32; ++cc) tmem_ld32(sbuf + h0 + cc * 32, r32[cc]);
            tmem_wait_ld();
#pragma unroll
            for (int cc = 0; cc < HALF / 32; ++cc) {
              reg_fence32(r32[cc]);
#pragma unroll
              for (int i = 0; i < 32; ++i) s[cc * 32 + i] = __uint_as_float(r32[cc][i]);
            }
          } else {
            uint32_t r16[16];
            tmem_ld16(sbuf + h0, r16);
            tmem_wait_ld();
            reg_fence16(r16);
#pragma unroll
            for (int i = 0; i < 16; ++i) s[i] = __uint_as_float(r16[i]);
          }
          if (!full_ok) {
#pragma unroll
            for (int i = 0; i < HALF; ++i) s[i] = (mine && h0 + i <= lim) ? s[i] : -INFINITY;
          }
        };
        // Pass 1: raw-score row max (three-input max chains; the positive
        // scale is folded into the exponent below). With one pass step
        // (N <= 64) the scores stay in registers for pass 2.
        constexpr bool kOneStep = (N <= HALF);
        float s_keep[kOneStep ? HALF : 1];
        float mraw = -INFINITY;
#pragma unroll 1
        for (int h0 = 0; h0 < N; h0 += HALF) {
          float s_loc[kOneStep ? 1 : HALF];
          float (&s)[kOneStep ? HALF : HALF] = *reinterpret_cast<float (*)[HALF]>(kOneStep ? s_keep : s_loc);
          load_half(h0, s);
          float mx8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = s[i];
#pragma unroll
          for (int i = 8; i < HALF; i += 2) mx8[(i >> 1) & 7] = max3(mx8[(i >> 1) & 7], s[i], s[i + 1]);
          mraw = max3(mraw, fmaxf(max3(mx8[0], mx8[1], mx8[2]), mx8[3]), max3(mx8[4], mx8[5], fmaxf(mx8[6], mx8[7])));
        }
        if (L == 0 && threadIdx.x == 64) SA_TRACE(g, 2);
        const float m_new = fmaxf(m_ref, mraw * p.scale_log2);
        if (first) {
          m_ref = m_new;
        } else {
          const bool need = m_new > m_ref + 8.0f;
          if (__any_sync(FULL, need)) {
            // O still holds the previous chunk's PV: wait for it, then rescale.
            ok = mbar_wait(smem_u32(&bar_v_empty[L][(g - 1) % NSV]), ((g - 1) / NSV) & 1, abort_v, p.err);
            if (!__all_sync(FULL, ok)) { ok = false; break; }
            tc_fence_after();
            const float alpha = need ? ex2(m_ref - m_new) : 1.0f;
#pragma unroll
            for (int cc = 0; cc < D / 32; ++cc) {
              uint32_t o32[32];
              tmem_ld32(tmem + lane_base + cc * 32, o32);
              tmem_wait_ld();
              reg_fence32(o32);
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
        const uint64_t sc2 = f2pack(p.scale_log2, p.scale_log2), nm2 = f2pack(-m_use, -m_use);
        uint64_t rs4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) rs4[i] = 0ull;
        // Pass 2: exponentials, row sum, and P (bf16 pairs) written over the
        // first N/2 columns of this S buffer, HALF/2 columns per step (those
        // columns were read by this or the previous step).
#pragma unroll 1
        for (int h0 = 0; h0 < N; h0 += HALF) {
          float s_loc[kOneStep ? 1 : HALF];
          float (&s)[HALF] = *reinterpret_cast<float (*)[HALF]>(kOneStep ? s_keep : s_loc);
          if constexpr (!kOneStep) load_half(h0, s);
          uint32_t pk[HALF / 2];
#pragma unroll
          for (int i = 0; i < HALF / 2; ++i) {
            float x0, x1;
            f2unpack(fma2(f2pack(s[2 * i], s[2 * i + 1]), sc2, nm2), x0, x1);
            const float p0 = ex2(x0), p1 = ex2(x1);
            rs4[i & 3] = add2(rs4[i & 3], f2pack(p0, p1));
            pk[i] = pack_bf16(p0, p1);
          }
          const uint32_t pdst = sbuf + h0 / 2;
          if constexpr (HALF / 2 >= 32) {
            tmem_st32(pdst, pk);
          } else if constexpr (HALF / 2 == 16) {
            tmem_st16(pdst, pk);
          } else {
            tmem_st8(pdst, pk);
          }
        }
        {
          float a0, a1, b0, b1;
          f2unpack(add2(rs4[0], rs4[1]), a0, a1);
          f2unpack(add2(rs4[2], rs4[3]), b0, b1);
          l += (a0 + a1) + (b0 + b1);
        }
        if (L == 0 && threadIdx.x == 64) SA_TRACE(g, 3);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&bar_p_full[L][g & 1]));
        if (L == 0 && threadIdx.x == 64) SA_TRACE(g, 4);
        ++g;
        first = false;
        if (last) break;
      }
      if (!ok) break;
      // ---------------------------------------------------------------- epilogue
      ok = mbar_wait(smem_u32(&bar_v_empty[L][(g - 1) % NSV]), ((g - 1) / NSV) & 1, abort_v, p.err);
      if (L == 0 && threadIdx.x == 64) SA_TRACE(g - 1, 10);
      if (!__all_sync(FULL, ok)) { ok = false; break; }
      tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __nv_bfloat16* orow = p.out + (int64_t)c.b * p.o_sb + (int64_t)c.h * p.o_sh + (int64_t)q_local * p.o_st;
      const bool out32 = (reinterpret_cast<uintptr_t>(orow) & 31u) == 0;
      uint32_t o32[D / 32][32];
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) tmem_ld32(tmem + lane_base + cc * 32, o32[cc]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(smem_u32(&bar_o_empty[L]));  // O is in registers: the next tile may overwrite TMEM
      if constexpr (D == 128) {
        // One thread owns one TMEM lane = one row. Pack the row to bf16, then
        // transpose row chunks inside groups of TG lanes (log2(TG) shfl_xor
        // butterfly stages): lane j of a group ends up with chunk j of each of
        // the group's TG rows, so a store instruction writes whole rows of the
        // group instead of one 32-byte piece of 32 rows.
        constexpr int TG = SA_EPI_GROUP;  // lanes per transpose group
        constexpr int CW = 64 / TG;       // 32-bit words per chunk
        uint32_t u[64];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          reg_fence32(o32[cc]);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            u[cc * 16 + i] =
                pack_bf16(__uint_as_float(o32[cc][2 * i]) * inv, __uint_as_float(o32[cc][2 * i + 1]) * inv);
        }
        const int j = lane % TG;
#pragma unroll
        for (int m = 1; m < TG; m <<= 1) {
          const bool jb = (j & m) != 0;
#pragma unroll
          for (int c0 = 0; c0 < TG; ++c0) {
            if (c0 & m) continue;
            const int c1 = c0 | m;
#pragma unroll
            for (int i = 0; i < CW; ++i) {
              const uint32_t r = __shfl_xor_sync(FULL, jb ? u[c0 * CW + i] : u[c1 * CW + i], m);
              if (jb)
                u[c0 * CW + i] = r;
              else
                u[c1 * CW + i] = r;
            }
          }
        }
        // lane j of a group now holds, in slot k, chunk j (CW words) of the group's row k
        const int gq = lane / TG;
#pragma unroll
        for (int kk = 0; kk < TG; ++kk) {
          const int r_local = c.q0 + wr * 32 + gq * TG + kk;
          if (r_local < p.T_q) {
            __nv_bfloat16* dst =
                p.out + (int64_t)c.b * p.o_sb + (int64_t)c.h * p.o_sh + (int64_t)r_local * p.o_st + j * (2 * CW);
            if ((reinterpret_cast<uintptr_t>(dst) & 31u) == 0) {
#pragma unroll
              for (int v8 = 0; v8 < CW / 8; ++v8) st_global_v8(dst + 16 * v8, u + kk * CW + 8 * v8);
            } else {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int i = 0; i < CW / 4; ++i)
                d4[i] = make_uint4(u[kk * CW + 4 * i], u[kk * CW + 4 * i + 1], u[kk * CW + 4 * i + 2],
                                   u[kk * CW + 4 * i + 3]);
            }
          }
        }
      } else {
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          reg_fence32(o32[cc]);
          if (row_ok) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              w[i] = pack_bf16(__uint_as_float(o32[cc][2 * i]) * inv, __uint_as_float(o32[cc][2 * i + 1]) * inv);
            __nv_bfloat16* dst = orow + cc * 32;
            if (out32) {
              st_global_v8(dst, w);
              st_global_v8(dst + 16, w + 8);
            } else {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            }
          }
        }
      }
      if (L == 0 && threadIdx.x == 64) SA_TRACE(g - 1, 11);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base_sh, Cfg::kTmemCols);
  if (threadIdx.x == 0) {
    // The last CTA to finish rearms the scheduler slot for a later launch.
    __threadfence();
    if (atomicAdd(&p.sched[1], 1u) == gridDim.x - 1) {
      p.sched[0] = 0;
      p.sched[1] = 0;
      __threadfence();
    }
  }
#ifdef SA_PHASE_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) {
    unsigned long long t_;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));
    g_sa_cta_trace[blockIdx.x * 2 + 1] = t_;
  }
#endif
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Scheduler slots: {next tile, CTAs finished} per launch, zero between launches
// (the last CTA of a launch resets its slot). Launches take slots round robin,
// so up to kSchedSlots prefill launches may be in flight at once on a device.
constexpr int kSchedSlots = 64;
__device__ uint32_t g_sa_sched[kSchedSlots][2];

static int sched_slot(uint32_t** out) {
  static uint32_t* base[64] = {nullptr};
  static unsigned seq[64] = {0};
  int dev = 0;
  SA_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return sa_fail(SA_ERR_UNSUPPORTED, "device index %d out of range", dev);
  if (!base[dev]) {
    void* p = nullptr;
    SA_CHECK_CUDA(cudaGetSymbolAddress(&p, g_sa_sched));
    base[dev] = static_cast<uint32_t*>(p);
  }
  *out = base[dev] + 2 * (__sync_fetch_and_add(&seq[dev], 1u) % kSchedSlots);
  return SA_OK;
}

template <int D, int N, int CTAS, int LANES>
static int launch_prefill(const PrefillParams& prm, int64_t ntiles, int sms, cudaStream_t stream) {
  using Cfg = PrefillCfg<D, N, CTAS, LANES>;
  auto kern = prefill_kernel<D, N, CTAS, LANES>;
  SA_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  SA_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  const int64_t slots = (int64_t)sms * CTAS;
  const int grid = (int)(ntiles < slots ? ntiles : slots);
  kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(prm);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

}  // namespace sa

using namespace sa;

static int sa_prefill_chunk() {
  static int v = 0;
  if (!v) {
    const char* e = getenv("SA_PREFILL_CHUNK");
    v = (e && atoi(e) == 128) ? 128 : 64;
  }
  return v;
}

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
  const int chunk = sa_prefill_chunk();
  const int N = bs >= chunk ? chunk : bs;
  PrefillParams prm;
  memset(&prm, 0, sizeof(prm));
  if ((rc = sa_make_map(&prm.tm_q, a->q, a->B, a->Hq, a->T_q, a->D, a->q_strides, kTileM, "q"))) return rc;
  if ((rc = sa_make_map(&prm.tm_k, a->k, a->B, a->Hkv, a->T_k, a->D, a->k_strides, N, "k"))) return rc;
  if ((rc = sa_make_map(&prm.tm_v, a->v, a->B, a->Hkv, a->T_k, a->D, a->v_strides, N, "v"))) return rc;
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
  const int qt_tail_env = getenv("SA_PREFILL_TAIL") ? atoi(getenv("SA_PREFILL_TAIL")) : -1;
  prm.scale_log2 = a->scale * 1.4426950408889634f;
  prm.err = sa_device_error_ptr();
  if ((rc = sched_slot(&prm.sched))) return rc;
  const int64_t ntiles = (int64_t)prm.nqt * a->B * a->Hq;
  if (ntiles > 0x7fffffff) return sa_fail(SA_ERR_INVALID, "too many tiles");
  int sms = a->num_sms > 0 ? a->num_sms : sa_num_sms();
  if (sms <= 0) return sa_fail(SA_ERR_CUDA, "cannot query SM count");
  {
    // Tail visited query-tile-major: enough (b, head) pairs for two tiles per
    // resident CTA, all of them when the launch's K/V stays in L2 (<= 96 MB;
    // measured on config-2 shards: 4 heads 107 -> 86 us).
    const int nbh = a->B * a->Hq;
    const int64_t kv_bytes = 2ll * a->B * a->Hkv * a->T_k * a->D * 2;
    int tail = (int)((2ll * 2 * sms + prm.nqt - 1) / prm.nqt);
    if (kv_bytes <= (96ll << 20)) tail = nbh;
    if (qt_tail_env >= 0) tail = qt_tail_env;
    prm.qt_tail = tail < 1 ? 1 : (tail > nbh ? nbh : tail);
  }
  // Chunk size: 64 keys with two CTAs per SM (default; their softmax
  // warpgroups interleave on the tensor core), or 128 keys with one CTA per SM
  // (SA_PREFILL_CHUNK=128).
  switch (a->D * 10000 + N) {
    case 1280128: return launch_prefill<128, 128, 1, 2>(prm, ntiles, sms, stream);
    case 1280064: return launch_prefill<128, 64, 2, 1>(prm, ntiles, sms, stream);
    case 1280032: return launch_prefill<128, 32, 2, 1>(prm, ntiles, sms, stream);
    case 1280016: return launch_prefill<128, 16, 2, 1>(prm, ntiles, sms, stream);
    case 640128: return launch_prefill<64, 128, 1, 2>(prm, ntiles, sms, stream);
    case 640064: return launch_prefill<64, 64, 2, 1>(prm, ntiles, sms, stream);
    case 640032: return launch_prefill<64, 32, 2, 1>(prm, ntiles, sms, stream);
    case 640016: return launch_prefill<64, 16, 2, 1>(prm, ntiles, sms, stream);
  }
  return sa_fail(SA_ERR_UNSUPPORTED, "no kernel for D=%d chunk=%d", a->D, N);
}

#ifdef SA_PHASE_TRACE
extern "C" SA_API int sa_debug_trace_clear() {
  static unsigned long long zeros[16 * 512];
  SA_CHECK_CUDA(cudaMemcpyToSymbol(sa::g_sa_trace, zeros, sizeof(zeros)));
  return SA_OK;
}
extern "C" SA_API int sa_debug_cta_trace_read(unsigned long long* host, int n) {
  SA_CHECK_CUDA(cudaDeviceSynchronize());
  SA_CHECK_CUDA(cudaMemcpyFromSymbol(host, sa::g_sa_cta_trace, sizeof(unsigned long long) * (n < 2048 ? n : 2048)));
  return SA_OK;
}
extern "C" SA_API int sa_debug_trace_read(unsigned long long* host, int n) {
  SA_CHECK_CUDA(cudaDeviceSynchronize());
  SA_CHECK_CUDA(cudaMemcpyFromSymbol(host, sa::g_sa_trace, sizeof(unsigned long long) * (n < 8192 ? n : 8192)));
  return SA_OK;
}
#endif
