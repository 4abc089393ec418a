// sa_pattern.cu — device-side pattern compiler: BigBird layouts, block bitmaps,
// token masks and legacy padded lists -> per-head block CSR.
//
// Bit-exact with the reference's Python builders:
//   BigBird rows     bigbird_pattern.py:212-271 (BigBirdPattern),
//                    :533-583 (BigBirdKeepRatioPattern, per-KV-group layouts),
//                    :697-753 (BigBird2Pattern, full last row)
//   random blocks    select_bigbird_random_block_ids, bigbird_pattern.py:23-41
//   token mask->CSR  build_block_pairs_from_mask, patterns/base.py:36-89
//   padded -> CSR    kv_block_list_to_pairs, patterns/base.py:92-133
// Every BigBird row is a union of at most four integer ranges (globals, two
// arcs of the rotated random candidates, the window), so rows are counted and
// emitted in closed form; offsets come from one block-wide scan per head.
#include <cstring>

#include "sa_common.cuh"

namespace sa {

constexpr int kMaxGroups = 64;

struct BigBirdParams {
  int32_t g[kMaxGroups], w[kMaxGroups], r[kMaxGroups];
  int32_t n_groups, n_heads, heads_per_group;
  int32_t nqb, nkb, qb_off, variant;
};

struct Range {
  int lo, hi;  // [lo, hi)
};

// Sorted, merged ranges of one BigBird row; returns the number of ranges.
__device__ __forceinline__ int bigbird_row_ranges(const BigBirdParams& P, int h, int qb_local, Range (&out)[4]) {
  const int grp = h / P.heads_per_group;
  const int g = P.g[grp], w = P.w[grp], r = P.r[grp];
  const int qb = P.qb_off + qb_local;
  Range rs[4];
  int n = 0;
  if (P.variant == SA_BIGBIRD2 && qb_local == P.nqb - 1) {
    rs[n++] = {0, P.nkb};
  } else {
    if (g > 0) rs[n++] = {0, g};
    const int ws = max(0, qb - w + 1), we = min(qb + 1, P.nkb);
    if (we > ws) rs[n++] = {ws, we};
    if (r > 0 && qb > 0) {
      const int local_start = max(g, qb - w + 1);
      const int cend = min(qb, local_start);
      const int nc = cend - g;
      if (nc > 0) {
        if (nc <= r) {
          rs[n++] = {g, cend};
        } else {
          const int64_t key = (int64_t)h * 131 + (int64_t)qb * 17 + (int64_t)P.nkb * 7;
          const int off = (int)(key % nc);
          if (off + r <= nc) {
            rs[n++] = {g + off, g + off + r};
          } else {
            rs[n++] = {g + off, g + nc};
            rs[n++] = {g, g + off + r - nc};
          }
        }
      }
    }
  }
  // insertion sort by lo, then merge overlapping/adjacent ranges
  for (int i = 1; i < n; ++i) {
    Range x = rs[i];
    int j = i - 1;
    while (j >= 0 && rs[j].lo > x.lo) {
      rs[j + 1] = rs[j];
      --j;
    }
    rs[j + 1] = x;
  }
  int m = 0;
  for (int i = 0; i < n; ++i) {
    if (m > 0 && rs[i].lo <= out[m - 1].hi) {
      out[m - 1].hi = max(out[m - 1].hi, rs[i].hi);
    } else {
      out[m++] = rs[i];
    }
  }
  return m;
}

// In-place inclusive scan of a[1..n] (a[0] is set to 0) by one thread block.
__device__ void block_scan_counts(int32_t* a, int n) {
  __shared__ int32_t s_warp[32];
  __shared__ int32_t s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = blockDim.x >> 5;
  if (tid == 0) {
    a[0] = 0;
    s_carry = 0;
  }
  __syncthreads();
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + tid;
    int v = i < n ? a[i + 1] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int t = lane < nw ? s_warp[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      if (lane < nw) s_warp[lane] = t;
    }
    __syncthreads();
    const int incl = x + (warp > 0 ? s_warp[warp - 1] : 0) + s_carry;
    if (i < n) a[i + 1] = incl;
    __syncthreads();
    if (tid == blockDim.x - 1) s_carry = incl;
    __syncthreads();
  }
}

__global__ void bigbird_offsets_kernel(const BigBirdParams P, int32_t* offsets) {
  const int h = blockIdx.x;
  int32_t* off = offsets + (int64_t)h * (P.nqb + 1);
  for (int qb = threadIdx.x; qb < P.nqb; qb += blockDim.x) {
    Range rr[4];
    const int m = bigbird_row_ranges(P, h, qb, rr);
    int c = 0;
    for (int i = 0; i < m; ++i) c += rr[i].hi - rr[i].lo;
    off[qb + 1] = c;
  }
  __syncthreads();
  block_scan_counts(off, P.nqb);
}

__global__ void bigbird_pairs_kernel(const BigBirdParams P, const int32_t* offsets, int32_t* pairs,
                                     int max_pairs) {
  const int h = blockIdx.y;
  const int qb = blockIdx.x * blockDim.x + threadIdx.x;
  if (qb >= P.nqb) return;
  const int32_t* off = offsets + (int64_t)h * (P.nqb + 1);
  int pos = off[qb];
  const int lim = min(off[qb + 1], max_pairs);
  int32_t* dst = pairs + (int64_t)h * max_pairs;
  Range rr[4];
  const int m = bigbird_row_ranges(P, h, qb, rr);
  for (int i = 0; i < m; ++i)
    for (int kb = rr[i].lo; kb < rr[i].hi && pos < lim; ++kb) dst[pos++] = kb;
}

// ---- block bitmap [H, NQB, NKB] -> CSR (one warp per row) -------------------
__global__ void bitmap_offsets_kernel(const uint8_t* bitmap, int NQB, int NKB, int32_t* offsets) {
  const int h = blockIdx.x;
  int32_t* off = offsets + (int64_t)h * (NQB + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int qb = warp; qb < NQB; qb += nw) {
    const uint8_t* row = bitmap + ((int64_t)h * NQB + qb) * NKB;
    int c = 0;
    for (int kb = lane; kb < NKB; kb += 32) c += row[kb] != 0;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) off[qb + 1] = c;
  }
  __syncthreads();
  block_scan_counts(off, NQB);
}

__global__ void bitmap_pairs_kernel(const uint8_t* bitmap, int H, int NQB, int NKB, const int32_t* offsets,
                                    int32_t* pairs, int max_pairs) {
  const int warps_per_block = blockDim.x >> 5;
  const int64_t gw = (int64_t)blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)H * NQB) return;
  const int h = (int)(gw / NQB), qb = (int)(gw % NQB);
  const uint8_t* row = bitmap + gw * NKB;
  int pos = offsets[(int64_t)h * (NQB + 1) + qb];
  int32_t* dst = pairs + (int64_t)h * max_pairs;
  for (int base = 0; base < NKB; base += 32) {
    const int kb = base + lane;
    const bool on = kb < NKB && row[kb] != 0;
    const uint32_t bal = __ballot_sync(0xffffffffu, on);
    const int idx = pos + __popc(bal & ((1u << lane) - 1u));
    if (on && idx < max_pairs) dst[idx] = kb;
    pos += __popc(bal);
  }
}

// ---- legacy padded list [H, NQB, MAX_KV] (-1 padding) -> CSR -----------------
__global__ void kvlist_offsets_kernel(const int32_t* lst, int NQB, int max_kv, int32_t* offsets) {
  const int h = blockIdx.x;
  int32_t* off = offsets + (int64_t)h * (NQB + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int qb = warp; qb < NQB; qb += nw) {
    const int32_t* row = lst + ((int64_t)h * NQB + qb) * max_kv;
    int c = 0;
    for (int i = lane; i < max_kv; i += 32) c += row[i] >= 0;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) off[qb + 1] = c;
  }
  __syncthreads();
  block_scan_counts(off, NQB);
}

__global__ void kvlist_pairs_kernel(const int32_t* lst, int H, int NQB, int max_kv, const int32_t* offsets,
                                    int32_t* pairs, int max_pairs) {
  const int warps_per_block = blockDim.x >> 5;
  const int64_t gw = (int64_t)blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)H * NQB) return;
  const int h = (int)(gw / NQB), qb = (int)(gw % NQB);
  const int32_t* row = lst + gw * max_kv;
  int pos = offsets[(int64_t)h * (NQB + 1) + qb];
  int32_t* dst = pairs + (int64_t)h * max_pairs;
  for (int base = 0; base < max_kv; base += 32) {
    const int i = base + lane;
    const int val = i < max_kv ? row[i] : -1;
    const bool on = val >= 0;
    const uint32_t bal = __ballot_sync(0xffffffffu, on);
    const int idx = pos + __popc(bal & ((1u << lane) - 1u));
    if (on && idx < max_pairs) dst[idx] = val;
    pos += __popc(bal);
  }
}

// ---- token mask [H, T_q, T_k] -> block bitmap [H, NQB, NKB] -----------------
// One CTA per (query block, head); a kept token marks its block (bitmap must be
// zeroed first). 16-byte vector path when rows are 16-byte aligned: with a block
// size >= 16, one aligned 16-byte vector never straddles two key blocks.
__global__ void token_mask_to_bitmap_kernel(const uint8_t* mask, int T_q, int T_k, int bs, int NQB, int NKB,
                                            uint8_t* bitmap) {
  const int qb = blockIdx.x, h = blockIdx.y;
  uint8_t* brow = bitmap + ((int64_t)h * NQB + qb) * NKB;
  const int r0 = qb * bs, r1 = min(T_q, r0 + bs);
  const bool vec = (T_k % 16) == 0 && ((reinterpret_cast<uintptr_t>(mask) & 15u) == 0);
  for (int r = r0; r < r1; ++r) {
    const uint8_t* row = mask + ((int64_t)h * T_q + r) * T_k;
    if (vec) {
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int i = threadIdx.x; i < T_k / 16; i += blockDim.x) {
        const uint4 x = __ldg(rv + i);
        if ((x.x | x.y | x.z | x.w) != 0u) {
          const int kb = (i * 16) / bs;
          if (!brow[kb]) brow[kb] = 1;
        }
      }
    } else {
      for (int c = threadIdx.x; c < T_k; c += blockDim.x)
        if (row[c]) {
          const int kb = c / bs;
          if (!brow[kb]) brow[kb] = 1;
        }
    }
  }
}

// Decode rows (T_q = 1) of heads [head_lo, head_lo + n_rows) for the key count
// in device memory: block rows depend on T_k only through nkb and the query
// block (T_k - 1) / bs, so a CUDA graph replaying a growing cache can recompute
// them on the device every step. offsets [n_rows, 2], pairs [n_rows, max_pairs].
__global__ void bigbird_decode_row_kernel(BigBirdParams P, const int32_t* seq_len, int bs, int head_lo, int n_rows,
                                          int32_t* offsets, int32_t* pairs, int max_pairs, int32_t* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_rows) return;
  const int T_k = max(1, __ldg(seq_len));
  P.nqb = 1;
  P.nkb = (T_k + bs - 1) / bs;
  P.qb_off = (T_k - 1) / bs;
  Range rr[4];
  const int m = bigbird_row_ranges(P, head_lo + i, 0, rr);
  int32_t* dst = pairs + (int64_t)i * max_pairs;
  int pos = 0;
  for (int k = 0; k < m; ++k)
    for (int kb = rr[k].lo; kb < rr[k].hi; ++kb) {
      if (pos < max_pairs) dst[pos] = kb;
      ++pos;
    }
  if (pos > max_pairs) {
    record_error(err, SA_DEV_ERR_INDEX);
    pos = max_pairs;
  }
  offsets[2 * i] = 0;
  offsets[2 * i + 1] = pos;
}

static int fill_bigbird(BigBirdParams* P, const sa_bigbird_layout* layouts, int n_groups, int n_heads, int T_q,
                        int T_k, int bs, int variant) {
  if (!layouts) return sa_fail(SA_ERR_INVALID, "layouts is NULL");
  if (n_groups <= 0 || n_groups > kMaxGroups)
    return sa_fail(SA_ERR_INVALID, "n_groups %d not in [1, %d]", n_groups, kMaxGroups);
  if (n_heads <= 0 || n_heads % n_groups)
    return sa_fail(SA_ERR_INVALID, "n_heads=%d must be a positive multiple of n_groups=%d", n_heads, n_groups);
  if (T_q <= 0 || T_k <= 0 || T_q > T_k) return sa_fail(SA_ERR_INVALID, "bad T_q=%d T_k=%d", T_q, T_k);
  if (bs <= 0) return sa_fail(SA_ERR_INVALID, "block_size %d must be positive", bs);
  if (variant != SA_BIGBIRD && variant != SA_BIGBIRD2) return sa_fail(SA_ERR_INVALID, "unknown variant %d", variant);
  memset(P, 0, sizeof(*P));
  for (int i = 0; i < n_groups; ++i) {
    if (layouts[i].global_blocks < 0 || layouts[i].sliding_blocks < 0 || layouts[i].random_blocks < 0)
      return sa_fail(SA_ERR_INVALID, "negative layout field in group %d", i);
    P->g[i] = layouts[i].global_blocks;
    P->w[i] = layouts[i].sliding_blocks;
    P->r[i] = layouts[i].random_blocks;
  }
  P->n_groups = n_groups;
  P->n_heads = n_heads;
  P->heads_per_group = n_heads / n_groups;
  P->nqb = (T_q + bs - 1) / bs;
  P->nkb = (T_k + bs - 1) / bs;
  P->qb_off = (T_k - T_q) / bs;
  P->variant = variant;
  return SA_OK;
}

}  // namespace sa

using namespace sa;

// ---------------------------------------------------------------------------
// CSR validation (the checks the attention kernels rely on)
// ---------------------------------------------------------------------------
// One CTA per head, one thread per row: offsets[h, 0] == 0, non-decreasing,
// offsets[h, NQB] <= pairs_stride; every index of a row in [0, NKB) and strictly
// increasing. The first violation found (by any thread) is recorded in
// result[0..3] = (kind, head, row, position); kind 0 = valid.
__global__ void validate_csr_kernel(const int32_t* __restrict__ pairs, const int32_t* __restrict__ offsets,
                                    int NQB, int NKB, int stride, int32_t* result) {
  const int h = blockIdx.x;
  const int32_t* off = offsets + (int64_t)h * (NQB + 1);
  const int32_t* row = pairs + (int64_t)h * stride;
  auto fail = [&](int kind, int r, int pos) {
    if (atomicCAS(result, 0, kind) == 0) {
      result[1] = h;
      result[2] = r;
      result[3] = pos;
    }
  };
  if (threadIdx.x == 0 && __ldg(off) != 0) fail(1, 0, 0);
  for (int r = threadIdx.x; r < NQB; r += blockDim.x) {
    const int o0 = __ldg(off + r), o1 = __ldg(off + r + 1);
    if (o1 < o0) {
      fail(2, r, o0);
      continue;
    }
    if (o1 > stride || o0 < 0) {
      fail(3, r, o1);
      continue;
    }
    int prev = -1;
    for (int i = o0; i < o1; ++i) {
      const int kb = __ldg(row + i);
      if (kb < 0 || kb >= NKB) {
        fail(4, r, i);
        break;
      }
      if (kb <= prev) {
        fail(5, r, i);
        break;
      }
      prev = kb;
    }
  }
}

extern "C" int sa_validate_csr(const int32_t* pairs, const int32_t* offsets, int32_t H, int32_t NQB, int32_t NKB,
                               int32_t pairs_stride, int32_t* result, sa_stream_t stream) {
  if (!pairs || !offsets || !result || H <= 0 || NQB <= 0 || NKB <= 0 || pairs_stride <= 0)
    return sa_fail(SA_ERR_INVALID, "bad arguments");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SA_CHECK_CUDA(cudaMemsetAsync(result, 0, 4 * sizeof(int32_t), s));
  validate_csr_kernel<<<H, 128, 0, s>>>(pairs, offsets, NQB, NKB, pairs_stride, result);
  SA_CHECK_CUDA(cudaGetLastError());
  int32_t host[4] = {0, 0, 0, 0};
  SA_CHECK_CUDA(cudaMemcpyAsync(host, result, sizeof(host), cudaMemcpyDeviceToHost, s));
  SA_CHECK_CUDA(cudaStreamSynchronize(s));
  static const char* what[] = {"", "offsets[h, 0] != 0", "offsets decrease", "offset outside [0, pairs_stride]",
                               "block index outside [0, NKB)", "row not strictly increasing"};
  if (host[0] != 0)
    return sa_fail(SA_ERR_CSR, "invalid CSR: %s (head %d, row %d, position %d)",
                   what[host[0] >= 1 && host[0] <= 5 ? host[0] : 0], host[1], host[2], host[3]);
  return SA_OK;
}

extern "C" int sa_bigbird_offsets(const sa_bigbird_layout* layouts, int32_t n_groups, int32_t n_heads,
                                  int32_t T_q, int32_t T_k, int32_t block_size, int32_t variant,
                                  int32_t* offsets, sa_stream_t stream) {
  BigBirdParams P;
  int rc = fill_bigbird(&P, layouts, n_groups, n_heads, T_q, T_k, block_size, variant);
  if (rc) return rc;
  if (!offsets) return sa_fail(SA_ERR_INVALID, "offsets is NULL");
  bigbird_offsets_kernel<<<n_heads, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(P, offsets);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_bigbird_pairs(const sa_bigbird_layout* layouts, int32_t n_groups, int32_t n_heads,
                                int32_t T_q, int32_t T_k, int32_t block_size, int32_t variant,
                                const int32_t* offsets, int32_t* pairs, int32_t max_pairs, sa_stream_t stream) {
  BigBirdParams P;
  int rc = fill_bigbird(&P, layouts, n_groups, n_heads, T_q, T_k, block_size, variant);
  if (rc) return rc;
  if (!offsets || !pairs || max_pairs <= 0) return sa_fail(SA_ERR_INVALID, "bad pairs/offsets/max_pairs");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SA_CHECK_CUDA(cudaMemsetAsync(pairs, 0, (size_t)n_heads * max_pairs * sizeof(int32_t), s));
  dim3 grid((P.nqb + 127) / 128, n_heads);
  bigbird_pairs_kernel<<<grid, 128, 0, s>>>(P, offsets, pairs, max_pairs);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_block_bitmap_from_token_mask(const uint8_t* token_mask, int32_t H, int32_t T_q, int32_t T_k,
                                               int32_t block_size, uint8_t* bitmap, sa_stream_t stream) {
  if (!token_mask || !bitmap) return sa_fail(SA_ERR_INVALID, "NULL pointer");
  if (H <= 0 || T_q <= 0 || T_k <= 0 || block_size < 16 || (block_size & (block_size - 1)))
    return sa_fail(SA_ERR_INVALID, "bad sizes (H=%d T_q=%d T_k=%d bs=%d; bs power of 2 >= 16)", H, T_q, T_k,
                   block_size);
  const int NQB = (T_q + block_size - 1) / block_size, NKB = (T_k + block_size - 1) / block_size;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SA_CHECK_CUDA(cudaMemsetAsync(bitmap, 0, (size_t)H * NQB * NKB, s));
  token_mask_to_bitmap_kernel<<<dim3(NQB, H), 256, 0, s>>>(token_mask, T_q, T_k, block_size, NQB, NKB, bitmap);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_bitmap_offsets(const uint8_t* bitmap, int32_t H, int32_t NQB, int32_t NKB, int32_t* offsets,
                                 sa_stream_t stream) {
  if (!bitmap || !offsets || H <= 0 || NQB <= 0 || NKB <= 0) return sa_fail(SA_ERR_INVALID, "bad arguments");
  bitmap_offsets_kernel<<<H, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(bitmap, NQB, NKB, offsets);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_bitmap_pairs(const uint8_t* bitmap, int32_t H, int32_t NQB, int32_t NKB, const int32_t* offsets,
                               int32_t* pairs, int32_t max_pairs, sa_stream_t stream) {
  if (!bitmap || !offsets || !pairs || H <= 0 || NQB <= 0 || NKB <= 0 || max_pairs <= 0)
    return sa_fail(SA_ERR_INVALID, "bad arguments");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SA_CHECK_CUDA(cudaMemsetAsync(pairs, 0, (size_t)H * max_pairs * sizeof(int32_t), s));
  const int64_t rows = (int64_t)H * NQB;
  bitmap_pairs_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(bitmap, H, NQB, NKB, offsets, pairs, max_pairs);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_kvlist_offsets(const int32_t* kv_block_list, int32_t H, int32_t NQB, int32_t max_kv,
                                 int32_t* offsets, sa_stream_t stream) {
  if (!kv_block_list || !offsets || H <= 0 || NQB <= 0 || max_kv <= 0) return sa_fail(SA_ERR_INVALID, "bad arguments");
  kvlist_offsets_kernel<<<H, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(kv_block_list, NQB, max_kv, offsets);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_kvlist_pairs(const int32_t* kv_block_list, int32_t H, int32_t NQB, int32_t max_kv,
                               const int32_t* offsets, int32_t* pairs, int32_t max_pairs, sa_stream_t stream) {
  if (!kv_block_list || !offsets || !pairs || H <= 0 || NQB <= 0 || max_kv <= 0 || max_pairs <= 0)
    return sa_fail(SA_ERR_INVALID, "bad arguments");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SA_CHECK_CUDA(cudaMemsetAsync(pairs, 0, (size_t)H * max_pairs * sizeof(int32_t), s));
  const int64_t rows = (int64_t)H * NQB;
  kvlist_pairs_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(kv_block_list, H, NQB, max_kv, offsets, pairs,
                                                                 max_pairs);
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_bigbird_decode_row(const sa_bigbird_layout* layouts, int32_t n_groups, int32_t n_heads,
                                     int32_t head_lo, int32_t n_rows, const int32_t* seq_len, int32_t block_size,
                                     int32_t variant, int32_t* offsets, int32_t* pairs, int32_t max_pairs,
                                     sa_stream_t stream) {
  BigBirdParams P;
  int rc = fill_bigbird(&P, layouts, n_groups, n_heads, 1, 1, block_size, variant);
  if (rc) return rc;
  if (variant == SA_BIGBIRD2) return sa_fail(SA_ERR_UNSUPPORTED, "decode rows: BigBird2 has no decode variant");
  if (!seq_len || !offsets || !pairs || max_pairs <= 0) return sa_fail(SA_ERR_INVALID, "bad pointers / max_pairs");
  if (head_lo < 0 || n_rows <= 0 || head_lo + n_rows > n_heads)
    return sa_fail(SA_ERR_INVALID, "heads [%d, %d) outside [0, %d)", head_lo, head_lo + n_rows, n_heads);
  bigbird_decode_row_kernel<<<(n_rows + 127) / 128, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      P, seq_len, block_size, head_lo, n_rows, offsets, pairs, max_pairs, sa_device_error_ptr());
  SA_CHECK_CUDA(cudaGetLastError());
  return SA_OK;
}
