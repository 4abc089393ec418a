/*
 * sparse_attn_b200.h — C ABI of the B200 (sm_100a) block-sparse attention backend.
 *
 * Every entry point takes plain device pointers, sizes and strides (in elements),
 * launches on the given CUDA stream, allocates nothing and never synchronises.
 * Each returns 0 on success or a negative SA_ERR_* code; sa_last_error() then
 * holds a one-line message for the calling host thread.
 *
 * The reference (rrroooyyywang/SparseAttentionInfer) has no native attention
 * code; each entry point names the Python/Triton interface it replaces.
 */
#ifndef SPARSE_ATTN_B200_H
#define SPARSE_ATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SA_API __attribute__((visibility("default")))
#else
#define SA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* sa_stream_t; /* a cudaStream_t (CUstream); NULL = legacy default stream */

enum {
  SA_OK = 0,
  SA_ERR_INVALID = -1,     /* bad shape, stride, alignment or parameter          */
  SA_ERR_UNSUPPORTED = -2, /* valid but unsupported (dtype, head_dim, device)    */
  SA_ERR_CUDA = -3,        /* a CUDA runtime/driver call failed                   */
  SA_ERR_TIMEOUT = -4,     /* a device-side bounded wait expired (see below)      */
  SA_ERR_CSR = -5          /* CSR schedule failed host-side validation           */
};

/* BigBird layout of one KV group: (block_size, global, sliding, random), the
 * tuple returned by bigbird_layout_from_topk / bigbird_layout_from_keep_ratio
 * (sparse_attentions/patterns/bigbird_pattern.py:12-20, 338-363). */
typedef struct {
  int32_t block_size;
  int32_t global_blocks;
  int32_t sliding_blocks;
  int32_t random_blocks;
} sa_bigbird_layout;

/* Pattern variants of sa_bigbird_offsets / sa_bigbird_pairs. */
enum {
  SA_BIGBIRD = 0,  /* BigBirdPattern / BigBirdKeepRatioPattern _get_block_pairs
                      (bigbird_pattern.py:212-271, 533-583)                    */
  SA_BIGBIRD2 = 1  /* BigBird2Pattern._get_block_pairs: last query-block row is
                      every key block (bigbird_pattern.py:697-753)              */
};

/* Version string of the library build. */
SA_API const char* sa_version(void);

/* Message of the last failing call on this host thread ("" if none). */
SA_API const char* sa_last_error(void);

/* Read and clear the device-side error word that bounded waits set when they
 * expire (SA_ERR_TIMEOUT) or that index checks set. Synchronises the device.
 * *code receives 0 when no kernel reported an error. */
SA_API int sa_device_error(int32_t* code);

/* ---------------------------------------------------------------------------
 * Pattern compiler (device side). Replaces the Python H x NQB loops of
 * BigBirdPattern._get_block_pairs (bigbird_pattern.py:212-271),
 * BigBirdKeepRatioPattern._get_block_pairs (:533-583) and
 * BigBird2Pattern._get_block_pairs (:697-753), bit-exact with them:
 * per head h and local query block qb the sorted union of global blocks
 * [0,g), the window [max(0,qba-w+1), min(qba+1,NKB)) and the rotated random
 * blocks of select_bigbird_random_block_ids (:23-41), qba = (T_k-T_q)/bs + qb.
 *
 * Two phases, because the reference's block_pairs width (max nnz over heads)
 * is data dependent:
 *   1. sa_bigbird_offsets writes offsets [H, NQB+1] (int32, per-head CSR
 *      starting at 0), NQB = ceil(T_q/bs);
 *   2. the caller reads max_h offsets[h, NQB], allocates pairs [H, max(1,that)]
 *      and sa_bigbird_pairs fills it, zero padded like the reference.
 * layouts is a HOST array of n_groups entries (n_groups divides n_heads; head h
 * uses group h / (n_heads/n_groups)); only their g/w/r fields are used, the
 * block size is `block_size` for every group (the reference uses
 * _next_pow2_min16(layouts[0][0]) for all groups, bigbird_pattern.py:545).
 * ------------------------------------------------------------------------- */
SA_API int sa_bigbird_offsets(const sa_bigbird_layout* layouts, int32_t n_groups, int32_t n_heads,
                       int32_t T_q, int32_t T_k, int32_t block_size, int32_t variant,
                       int32_t* offsets, sa_stream_t stream);
SA_API int sa_bigbird_pairs(const sa_bigbird_layout* layouts, int32_t n_groups, int32_t n_heads,
                     int32_t T_q, int32_t T_k, int32_t block_size, int32_t variant,
                     const int32_t* offsets, int32_t* pairs, int32_t max_pairs,
                     sa_stream_t stream);

/* Decode rows (T_q = 1) of query heads [head_lo, head_lo + n_rows) for the key
 * count *seq_len read on the device (the rows of sa_bigbird_offsets/_pairs with
 * T_q = 1, T_k = *seq_len; BigBirdKeepRatioPattern's decode build,
 * bigbird_pattern.py:533-583 with T_q = 1): offsets [n_rows, 2] = {0, nnz},
 * pairs [n_rows, max_pairs] (row h holds its blocks, rest untouched). A row
 * longer than max_pairs is cut and sets SA_DEV_ERR_INDEX in the device error
 * word. A dense causal row is the layout (block_size, 0, window >= rows, 0).
 * For graph-replayed decode, where the host does not see the growing length. */
SA_API int sa_bigbird_decode_row(const sa_bigbird_layout* layouts, int32_t n_groups, int32_t n_heads,
                                 int32_t head_lo, int32_t n_rows, const int32_t* seq_len, int32_t block_size,
                                 int32_t variant, int32_t* offsets, int32_t* pairs, int32_t max_pairs,
                                 sa_stream_t stream);

/* Arbitrary retained-block masks. Replaces build_block_pairs_from_mask
 * (sparse_attentions/patterns/base.py:36-89).
 * sa_block_bitmap_from_token_mask: token mask [H, T_q, T_k] (bool/uint8,
 * contiguous) -> block bitmap [H, NQB, NKB] (uint8 0/1): a block is kept when
 * any token of it is kept (base.py:67-73).
 * sa_bitmap_offsets / sa_bitmap_pairs: block bitmap -> CSR, same two-phase
 * protocol as the BigBird compiler (base.py:75-89). */
SA_API int sa_block_bitmap_from_token_mask(const uint8_t* token_mask, int32_t H, int32_t T_q,
                                   int32_t T_k, int32_t block_size, uint8_t* bitmap,
                                   sa_stream_t stream);
SA_API int sa_bitmap_offsets(const uint8_t* bitmap, int32_t H, int32_t NQB, int32_t NKB,
                      int32_t* offsets, sa_stream_t stream);
SA_API int sa_bitmap_pairs(const uint8_t* bitmap, int32_t H, int32_t NQB, int32_t NKB,
                    const int32_t* offsets, int32_t* pairs, int32_t max_pairs,
                    sa_stream_t stream);

/* CSR validation: the properties the attention kernels rely on. Per head h of
 * pairs [H, pairs_stride] / offsets [H, NQB+1]: offsets[h, 0] == 0, offsets
 * non-decreasing and <= pairs_stride, every block index of row q in [0, NKB)
 * and strictly increasing along the row (the reference's builders emit sorted
 * rows: build_block_pairs_from_mask takes nonzero() of each row,
 * sparse_attentions/patterns/base.py:75-89; _get_block_pairs sorts each row,
 * bigbird_pattern.py:533-583). `result` is 4 int32 of device scratch. Blocks
 * until done (one device->host read). Returns SA_ERR_CSR and names the first
 * violation in sa_last_error() when invalid. Replaces the reference wrapper's
 * host-side input checks (kernels/triton/universal_sparse_attn.py:187-199). */
SA_API int sa_validate_csr(const int32_t* pairs, const int32_t* offsets, int32_t H, int32_t NQB, int32_t NKB,
                           int32_t pairs_stride, int32_t* result, sa_stream_t stream);

/* Legacy padded schedule -> CSR. Replaces kv_block_list_to_pairs
 * (sparse_attentions/patterns/base.py:92-133): kv_block_list [H, NQB, MAX_KV]
 * int32 with -1 padding. Same two-phase protocol. */
SA_API int sa_kvlist_offsets(const int32_t* kv_block_list, int32_t H, int32_t NQB, int32_t max_kv,
                      int32_t* offsets, sa_stream_t stream);
SA_API int sa_kvlist_pairs(const int32_t* kv_block_list, int32_t H, int32_t NQB, int32_t max_kv,
                    const int32_t* offsets, int32_t* pairs, int32_t max_pairs,
                    sa_stream_t stream);

/* ---------------------------------------------------------------------------
 * Block-sparse attention forward (prefill / any T_q). Replaces
 * universal_sparse_attn + _universal_sparse_attn_kernel
 * (kernels/triton/universal_sparse_attn.py:45-238) behind
 * TritonUniversalBackend.forward (sparse_attentions/attention/triton_universal_backend.py:47-66).
 *
 *   out[b,h,i,:] = sum_j softmax_j(scale * q[b,h,i]·k[b,kvh,j]) v[b,kvh,j]
 * over keys j whose block j/bs is listed in CSR row (h, i/bs), with j <= i +
 * (T_k - T_q) (causal, bottom-right aligned) and j < T_k. Rows with no valid
 * key are written as 0 (universal_sparse_attn.py:150-153). kvh = h / (Hq/Hkv)
 * (GQA without repeat_kv).
 *
 * q/out: [B, Hq, T_q, D] bf16, k/v: [B, Hkv, T_k, D] bf16, each with the given
 * element strides for b, h and t (stride of d must be 1); strides and base
 * addresses must be 16-byte aligned. D in {64, 128}. block_size a power of two
 * in [16, 512]. pairs [Hq, pairs_stride] / offsets [Hq, NQB+1] int32 device
 * arrays, NQB = ceil(T_q / block_size).
 * Uses tcgen05 MMAs with TMEM accumulators and TMA tile loads; persistent grid.
 * Tiles are handed out by a counter in one of 64 library-owned scheduler slots;
 * each call takes the next slot (round robin per device) and its last CTA
 * re-arms it. So at most 64 prefill launches may be in flight at once on a
 * device, and a launch recorded in a CUDA graph keeps its slot: replays of it
 * must not overlap each other, nor run while 64 or more other prefill launches
 * are issued and still in flight.
 * ------------------------------------------------------------------------- */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  const int32_t* pairs;
  const int32_t* offsets;
  int64_t q_strides[3];   /* b, h, t (elements) */
  int64_t k_strides[3];
  int64_t v_strides[3];
  int64_t o_strides[3];
  int32_t B, Hq, Hkv, T_q, T_k, D;
  int32_t block_size;
  int32_t pairs_stride;   /* row stride of pairs (elements) */
  float scale;            /* softmax scale, usually 1/sqrt(D) */
  int32_t num_sms;        /* persistent grid size; 0 = all SMs */
} sa_attn_args;

SA_API int sa_prefill_fwd(const sa_attn_args* args, sa_stream_t stream);

/* ---------------------------------------------------------------------------
 * Split-KV sparse decode (T_q == 1). Replaces the decode use of
 * universal_sparse_attn (Q_OFFSET = T_k, universal_sparse_attn.py:84-89),
 * where the Triton kernel runs one 1-row query block per (b, h).
 * One CTA per (b, kv head, split) serves the Hq/Hkv query heads of the group
 * and reads the union of their CSR rows' key blocks once (the reference's
 * random blocks differ per query head, bigbird_pattern.py:23-41).
 * Scratch (caller-allocated, float32): partial_o [B, Hq, n_split, D] and
 * partial_ml [B, Hq, n_split, 2]; a second kernel merges the splits into out.
 * n_split in [1, 64]; Hq/Hkv in {1, 2, 4, 8}; D in {64, 128};
 * ceil(T_k / block_size) <= 8192 and min(ceil(T_k / block_size),
 * (Hq/Hkv) * pairs_stride) <= 2048 (the union of a KV group's rows is built in
 * shared memory), SA_ERR_UNSUPPORTED otherwise.
 * ------------------------------------------------------------------------- */
SA_API int sa_decode_fwd(const sa_attn_args* args, int32_t n_split, float* partial_o,
                  float* partial_ml, sa_stream_t stream);

/* ---------------------------------------------------------------------------
 * sa_decode_fwd without caller scratch. No counterpart in the reference: it is
 * for callers that cannot allocate device memory at call time (code that owns
 * no allocator, such as a plugin running inside another framework's memory
 * pool, or a serving loop that must not allocate while it runs). The split
 * partials live in a fixed array compiled into this library, SA_DECODE_SCRATCH_FLOATS
 * floats (16 MiB) that every GPU which loads the library keeps until exit;
 * calls needing B*Hq*n_split*(D+2) floats beyond that fail with SA_ERR_INVALID.
 * Nothing here calls cudaMalloc/cudaFree. The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture. All calls share the one array: calls that overlap
 * on the GPU (other streams, other threads) race and must be serialised by the
 * caller. Every split result is fully rewritten by each call, so nothing has to
 * start at zero. With n_split == 1 the kernel writes the output directly and
 * the array is not used (no size limit). Same arguments, output, limits and
 * error codes as sa_decode_fwd otherwise.
 * ------------------------------------------------------------------------- */
#define SA_DECODE_SCRATCH_FLOATS (4 * 1024 * 1024)
SA_API int sa_decode_fwd_noalloc(const sa_attn_args* args, int32_t n_split, sa_stream_t stream);

/* ---------------------------------------------------------------------------
 * sa_decode_fwd with the key count read from device memory: args->k / args->v
 * span args->T_k rows (the cache capacity) and the kernel attends to keys
 * [0, *seq_len) (clamped to [0, args->T_k]), so one launch recorded into a CUDA
 * graph serves every step of a growing cache. The caller keeps the CSR rows
 * valid for the live length (the decode row of block (*seq_len - 1) / bs).
 * Rows past *seq_len are read in whole 64-key stages and masked; they must hold
 * finite values (a zero-initialised cache does). Replaces the same decode call
 * as sa_decode_fwd; the reference passes the length on the host.
 * ------------------------------------------------------------------------- */
SA_API int sa_decode_fwd_seqlen(const sa_attn_args* args, const int32_t* seq_len, int32_t n_split,
                                float* partial_o, float* partial_ml, sa_stream_t stream);

/* ---------------------------------------------------------------------------
 * Decoder-layer steps around attention (Qwen3 layer arithmetic; bf16 tensors,
 * fp32 arithmetic, one rounding per stored value).
 *
 * sa_qk_norm_rope_append: from the fused projection output qkv [B, T, Hq+2*Hkv, D]
 * (element strides qkv_sb, qkv_st; heads contiguous), writes
 *   q_out[b, h, t]            = RoPE(RMSNorm(q) * q_weight) at position pos + t,
 *   k_cache[b, h, pos + t]    = RoPE(RMSNorm(k) * k_weight),
 *   v_cache[b, h, pos + t]    = v,
 * with rotate-half RoPE from the cos/sin tables [capacity, D]. pos is *pos_dev
 * when pos_dev is non-NULL (graph replays), else the host value. Replaces the
 * hook's q_norm / k_norm / apply_rotary_pos_emb / cache update
 * (modeling_sparse_qwen3.py:211-231). D in {64, 128}.
 * ------------------------------------------------------------------------- */
typedef struct sa_qkv_prologue_args {
  const void* qkv;
  int64_t qkv_sb, qkv_st;
  const void* q_weight;   /* [D] */
  const void* k_weight;   /* [D] */
  const void* cos;        /* [capacity, D] */
  const void* sin;        /* [capacity, D] */
  void* q_out;            /* [B, Hq, T, D] */
  int64_t q_strides[3];   /* b, h, t */
  void* k_cache;          /* [B, Hkv, capacity, D] */
  int64_t k_strides[3];
  void* v_cache;
  int64_t v_strides[3];
  int32_t B, T, Hq, Hkv, D, capacity;
  int32_t pos;
  const int32_t* pos_dev;
  float eps;
} sa_qkv_prologue_args;

SA_API int sa_qk_norm_rope_append(const sa_qkv_prologue_args* args, sa_stream_t stream);

/* Residual add + RMSNorm over rows of n elements (n % 8 == 0, 16-byte aligned rows):
 *   x = x + y (stored, bf16; y may be NULL), out = x * rsqrt(mean(x^2) + eps) * weight.
 * Qwen3RMSNorm after each decoder sub-block. */
SA_API int sa_add_rms_norm(void* x, const void* y, const void* weight, void* out, int64_t rows, int32_t n,
                           int64_t x_stride, int64_t y_stride, int64_t out_stride, float eps,
                           sa_stream_t stream);

/* SwiGLU activation: out[r, i] = silu(gu[r, i]) * gu[r, inter + i] (Qwen3MLP act_fn(gate) * up). */
SA_API int sa_silu_mul(const void* gate_up, void* out, int64_t rows, int32_t inter, int64_t gu_stride,
                       int64_t out_stride, sa_stream_t stream);

/* Projection of M <= 8 tokens (decode), bf16 in and out, fp32 accumulation:
 *   glu == 0: out[m, n] = sum_k x[m, k] * w[n, k],  n < N   (nn.Linear, no bias)
 *   glu != 0: g, u = bf16 of the same sums over w rows n and N + n (the fused
 *             [gate; up] weight), out[m, n] = bf16(silu(g) * u)  (Qwen3MLP
 *             act_fn(gate_proj(x)) * up_proj(x) in one launch).
 * K a multiple of 256, N a multiple of 16, x and w rows 16-byte aligned
 * (element strides multiples of 8). Replaces the GEMM launches of the decoder
 * layer at decode batch sizes, where the weight stream is the whole cost. */
SA_API int sa_linear_m8(const void* x, int32_t M, int32_t K, int64_t x_stride, const void* w, int32_t N,
                        int64_t w_stride, void* out, int64_t out_stride, int32_t glu, sa_stream_t stream);

/* ---------------------------------------------------------------------------
 * Data-dependent top-k attention (TopKPattern; MaskedSdpaBackend's "topk" kind,
 * masked_sdpa.py:51-63), second half: given fp32 scores q.k^T.scale of a block
 * of query rows (a [B, Hkv, G * rows_per_head, T_k] GEMM output, row stride
 * s_row, for query positions [t0, t0 + rows_per_head)), masks each row causally
 * (bottom-right aligned) in place, keeps its top_k scores, and writes
 * out[b, h, t] = softmax(kept) . V with h = kv_head * G + g. v is bf16
 * [B, Hkv, T_k, D] (element strides); out is bf16, or fp32 with out_f32.
 * Scores tied exactly at the k-th value are all kept. D in {64, 128}.
 * ------------------------------------------------------------------------- */
typedef struct sa_topk_args {
  void* scores;
  int64_t s_row;
  const void* v;
  int64_t v_strides[3];
  void* out;
  int64_t o_strides[3];
  int32_t out_f32;
  int32_t B, Hkv, G, rows_per_head, t0, T_q, T_k, D, top_k;
} sa_topk_args;

SA_API int sa_topk_softmax_pv(const sa_topk_args* args, sa_stream_t stream);

/* ---------------------------------------------------------------------------
 * Tensor-parallel all-reduce over NVLink peer memory, fused with the residual
 * add and the next RMSNorm (no counterpart in the reference, which runs on one
 * device; it replaces the NCCL all-reduce after o_proj / down_proj for small,
 * latency-bound decode messages).
 *
 * Buffers: each rank allocates with sa_ar_alloc a data region (two slots of
 * rows*n bf16 each) and a flag region (max_ctas * SA_AR_MAX_WORLD uint32), shares
 * them with sa_ar_ipc_handle / sa_ar_ipc_open, and keeps max_ctas uint32 epoch
 * counters in its own memory (zeroed). Every rank writes its partial sum
 * y_rank [rows, n] (contiguous) at data[rank] + data_offset, then calls
 * sa_allreduce_add_rms_norm with the same arguments on every rank:
 *   x += y_0 + ... + y_{world-1}   (fp32 sum in rank order, stored bf16),
 *   out = x * rsqrt(mean(x^2) + eps) * weight.
 * Consecutive calls must alternate between the two slots. Waits for peers are
 * bounded (2 s); on expiry the device error word reads SA_DEV_ERR_TIMEOUT and x
 * is left unchanged. A timed-out call has already advanced this rank's epochs
 * and published its flags while the missing peer has not, so before the next
 * call every rank must zero its epoch counters and its flag region (all ranks
 * together, between barriers: NvlinkAllReduce.reset() in Python). Plain
 * loads/stores to peer memory only (no multicast).
 * ------------------------------------------------------------------------- */
#define SA_AR_MAX_WORLD 8
typedef struct sa_ar_peers {
  int32_t rank, world;
  void* data[SA_AR_MAX_WORLD];       /* each rank's data region (own and peers' mappings) */
  uint32_t* flags[SA_AR_MAX_WORLD];  /* each rank's flag region */
  uint32_t* epoch;                   /* this rank's counters [max_ctas] */
  int32_t max_ctas;
} sa_ar_peers;

SA_API int sa_ar_alloc(size_t bytes, void** ptr);
SA_API int sa_ar_free(void* ptr);
SA_API int sa_ar_ipc_handle(void* ptr, void* handle /* 64 bytes */);
SA_API int sa_ar_ipc_open(const void* handle /* 64 bytes */, void** ptr);
SA_API int sa_ar_ipc_close(void* ptr);
SA_API int sa_allreduce_add_rms_norm(const sa_ar_peers* peers, int64_t data_offset, void* x, const void* weight,
                                     void* out, int64_t rows, int32_t n, int64_t x_stride, int64_t out_stride,
                                     float eps, sa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSE_ATTN_B200_H */
