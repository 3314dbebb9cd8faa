/*
 * hga_b200.h — C ABI of the B200 (sm_100a) kernels for HGA's routed-attention hot path.
 *
 * Plain pointers and sizes only: every tensor is device memory owned by the caller (in the
 * Python host layer: the PyTorch caching allocator), every call is asynchronous on the given
 * CUDA stream, and nothing here allocates device memory.  Every entry point returns 0 on
 * success or a negative HGA_E* code; hga_last_error() then holds a message for the calling
 * host thread.
 *
 * Layout conventions (row-major, innermost last):
 *   q                 [B, H,   S,   Dh]   (q_layout 0)  or [B, S, H, Dh] (q_layout 1)
 *   k_raw, k_rope, v  [B, KVH, cap, Dh]   token rows of one (batch, kv-head) are contiguous;
 *                                          `kv_cap` = rows allocated per (batch, kv-head)
 *   chunk_k           [B, KVH, ccap, Dh]
 *   group_k, group_v  [B, KVH, ccap, M, Dh] `sum_cap` = chunks allocated per (batch, kv-head)
 *   rotary cos / sin  [R, Dh]             row r = absolute position rot_row0 + r
 * N = ceil(S / chunk_size) query chunks; M = chunk_size / group_size groups per chunk.
 */
#ifndef HGA_B200_H_
#define HGA_B200_H_

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { HGA_DTYPE_F32 = 0, HGA_DTYPE_BF16 = 1, HGA_DTYPE_F16 = 2 };
/* How hga_summaries reads its rotary table. */
enum { HGA_ROT_F32 = 0,         /* fp32 table, used as fp32 (ChunkRouter._rotary_for_positions) */
       HGA_ROT_MODEL = 1,       /* table already in the model dtype */
       HGA_ROT_F32_ROUNDED = 2  /* fp32 table, each entry rounded to the model dtype first (cos.to(x.dtype)) */ };
enum { HGA_OK = 0, HGA_E_INVALID = -1, HGA_E_UNSUPPORTED = -2, HGA_E_CUDA = -3, HGA_E_DEVICE = -4 };

/* Hyper-parameters of one routed-attention layer.  Mirrors RouterConfig + ChunkPlacementPolicy
 * (ExistingModelFineTuning/KvRouter/chunk_router.py:59-90, chunk_placement_policy.py:13-38). */
typedef struct hga_params {
  int32_t batch, nhead, kv_heads, head_dim;
  int32_t chunk_size, group_size;
  int32_t topk_chunks, topk_groups;
  int32_t keep_first, keep_last;
  int32_t cutoff_pair; /* mixed-RoPE cutoff: pairs < cutoff_pair are summed token-wise (vectorized.py:146-165) */
  int32_t dtype;       /* HGA_DTYPE_* of q / k / v / summaries / outputs */
  float scale;         /* head_dim ** -0.5 (chunk_router.py:84-85) */
  float group_kv_scale;/* 1 / (group_size + sqrt(group_size)) (chunk_router.py:87-90) */
} hga_params;

const char* hga_version(void);
const char* hga_last_error(void);

/* (1) Summary builder — mixed-RoPE chunk and group key summaries plus scaled group value sums.
 * Replaces vectorized.py:265-287 (_rope_summary, :168-183) for the chunk-parallel prefill and
 * ChunkRouter._rope_summary_at / _seed_store_from_block / _close_active_chunk
 * (chunk_router.py:553-599, 631-657, 693-700) for the store.
 * Summarises tokens [0, seq_len) of the K/V rows (a partial last chunk uses the middle of its
 * valid tokens as anchor, vectorized.py:265-270) into chunk slots [out_chunk0, out_chunk0+N).
 * Token 0 sits at absolute position pos0 (a multiple of chunk_size).  cos/sin are read at the
 * anchor positions, interpreted per rot_mode (HGA_ROT_*): the chunk-parallel path rounds the fp32
 * table to the model dtype (HierarchicalGlobalAttentionRouted.py:168), the store seed uses fp32
 * (chunk_router.py:702-709).  group_v may be NULL. */
int hga_summaries(const hga_params* p, int64_t seq_len, int64_t pos0,
                  const void* k_raw, const void* k_rope, const void* v, int64_t kv_cap,
                  const void* cos, const void* sin, int32_t rot_mode, int64_t rot_row0,
                  void* chunk_k, void* group_k, void* group_v, int64_t sum_cap, int64_t out_chunk0,
                  cudaStream_t stream);

/* Both summary sets of a fresh prefill from one read of K/V (bf16/fp16, head_dim 64/128, chunk and
 * group sizes multiples of 16; HGA_E_UNSUPPORTED otherwise).  Set A = hga_summaries of all
 * N = ceil(seq_len / chunk_size) chunks with fp32 table A (entries rounded to the model dtype
 * first when round_a != 0: the chunk-parallel path's cos.to(dtype), vectorized.py:265-287) into
 * chunk_a / group_a (capacity sum_cap_a, from slot out_a0).  Set B = the store seed of the first
 * n_b closed chunks with fp32 table B (chunk_router.py:553-599, fixed anchors) into chunk_b /
 * group_b / group_vb (group_vb may be NULL).  Each set equals the corresponding hga_summaries call
 * bit for bit; the K/V rows are read once instead of twice. */
int hga_summaries_dual(const hga_params* p, int64_t seq_len, int64_t pos0, const void* k_raw, const void* k_rope,
                       const void* v, int64_t kv_cap, const float* cos_a, const float* sin_a, int64_t rot_row0_a,
                       int32_t round_a, void* chunk_a, void* group_a, int64_t sum_cap_a, int64_t out_a0,
                       const float* cos_b, const float* sin_b, int64_t rot_row0_b, int64_t n_b, void* chunk_b,
                       void* group_b, void* group_vb, int64_t sum_cap_b, int64_t out_b0, cudaStream_t stream);

/* (2) Two-level router of the chunk-parallel prefill (vectorized.py:296-384).
 * For every (b, h, query chunk n) writes the selected routed chunks and the opened groups that
 * some query row can see, each with t0 = first query row (0..chunk_size-1) of the chunk that sees
 * it; rows t >= t0 see it (the reference's cumulative-OR visibility).  Lists are sorted by
 * chunk / group id and padded with -1:
 *   sel_chunk, sel_t0 [B, H, N, Kc]   Kc = min(topk_chunks, N)
 *   open_gid,  open_t0 [B, H, N, Kg]  Kg = min(topk_groups, Kc*M); gid = chunk*M + group
 * Ties are broken by higher score, then lower index.  dbg_l1 [B,H,N,C,N] / dbg_l2 [B,H,N,C,Kc*M]
 * (fp32, may be NULL) receive the rounded routing scores (l2 in open-candidate order: selected
 * chunks ascending, groups ascending) for the parity tests. */
int hga_route_prefill(const hga_params* p, int64_t seq_len, const void* q, int32_t q_layout,
                      const void* chunk_k, const void* group_k, int64_t sum_cap,
                      int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid, int32_t* open_t0,
                      float* dbg_l1, float* dbg_l2, cudaStream_t stream);

/* hga_route_prefill with an explicit kernel choice: impl 0 = auto, 1 = portable SIMT router,
 * 2 = tcgen05 router (bf16, head_dim 128, chunk 64, group 16, topk_chunks <= 32).  Both
 * implement the same rules and tie order; the tensor-core one accumulates the scoring dot
 * products in a different order (same fp32 accumulator, same bf16 rounding points). */
int hga_route_prefill_impl(const hga_params* p, int64_t seq_len, const void* q, int32_t q_layout,
                           const void* chunk_k, const void* group_k, int64_t sum_cap,
                           int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid, int32_t* open_t0,
                           float* dbg_l1, float* dbg_l2, int32_t impl, cudaStream_t stream);

/* (3)+(4) Working-set attention of the chunk-parallel prefill: replaces the token-segment
 * assembly of vectorized.py:386-490 and RoutedKV.attend(use_summaries=False)
 * (chunk_router.py:139-158).  Query row t of chunk n attends, with an fp32 online softmax, to
 * the causal prefix of its own chunk, the keep_last window [l_lo, n), the keep_first window
 * [0, f_hi) and every opened group with t0 <= t.  Output [B,H,S,Dh] (out_layout 0) or
 * [B,S,H,Dh] (out_layout 1) in p->dtype.  impl: 0 = auto, 1 = portable SIMT kernel,
 * 2 = tcgen05/TMEM tensor-core kernel (bf16, head_dim 128, chunk 64, group 16).  The tensor-core
 * kernel streams whole 16-row units: K/V rows [seq_len, round_up(seq_len, 16)) of every
 * (batch, kv-head) block must hold finite values (the stores zero-fill their buffers). */
int hga_attend_prefill(const hga_params* p, int64_t seq_len, const void* q, int32_t q_layout,
                       const void* k_rope, const void* v, int64_t kv_cap,
                       const int32_t* open_gid, const int32_t* open_t0,
                       void* out, int32_t out_layout, int32_t impl, cudaStream_t stream);

/* Query-chunk ranges of the two prefill steps (the unit a multi-GPU prefill shards): routing /
 * attention of query chunks [chunk_lo, chunk_hi) of a sequence of seq_len tokens, whose keys,
 * summaries and K/V rows cover the whole prefix [0, seq_len).  q holds only the range's rows
 * (sq = min(seq_len, chunk_hi*C) - chunk_lo*C rows per batch entry, same layouts as above); the
 * routing lists are [B, H, chunk_hi - chunk_lo, K] and out holds the range's sq rows.  No
 * counterpart in the reference, which routes a whole block on one device; each chunk's result
 * equals that of the whole-sequence calls. */
int hga_route_prefill_range(const hga_params* p, int64_t seq_len, int64_t chunk_lo, int64_t chunk_hi,
                            const void* q, int32_t q_layout, const void* chunk_k, const void* group_k,
                            int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid,
                            int32_t* open_t0, float* dbg_l1, float* dbg_l2, int32_t impl, cudaStream_t stream);
int hga_attend_prefill_range(const hga_params* p, int64_t seq_len, int64_t chunk_lo, int64_t chunk_hi,
                             const void* q, int32_t q_layout, const void* k_rope, const void* v, int64_t kv_cap,
                             const int32_t* open_gid, const int32_t* open_t0, void* out, int32_t out_layout,
                             int32_t impl, cudaStream_t stream);

/* Projection epilogue of the routed module: q/k RMSNorm + RoPE + KV-store layout in one pass.
 * Replaces the eager prologue of HierarchicalGlobalAttentionRouted.forward
 * (HierarchicalGlobalAttentionRouted.py:151-157) and QwenRoutedAttention.forward
 * (qwen_routed_attention.py:171-176).  qkv: [B, S, row_stride] rows holding H query heads, then
 * KVH key heads, then KVH value heads (Dh each) — one fused projection GEMM.  q_norm_w / k_norm_w
 * (Dh, model dtype) may be NULL (no qk norm).  norm_mode 0 = fp32 weight product (the routed
 * module's RMSNorm), 1 = HF Qwen3 RMSNorm rounding.  rope_mode 0 = fp32 math on an fp32 table,
 * 1 = model-dtype math on a model-dtype table (HF apply_rotary_pos_emb).  Table row r = absolute
 * position rot_row0 + r; token t sits at absolute position pos0 + t.  Writes q_rope [B,S,H,Dh]
 * and rows [kv_row0, kv_row0+S) of k_raw / k_rope / v [B,KVH,kv_cap,Dh]. */
int hga_qkv_prologue(const hga_params* p, int64_t seq_len, const void* qkv, int64_t row_stride,
                     const void* q_norm_w, const void* k_norm_w, float eps, int32_t norm_mode,
                     const void* cos, const void* sin, int32_t rope_mode, int64_t rot_row0, int64_t pos0,
                     void* q_rope, void* k_raw, void* k_rope, void* v, int64_t kv_cap, int64_t kv_row0,
                     cudaStream_t stream);

/* ---- incremental decode (ChunkRouter.decode_block, chunk_router.py:188-407) ----------------
 * A block of L (1 <= L <= chunk_size) new tokens per sequence, all inside the sequence's active
 * chunk; seq_pos [B] (device int32) = absolute position of each sequence's first new token, so
 * the sequences of one batch may sit at different positions (no reference equivalent: the
 * reference keeps one position per layer).  q [B, H, L, Dh] contiguous, RoPE applied.
 *
 * hga_route_decode: routing of chunk_router.py:210-277 against the store's closed-chunk
 * summaries; nmid_max >= the largest routed pool of the batch.  Writes, per (b, h), the routed
 * chunks mid_chunk/mid_t0 [B,H,Kc] and the visible opened groups open_gid/open_t0 [B,H,Kg]
 * (Kc = min(topk_chunks, nmid_max), Kg = min(topk_groups, Kc*M); t0 = first of the L rows that
 * sees it; lists sorted, padded with -1). */
int hga_route_decode(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos,
                     const void* chunk_k, const void* group_k, int64_t sum_cap, int32_t nmid_max,
                     int32_t* mid_chunk, int32_t* mid_t0, int32_t* open_gid, int32_t* open_t0,
                     cudaStream_t stream);

/* hga_attend_decode: token-only attention of one decode block (chunk_router.py:336-401 and the
 * flat branch of RoutedKV.attend, :159-162) over the keep_first window, the keep_last window, the
 * opened groups (rows >= t0) and the active chunk (key u visible to row t iff u <= pos%C + t).
 * Window and active-chunk rows come from `hot`, opened groups from `cold` (the complete token
 * record, may be mapped pinned host memory; with hot_mode 1 any buffer that open_gid indexes by
 * 16-row group, e.g. the VRAM bank of hga_gather_h2d with its open_slot list).  hot_mode 0: hot is addressed like cold (the VRAM
 * tier, hot == cold); hot_mode 1: hot is a slot buffer [B,KVH,(kf+kl+1)*C,Dh] holding first-window
 * chunk c in slot c, last-window chunk c in slot kf + c % kl and the active chunk in slot kf + kl.
 * out [B, H, L, Dh]. */
int hga_attend_decode(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos,
                      const void* hot_k, const void* hot_v, int64_t hot_cap, int32_t hot_mode,
                      const void* cold_k, const void* cold_v, int64_t cold_cap,
                      const int32_t* open_gid, const int32_t* open_t0, int32_t Kg, void* out,
                      cudaStream_t stream);

/* hga_attend_decode_dca: the Dual Chunk Attention variant of hga_attend_decode (the Qwen3
 * wrapper's dca_chunk > 0 path, QwenRoutedAttention._dca_attend, qwen_routed_attention.py:247-283,
 * whose key positions the reference threads back through route_query_block(return_positions=True),
 * chunk_router.py:463-516).  Same key layout, visibility and buffers as hga_attend_decode; the
 * stored keys are the intra-chunk-roped ones (position pos % dca_chunk).  q [B,H,L,Dh] holds the
 * queries BEFORE RoPE; each row is roped three ways in fp32 from dca_cos / dca_sin
 * [dca_ceil + 1][Dh] (fp32 rotate-half tables, row = position): intra at qp = pos % dca_chunk,
 * successor at min(qp + dca_chunk, dca_ceil), inter at dca_ceil, dca_ceil = dca_chunk +
 * dca_local.  A key is scored with the intra query when it lies in the query's DCA chunk
 * (position / dca_chunk equal), the successor query in the chunk just before, else the inter one;
 * fp32 softmax and P.V.  open_pos [B,H,Kg] gives the opened groups' ids for their positions (the
 * routing's open_gid; NULL = open_gid itself, i.e. open_gid is not a bank-slot list). */
int hga_attend_decode_dca(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos,
                          const void* hot_k, const void* hot_v, int64_t hot_cap, int32_t hot_mode,
                          const void* cold_k, const void* cold_v, int64_t cold_cap,
                          const int32_t* open_gid, const int32_t* open_t0, const int32_t* open_pos, int32_t Kg,
                          const float* dca_cos, const float* dca_sin, int32_t dca_chunk, int32_t dca_ceil,
                          void* out, cudaStream_t stream);

/* The two decode entry points above with an explicit kernel choice: impl 0 = automatic (the
 * fast kernels when the shape allows), 1 = the portable kernels, 2 = the fast kernels (routing:
 * L == 1 and head_dim 64/128; attention: bf16/fp16, group_size 16, head_dim 64/128, L <= 8;
 * HGA_E_UNSUPPORTED otherwise).  Both choices compute the same routing rules and attention. */
int hga_route_decode_impl(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos,
                          const void* chunk_k, const void* group_k, int64_t sum_cap, int32_t nmid_max,
                          int32_t* mid_chunk, int32_t* mid_t0, int32_t* open_gid, int32_t* open_t0,
                          int32_t impl, cudaStream_t stream);
int hga_attend_decode_impl(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos,
                           const void* hot_k, const void* hot_v, int64_t hot_cap, int32_t hot_mode,
                           const void* cold_k, const void* cold_v, int64_t cold_cap,
                           const int32_t* open_gid, const int32_t* open_t0, int32_t Kg, void* out,
                           int32_t impl, cudaStream_t stream);

/* hga_gather_h2d: the RAM tier's VRAM token bank, one launch per decode step (the bounded LRU
 * bank of ram_kv_cache_store.py:266-317, its gathers :547-607 and the KV-head union dedup of
 * gather_chunk_tokens_kvh :397-438).  Per (sequence, KV head): the opened groups of the KV head's
 * query heads (open_gid [B,H,Kg], -1 padded) are de-duplicated; groups already in the bank are
 * stamped `stamp` (hits); the others (misses) replace the least recently used slots (smallest
 * stamp, then lowest slot; never a slot stamped by this call) and their 16 token rows of K and V are
 * copied from the record rec_k / rec_v [B,KVH,rec_cap,Dh] (pinned host memory read over the host
 * link, or device memory) into bank_k / bank_v [B,KVH,n_slots*group_size,Dh].  Device maps:
 * slot_gid [B,KVH,n_slots] (-1 = empty), gid_slot [B,KVH,gid_cap] (-1 = absent), slot_stamp
 * [B,KVH,n_slots] (-1 = never used), all owned by the caller and initialised to -1.  open_slot
 * [B,H,Kg] receives each entry's bank slot (-1 for padding), so hga_attend_decode can read the
 * opened groups from the bank (cold = bank, cold_cap = n_slots*group_size, open_gid = open_slot).
 * counters (may be NULL): [0] += unique groups found in the bank, [1] += groups copied.  Requires
 * n_slots >= (H/KVH) * Kg.  Runs on `stream` (a side stream of the caller's choosing, ordered by
 * the caller after the routing and before the attention). */
int hga_gather_h2d(const hga_params* p, const int32_t* open_gid, int32_t Kg, const void* rec_k, const void* rec_v,
                   int64_t rec_cap, void* bank_k, void* bank_v, int32_t n_slots, int32_t* slot_gid, int32_t* gid_slot,
                   int64_t gid_cap, int32_t* slot_stamp, int32_t stamp, int32_t* open_slot,
                   unsigned long long* counters, cudaStream_t stream);

/* hga_append_tokens: write L new K (RoPE applied) / V rows per sequence at seq_pos into the hot
 * rows (and, for hot_mode 1, the cold record), and their pre-RoPE K into active_raw
 * [B,KVH,C,Dh] (may be NULL) — ChunkRouter._append_active (chunk_router.py:603-614). */
int hga_append_tokens(const hga_params* p, int32_t L, const int32_t* seq_pos, const void* k_rope,
                      const void* v, const void* k_raw, void* hot_k, void* hot_v, int64_t hot_cap,
                      int32_t hot_mode, void* cold_k, void* cold_v, int64_t cold_cap, void* active_raw,
                      cudaStream_t stream);

/* Unpack of a multi-GPU prefill's all-gathered buffer (no counterpart in the reference, which
 * runs on one device).  Rank r's data starts at recv + r * rank_stride (bytes); one part of it
 * starts part_offset bytes further and holds `pieces` blocks of [bk][rows][row_bytes], piece j of
 * rank r being block dst_block[r * pieces + j] (a host array) of the sequence.  dst receives
 * [bk][world * pieces][rows][row_bytes].  row_bytes, the strides and both pointers must be 16-byte
 * aligned; world * pieces <= 128. */
int hga_shard_unpack(const void* recv, int64_t rank_stride, int64_t part_offset, int32_t world, int32_t pieces,
                     const int32_t* dst_block, int64_t bk, int64_t rows, int64_t row_bytes, void* dst,
                     cudaStream_t stream);

/* Device-side error words: 0, or the first code recorded.  The tensor-core kernels record a
 * bounded mbarrier wait that timed out (the CTA then released its TMEM and returned without
 * output); the decode kernels record 0x101 / 0x102 / 0x103 (routing / attention / append) when a
 * sequence position or a list entry addresses rows past a buffer's capacity (those rows are
 * skipped; a (b, h) whose position is past the capacity gets a zero output), and 0x101 also when
 * a sequence's routed pool exceeds the nmid_max given to hga_route_decode (its lists stay -1).
 * Synchronous (reads device memory); clear != 0 resets the words. */
int hga_device_status(int32_t* code, int32_t clear);

/* Test hook of the bounded waits' failure path (no reference counterpart).  Sets, for the next
 * tensor-core hga_attend_prefill launch only, the limit of its bounded mbarrier waits
 * (wait_limit_ns; 0 = the default 2 s) and, with mode 1, makes the CTA of the last query chunk,
 * query heads 0-1, batch row 0 skip its tile-1 K load, so that a wait of that CTA runs out: it
 * records the wait's code (hga_device_status), lets its copies and MMAs in flight land, releases
 * its TMEM and returns without writing its rows.  Nothing faults or hangs; every later launch
 * runs normally.  Not thread-safe; for tests. */
int hga_debug_fault(int32_t mode, int64_t wait_limit_ns);

#ifdef __cplusplus
}
#endif
#endif /* HGA_B200_H_ */
