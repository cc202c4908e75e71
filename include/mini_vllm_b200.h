/*
 * mini_vllm_b200.h — C ABI of the B200 paged-attention library (libmvb200.so).
 *
 * The library replaces the Triton kernels behind mini-vLLM's attention plug-in
 * (mini_vllm/attention/paged_attention_gpu.py) with hand-written sm_100a CUDA.
 * Every entry point takes plain pointers, sizes and strides; nothing in these
 * signatures is a torch type, so ctypes, cgo, JNI or N-API can bind them.
 *
 * Conventions shared by all entry points
 *  - Tensors live in device memory of the current CUDA device.
 *  - Strides are in ELEMENTS, not bytes; the innermost (head_dim) dimension of
 *    every tensor must be contiguous.
 *  - The KV pool tensors have the reference layout
 *        key_cache[num_blocks][num_kv_heads][block_size][head_dim]
 *    (mini_vllm/cache/pool.py:93-102), contiguous.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). No entry point
 *    synchronises; all work is enqueued on `stream`.
 *  - The return value is a host-side status (MVB_OK or a negative MVB_ERR_*)
 *    and no C++ exception ever crosses the ABI.  Problems that only the device
 *    can see (a bad slot, a bad block id, kv_len < 1, a duplicate slot) are
 *    OR-ed as MVB_DEV_* bits into the caller's int32 `error_flags` word in
 *    device memory; the caller reads it when it wants the check (the Python
 *    shim reads it after every call in strict mode, which mirrors the host
 *    syncs the reference performs at paged_attention_gpu.py:128-135,296).
 */
#ifndef MINI_VLLM_B200_H
#define MINI_VLLM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element types of the KV pool / query / output ---------------------- */
#define MVB_DTYPE_F32  0
#define MVB_DTYPE_F16  1
#define MVB_DTYPE_BF16 2

/* ---- host-side status codes --------------------------------------------- */
#define MVB_OK                 0
#define MVB_ERR_INVALID_ARG   -1  /* shape / size / stride inconsistency       */
#define MVB_ERR_DTYPE         -2  /* unsupported element type                  */
#define MVB_ERR_HEAD_DIM      -3  /* head_dim not in {64, 128}                 */
#define MVB_ERR_BLOCK_SIZE    -4  /* block_size not a positive power of two    */
#define MVB_ERR_ALIGNMENT     -5  /* pointer or stride breaks the vector width */
#define MVB_ERR_CUDA          -6  /* a CUDA runtime call or launch failed      */
#define MVB_ERR_WORKSPACE     -7  /* split-K workspace missing or too small    */
#define MVB_ERR_TENSOR_MAP    -8  /* cuTensorMapEncodeTiled failed             */
#define MVB_ERR_VARIANT       -9  /* requested kernel variant cannot run here  */
#define MVB_ERR_HEADS        -10  /* num_heads not a multiple of num_kv_heads  */

/* ---- device-side error bits (OR-ed into *error_flags) ------------------- */
#define MVB_DEV_KV_LEN        1   /* some kv_len_after < 1                      */
#define MVB_DEV_BLOCK_ID      2   /* a block id needed by kv_len is <0 or >=NB  */
#define MVB_DEV_TABLE_SHORT   4   /* ceil(kv_len/block_size) > max_blocks       */
#define MVB_DEV_SLOT_RANGE    8   /* slot not -1 and outside [0, NB*BS)         */
#define MVB_DEV_DUP_SLOT     16   /* two tokens of one write target one slot    */
#define MVB_DEV_TIMEOUT      32   /* a bounded pipeline wait ran out            */
#define MVB_DEV_POSITION     64   /* a rope position outside the cos/sin table  */
#define MVB_DEV_SCHEDULE    128   /* a decode schedule did not fit its workspace
                                     (internal: the planned bound was wrong)   */

/* ---- decode kernel variants --------------------------------------------- */
#define MVB_DECODE_AUTO 0  /* bf16/f16, BS%16==0: MMA unsplit for contexts <= 256
                              tokens, MMA split-K when its 512-token partitions fill
                              at most 2 CTAs per SM, else STREAM (<= 4096 sequences),
                              else SCHED; FMA for everything else                   */
#define MVB_DECODE_FMA  1  /* CUDA-core FP32 FMA kernel (any dtype, any BS)      */
#define MVB_DECODE_MMA  2  /* TMA-staged tensor-core kernel, one CTA per (seq, KV head),
                              split-K + reduction for long contexts (bf16/f16, BS%16==0) */
#define MVB_DECODE_STREAM 3 /* persistent stream-K variant of MVB_DECODE_MMA: equal tile
                              ranges per warp + a fixup kernel merging cut units
                              (num_seqs <= 4096) */
#define MVB_DECODE_SCHED 4  /* scheduled persistent variant (bf16/f16, BS%16==0, up to 16384
                              sequences): a per-step schedule cuts the tile stream of every
                              (seq, KV head) unit into one equal range per SM and resolves
                              its pool rows; one CTA per SM streams its range with
                              self-issuing consumer warps, and the last piece of a unit cut
                              by a range boundary merges it */

/* Logical -> physical gather of cached K/V for a batch of sequences (the
 * prefill path's prefix read) into contiguous [total_tokens, KH, D] outputs:
 *   key_out[out_offsets[i] + p] = key_cache[block_table[seq_rows[i]][p / BS], :, p % BS, :]
 * for p < out_offsets[i + 1] - out_offsets[i] (same for value_out).
 * Replaces gather_prefix_kv / _gather_prefix_kv_kernel
 * (mini_vllm/attention/paged_attention_gpu.py:329-433) and batches
 * gather_paged_kv (mini_vllm/cache/cache_read.py:19-84).
 * block_table: int64 [block_table_rows, >= max_blocks_per_seq], row stride
 * block_table_stride; seq_rows: int64 [num_seqs] rows of it; out_offsets:
 * int64 [num_seqs + 1], an exclusive prefix of the token counts
 * (out_offsets[num_seqs] == total_tokens), all device memory.  Rows must be
 * 16-byte multiples (head_dim * element size) and every pointer 16-byte aligned.
 * Device errors (the row is zero-filled): a logical block past
 * max_blocks_per_seq -> MVB_DEV_TABLE_SHORT; a block id outside
 * [0, num_blocks) or a sequence row outside the table -> MVB_DEV_BLOCK_ID;
 * offsets that are not an increasing prefix from 0 -> MVB_DEV_KV_LEN.
 * work_counter: optional, two 4-byte-aligned uint32 device words that are zero
 * before the call (zero them once when allocating them); every call leaves
 * them zero again.  With them the tile-copy kernel hands the last half of the
 * work out in small pieces, so that SMs with more memory bandwidth take more
 * of it; NULL splits the work evenly in advance (same result, slower tail).
 * Calls that share the words must not overlap on the GPU: give each stream
 * its own pair. */
int mvb_paged_gather(const void* key_cache, const void* value_cache, const int64_t* block_table,
                     int64_t block_table_rows, int64_t block_table_stride, int32_t max_blocks_per_seq,
                     const int64_t* seq_rows, const int64_t* out_offsets, void* key_out, void* value_out,
                     int32_t num_seqs, int64_t total_tokens, int32_t num_kv_heads, int32_t head_dim,
                     int32_t block_size, int32_t num_blocks, int32_t dtype, uint32_t* work_counter,
                     int32_t* error_flags, void* stream);

/* Causal paged prefill attention of a batch of chunks, read in place from the
 * paged pool on the tensor cores (bf16 / f16, head_dim 64 or 128, any power-of-
 * two block_size).  Chunk i has query_len[i] query tokens at rows
 * [sum_{j<i} query_len[j], ...) of `query` (and `out`), the block-table row
 * seq_rows[i], and cached_len[i] tokens already in the cache before it; its
 * token t attends cache positions [0, cached_len[i] + t].  Positions before
 * cached_len[i] are read from the pool; the chunk's own positions from `key` /
 * `value` ([total_q, KH, D] rows, strides in elements) when given, else from the
 * pool (the reference's runner writes the chunk into the cache before
 * attention).  seq_rows / cached_len / query_len are int64 device arrays
 * (num_chunks <= 4096), so the call needs no host synchronisation; the chunks
 * must hold at most total_q tokens (else MVB_DEV_BLOCK_ID and no output), and
 * a chunk whose cache end exceeds max_blocks_per_seq * block_size gets zero
 * rows and MVB_DEV_TABLE_SHORT.  Replaces AttentionBackendGPU.prefill_attention
 * (mini_vllm/attention/paged_attention_gpu.py:577-661: per-sequence gather of
 * the prefix, concatenation with the chunk, GQA repeat and torch SDPA with the
 * offset causal mask). */
int mvb_paged_prefill(const void* query, int64_t q_stride_tok, int64_t q_stride_head, const void* key,
                      int64_t k_stride_tok, int64_t k_stride_head, const void* value, int64_t v_stride_tok,
                      int64_t v_stride_head, const void* key_cache, const void* value_cache,
                      const int64_t* block_table, int64_t block_table_rows, int64_t block_table_stride,
                      int32_t max_blocks_per_seq, const int64_t* seq_rows, const int64_t* cached_len,
                      const int64_t* query_len, int32_t num_chunks, int32_t total_q, void* out,
                      int64_t out_stride_tok, int64_t out_stride_head, int32_t num_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t block_size, int32_t num_blocks, float scale, int32_t dtype,
                      int32_t* error_flags, void* stream);

/* Rotary position embedding of the step's query and key rows fused with the
 * paged KV-cache write of the rotated keys and the values: bit for bit the
 * reference's  q = rope(q, pos); k = rope(k, pos); write_kv_cache(k, v, slots)
 * (mini_vllm/model_runner/qwen_runner.py:163-170, mini_vllm/model/rotary.py:47-85:
 * out = x * cos[pos] + rotate_half(x) * sin[pos], each operation rounded to the
 * dtype).  query / key / value: [T, H|KH|KH, D] with element strides (value may
 * be a view of the fused QKV output); query_out: [T, H, D] with strides (may
 * equal query); key_out: optional contiguous [T, KH, D] receiving the rotated
 * keys (NULL: cache only); positions: int64 [T]; cos_table / sin_table:
 * contiguous [table_rows, D] of the same dtype (the RotaryEmbedding cache).
 * Slots follow mvb_kv_cache_write (-1 skipped, range and duplicate checks);
 * a position outside [0, table_rows) sets MVB_DEV_POSITION and leaves that
 * token's query/key rows unwritten.  Replaces, as one launch, RotaryEmbedding.__call__
 * for q and k and triton_cache_write (paged_attention_gpu.py:90-154). */
int mvb_rope_kv_cache_write(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                            void* query_out, int64_t qo_stride_token, int64_t qo_stride_head,
                            const void* key, int64_t k_stride_token, int64_t k_stride_head,
                            const void* value, int64_t v_stride_token, int64_t v_stride_head,
                            const int64_t* positions, const void* cos_table, const void* sin_table,
                            int64_t table_rows, void* key_cache, void* value_cache,
                            const int64_t* slot_mapping, void* key_out, int32_t num_tokens,
                            int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                            int32_t block_size, int32_t num_blocks, int32_t dtype,
                            uint32_t* slot_claims, uint32_t epoch, int32_t* error_flags,
                            void* stream);

/* The per-step attention metadata on the device, for a step of num_seqs
 * sequences (prefill chunks first, then decodes): replaces the per-token host
 * loops of ModelInputBuilder.build (mini_vllm/engine/input_builder.py:48-196).
 * Inputs (device, int64): sequence s's block table B_s is
 * blocks[block_starts[s] .. block_starts[s] + block_counts[s]) (the lists
 * concatenated, or the rows of a padded table); cached_len [S] =
 * cached_len_before; token_offsets [S + 1] the exclusive prefix of the query
 * lengths q_s.  Outputs (device): positions [T] = c_s + i; slot_mapping [T] =
 * B_s[p / BS] * BS + p % BS (input_builder.py:202-221); block_tables
 * [S, max_blocks] int64, B_s then -1 padding (input_builder.py:238-256);
 * kv_len_after [S] int32 = c_s + q_s.  A position past B_s sets
 * MVB_DEV_TABLE_SHORT (the reference's "Block not allocated") and gets slot -1. */
int mvb_build_step_metadata(const int64_t* blocks, const int64_t* block_starts, const int64_t* block_counts,
                            const int64_t* cached_len, const int64_t* token_offsets, int32_t num_seqs,
                            int64_t num_tokens, int32_t max_blocks, int32_t block_size, int64_t* positions,
                            int64_t* slot_mapping, int64_t* block_tables, int32_t* kv_len_after,
                            int32_t* error_flags, void* stream);

/* Test hook of the bounded waits — no reference counterpart.  Runs
 * mvb_paged_decode with `variant` (MVB_DECODE_STREAM or MVB_DECODE_SCHED),
 * except that the load of one tile is never issued and every pipeline wait
 * gives up after `wait_limit` (1 .. 2^22) try-waits.  The held tile is local
 * tile `hold_tile` of stream warp `hold_warp` (MVB_DECODE_STREAM), or tile
 * number `hold_tile` of consumer warp `hold_warp` (CTA * consumers per CTA +
 * consumer, 11 consumers at head_dim 64 and 6 at 128; MVB_DECODE_SCHED).  The wait
 * on it runs out and reports MVB_DEV_TIMEOUT; the kernel's other waits give up
 * too (the scheduled kernel aborts the whole CTA), each role waits (bounded)
 * for its own loads in flight and leaves, and the context stays usable.  Used
 * by the failure-detection test; never needed in production. */
int mvb_test_decode_wait_timeout(const void* query, int64_t q_stride_seq, int64_t q_stride_head,
                                 const void* key_cache, const void* value_cache,
                                 const int64_t* block_table, int64_t block_table_stride,
                                 int32_t max_blocks_per_seq, const int32_t* kv_len, void* out,
                                 int64_t out_stride_seq, int64_t out_stride_head, int32_t num_seqs,
                                 int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t block_size, int32_t num_blocks, float scale, int32_t dtype,
                                 void* workspace, int64_t workspace_bytes, int32_t* error_flags,
                                 void* stream, int32_t hold_warp, int32_t hold_tile, int32_t wait_limit,
                                 int32_t variant);

/* Flag ORed into `variant` of mvb_paged_decode (ignored by the plan): the
 * kernel launched immediately before this call on `stream` is
 * mvb_kv_cache_write (or a kernel that signals its dependents only when it
 * finishes).  The stream kernel then reads query, block_table and kv_len and
 * resolves its first tiles BEFORE waiting for that kernel, overlapping its
 * set-up with the write; only the cache reads wait.  Without the flag every
 * input is read after the wait.  A preceding kernel that signals its
 * dependents early and still writes query, block_table or kv_len afterwards
 * must not be followed by a call with this flag. */
#define MVB_DECODE_AFTER_WRITE 0x100

/* Flag ORed into `variant` of mvb_paged_decode (the stream and scheduled
 * kernels): the workspace already holds the schedule of this batch, built by
 * mvb_paged_decode_schedule from the same kv_len and block-table contents and
 * shape arguments (kv_len and the block tables are the same for every layer of a model step,
 * so one schedule serves all of them).  Without the flag the call builds the
 * schedule itself (one extra launch).  The decode reads the schedule before
 * its grid-dependency wait only when MVB_DECODE_AFTER_WRITE is also set; the
 * kernel right before it is then the KV write, which starts only after the
 * schedule kernel has finished. */
#define MVB_DECODE_SCHEDULE_READY 0x200

/*
 * Build the per-step decode schedule of a batch into `workspace`, for the
 * kernel the plan picks for `variant` (MVB_DECODE_AUTO and the shape
 * arguments of the decodes that will use it).  kv_len and the block tables are
 * the same for every layer of a model step, so one schedule serves all of them
 * (mvb_paged_decode with MVB_DECODE_SCHEDULE_READY).
 *   MVB_DECODE_STREAM: the stream kernel's set-up — the tile prefix of the
 *     step, the pool row of every tile, and for every stream warp its tile range
 *     with its first 32 rows — so each decode issues its first loads after one
 *     read instead of deriving them from kv_len and the tables.
 *   MVB_DECODE_SCHED: the scheduled kernel's per-SM tile ranges, their pieces
 *     and pool rows.
 *   any other kernel: nothing to build; returns MVB_OK.
 * It reads kv_len (int32 [num_seqs]) and the block tables (int64, row stride
 * block_table_stride), both in device memory; workspace_bytes must be at least
 * the plan's (mvb_paged_decode_plan with the same arguments).  A sequence whose
 * kv_len is < 1 or needs more than max_blocks_per_seq blocks sets
 * MVB_DEV_KV_LEN / MVB_DEV_TABLE_SHORT and gets zero output rows from every
 * decode that uses the schedule; a block id outside [0, num_blocks) sets
 * MVB_DEV_BLOCK_ID and its tile is skipped.  `flags`: MVB_DECODE_AFTER_WRITE
 * when the kernel launched just before on `stream` is the KV write (the
 * schedule is then computed while the write runs).  No reference counterpart:
 * the Triton decode (paged_attention_gpu.py:252-321) has no per-step set-up;
 * this hoists the work every layer's decode would repeat (the kv_len prefix and
 * the block-table walk) out of the per-layer calls.  A decode that reported
 * MVB_DEV_TIMEOUT may leave a scheduled kernel's counters dirty: build it again
 * before the next call.
 */
int mvb_paged_decode_schedule(const int32_t* kv_len, const int64_t* block_table,
                              int64_t block_table_stride, int32_t num_seqs, int32_t num_heads,
                              int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                              int32_t num_blocks, int32_t max_blocks_per_seq, int32_t dtype,
                              int32_t variant, int32_t flags, void* workspace,
                              int64_t workspace_bytes, int32_t* error_flags, void* stream);

/* ABI version; bumped whenever a signature below changes. */
int mvb_abi_version(void);

/* Human-readable text for a host status code (static storage). */
const char* mvb_status_string(int status);

/*
 * KV-cache write: for every token t with slot_mapping[t] != -1,
 *     key_cache  [slot / BS][h][slot % BS][:] = key  [t][h][:]
 *     value_cache[slot / BS][h][slot % BS][:] = value[t][h][:]
 * for all KV heads h.  Replaces triton_cache_write / _cache_write_kernel
 * (mini_vllm/attention/paged_attention_gpu.py:90-154, :32-87) and computes the
 * same bytes as the torch oracle write_to_paged_cache
 * (mini_vllm/cache/cache_write.py:25-74).
 *
 * key/value may be strided views (e.g. V as a slice of a fused QKV output);
 * pass their token and head strides.  A slot outside [0, NB*BS) other than -1
 * is skipped and sets MVB_DEV_SLOT_RANGE.  When `slot_claims` is non-NULL it
 * must point to NB*BS zero-initialised uint32 words that persist across calls;
 * `epoch` must differ from every epoch used before with that array (never 0),
 * and two tokens that target one slot set MVB_DEV_DUP_SLOT (the reference
 * forbids duplicates, paged_attention_gpu.py:126-135).
 */
int mvb_kv_cache_write(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                       const void* value, int64_t value_stride_token, int64_t value_stride_head,
                       void* key_cache, void* value_cache,
                       const int64_t* slot_mapping, int32_t num_tokens,
                       int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                       int32_t num_blocks, int32_t dtype,
                       uint32_t* slot_claims, uint32_t epoch,
                       int32_t* error_flags, void* stream);

/*
 * Plan a paged decode: picks the kernel variant and the split-K partition
 * length for the given shape and returns the workspace size in bytes (0 when
 * the decode needs none) and the number of kernels one mvb_paged_decode call
 * launches without MVB_DECODE_SCHEDULE_READY (launches_out; NULL to skip).
 * MVB_DECODE_STREAM reports partition_tokens = 0 and num_partitions = 0; its
 * workspace needs no initialisation, and one workspace serves one stream at a
 * time.  `variant` / `partition_tokens` are the caller's
 * requests (MVB_DECODE_AUTO / 0 = let the library choose).  `cache_ptr` is
 * only inspected for TMA alignment (it may be NULL, in which case alignment
 * is assumed).
 */
int mvb_paged_decode_plan(int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                          int32_t head_dim, int32_t block_size, int32_t num_blocks,
                          int32_t max_blocks_per_seq, int32_t dtype,
                          int32_t variant, int32_t partition_tokens, const void* cache_ptr,
                          int32_t* variant_out, int32_t* partition_tokens_out,
                          int32_t* num_partitions_out, int64_t* workspace_bytes_out,
                          int32_t* launches_out);

/*
 * Paged decode attention, one query token per sequence:
 *   out[s][h][:] = softmax(scale * q[s][h] . K[s][h/G]^T) . V[s][h/G]
 * over kv_len[s] tokens reached through block_table[s][0 .. ceil(kv_len/BS)).
 * G = num_heads / num_kv_heads (repeat_interleave GQA mapping).  Replaces
 * triton_decode_attention / _paged_decode_kernel
 * (mini_vllm/attention/paged_attention_gpu.py:252-321, :162-249); the math is
 * that of AttentionBackendRef.decode_attention
 * (mini_vllm/attention/paged_attention_ref.py:102-161).
 *
 * block_table is int64 [num_seqs][max_blocks_per_seq] (-1 padded, row stride
 * block_table_stride); kv_len is int32 [num_seqs]; query/out are
 * [num_seqs][num_heads][head_dim] with the given strides; out has the query's
 * dtype.  When the plan (same arguments) says num_partitions > 1 the call runs
 * the flash-decoding split-K kernel followed by the cross-partition reduction
 * and needs `workspace` of at least workspace_bytes (256-byte aligned).
 * MVB_DECODE_STREAM also needs the workspace (see mvb_paged_decode_plan).
 */
int mvb_paged_decode(const void* query, int64_t q_stride_seq, int64_t q_stride_head,
                     const void* key_cache, const void* value_cache,
                     const int64_t* block_table, int64_t block_table_stride,
                     int32_t max_blocks_per_seq, const int32_t* kv_len,
                     void* out, int64_t out_stride_seq, int64_t out_stride_head,
                     int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                     int32_t head_dim, int32_t block_size, int32_t num_blocks,
                     float scale, int32_t dtype, int32_t variant, int32_t partition_tokens,
                     void* workspace, int64_t workspace_bytes,
                     int32_t* error_flags, void* stream);

/*
 * Paged decode without a caller workspace.  This entry point has no
 * counterpart in the reference; it exists for callers that cannot allocate
 * device memory at decode time — a serving process that gives all free HBM to
 * the KV pool at start-up and allows no allocation afterwards, or a host
 * binding (cgo, JNI, a C runtime) with no device allocator of its own.
 *
 * Same arguments and results as mvb_paged_decode without `workspace` /
 * `workspace_bytes`.  It runs the split-K family only (variant MVB_DECODE_AUTO
 * picks MVB_DECODE_MMA when eligible, else MVB_DECODE_FMA; MVB_DECODE_STREAM
 * returns MVB_ERR_VARIANT) and keeps the partial states in a 16 MiB device
 * array inside the library: a shape whose workspace (mvb_paged_decode_plan)
 * exceeds 16 MiB returns MVB_ERR_WORKSPACE.  It calls no cudaMalloc, cudaFree
 * or allocating library routine.  Every GPU that loads the library holds the
 * array until exit; the first call on a device looks up its address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * All calls on one device share that device's copy of the array and find the
 * previous call's contents there: calls that overlap on the same GPU (for
 * example on two streams) race on it and must be ordered by the caller.
 * Each device has its own copy, so calls on different devices do not race.
 */
int mvb_paged_decode_noalloc(const void* query, int64_t q_stride_seq, int64_t q_stride_head,
                             const void* key_cache, const void* value_cache,
                             const int64_t* block_table, int64_t block_table_stride,
                             int32_t max_blocks_per_seq, const int32_t* kv_len,
                             void* out, int64_t out_stride_seq, int64_t out_stride_head,
                             int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t block_size, int32_t num_blocks,
                             float scale, int32_t dtype, int32_t variant, int32_t partition_tokens,
                             int32_t* error_flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINI_VLLM_B200_H */
