// C ABI of libmvb200.so: argument checks, the decode plan (kernel variant and
// split-K partitioning), the TMA tensor-map cache, and the launches.
// Declarations and contracts: include/mini_vllm_b200.h.
#include <cudaTypedefs.h>

#include <mutex>

#include "mvb_common.cuh"

namespace mvb {

cudaError_t launch_kv_write(const void* key, int64_t k_st, int64_t k_sh, const void* value,
                            int64_t v_st, int64_t v_sh, void* kc, void* vc, const int64_t* slots,
                            int num_tokens, int kh, int row_bytes, int esize, int block_size,
                            int64_t total_slots, uint32_t* claims, uint32_t epoch, int* err,
                            cudaStream_t stream, int sm_count);
cudaError_t launch_decode_fma(const DecodeArgs& a, int dtype, int head_dim, int maxg,
                              cudaStream_t stream);
cudaError_t launch_decode_reduce(const DecodeArgs& a, int dtype, int head_dim, cudaStream_t stream);
cudaError_t launch_decode_mma(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                              int dtype, int head_dim, int max_bids, cudaStream_t stream);
cudaError_t launch_decode_stream(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                                 int dtype, int head_dim, int* scratch, float* part, int max_warps,
                                 int sm_count, const StreamSchedPtrs* sp, cudaStream_t stream);
cudaError_t launch_decode_stream_schedule(const DecodeArgs& a, int dtype, int head_dim, int max_warps, int sm_count,
                                          const StreamSchedPtrs& sp, bool wait_at_end, cudaStream_t stream);
int stream_warps_per_cta(int head_dim);
int stream_smem_bytes(int head_dim, int num_seqs);
constexpr int kPrefillMaxSeqsHost = 4096;  // chunks per prefill launch (prefill_mma.cu)
constexpr int kPrefillHeadsHost = 8;       // query heads per prefill CTA (prefill_mma.cu)
cudaError_t launch_prefill(const PrefillArgs& a, int dtype, int head_dim, cudaStream_t stream);
int prefill_smem_bytes(int head_dim, int n);
SchedLayout sched_layout(int num_seqs, int num_kv_heads, int head_groups, int G, int max_blocks,
                         int block_size, int head_dim, int ctas);
cudaError_t launch_decode_schedule(const DecodeArgs& a, int head_dim, const SchedLayout& l, void* ws,
                                   bool wait_at_end, cudaStream_t stream);
cudaError_t launch_decode_sched(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a, int dtype,
                                int head_dim, const SchedLayout& l, void* ws, cudaStream_t stream);

// cuTensorMapEncodeTiled from the driver (nullptr when the driver lacks it);
// shared by the decode (pool maps) and the gather (output maps).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

namespace {

constexpr int kAbiVersion = 6;
// Longest context the auto plan serves with one CTA per (sequence, KV head);
// beyond it the flash-decoding split is used.
constexpr int64_t kUnsplitMaxTokens = 8192;
// Split-K partition length of the auto plan (the north-star's 512 tokens).
constexpr int kAutoPartitionTokens = 512;
// AUTO: contexts up to this many tokens run one CTA per (sequence, KV head, head group), unsplit.
constexpr int64_t kAutoShortTokens = 256;
// Largest partition an MMA CTA accepts (bounds its block-id cache).
constexpr int kMmaMaxPartitionTokens = 65536;
constexpr int kMmaHeadGroup = 16;
// Largest batch the stream kernel serves (its CTAs hold the per-sequence tile prefix in smem).
constexpr int kStreamMaxSeqs = 4096;

// Shared memory of one B200 SM, used when no device can be queried.
constexpr int kDefaultSmemPerSm = 233472;

int elem_size(int dtype) { return dtype == MVB_DTYPE_F32 ? 4 : 2; }
bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }
int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

int sm_count_current() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int smem_per_sm_current() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kDefaultSmemPerSm;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess || v <= 0)
      v = kDefaultSmemPerSm;
    cache[dev] = v;
  }
  return cache[dev];
}

struct Plan {
  int variant;
  int part_tokens;
  int num_parts;
  int head_groups;
  int maxg;      // heads per CTA group
  int max_bids;  // block-table entries one partition can span
  int64_t ws_bytes;
  int64_t off_m, off_l;  // workspace offsets of the m / l arrays
  int max_warps;         // stream variant: warps the partial-state slots cover
  int64_t off_part;      // stream variant: workspace offset of the partial slots
  // stream variant: its per-step schedule after the per-launch part
  int64_t off_shdr, off_spre, off_sctx, off_srows, off_srec, off_sdesc;
  SchedLayout sched;     // sched variant: workspace layout
};

StreamSchedPtrs stream_sched_ptrs(const Plan& pl, char* ws) {
  StreamSchedPtrs sp;
  sp.hdr = ws + pl.off_shdr;
  sp.pre = reinterpret_cast<const int*>(ws + pl.off_spre);
  sp.ctx = reinterpret_cast<const int*>(ws + pl.off_sctx);
  sp.rows = reinterpret_cast<const int*>(ws + pl.off_srows);
  sp.rec = ws + pl.off_srec;
  sp.desc = ws + pl.off_sdesc;
  return sp;
}

int make_plan(int num_seqs, int num_heads, int num_kv_heads, int head_dim, int block_size,
              int num_blocks, int max_blocks, int dtype, int variant, int partition_tokens,
              const void* cache_ptr, Plan* pl) {
  if (dtype != MVB_DTYPE_F32 && dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16)
    return MVB_ERR_DTYPE;
  if (head_dim != 64 && head_dim != 128) return MVB_ERR_HEAD_DIM;
  if (!is_pow2(block_size)) return MVB_ERR_BLOCK_SIZE;
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || max_blocks < 0)
    return MVB_ERR_INVALID_ARG;
  if (num_heads % num_kv_heads != 0) return MVB_ERR_HEADS;
  const int G = num_heads / num_kv_heads;
  const int64_t rows = (int64_t)num_blocks * num_kv_heads * block_size;
  if (rows * head_dim >= ((int64_t)1 << 62)) return MVB_ERR_INVALID_ARG;

  const bool aligned = cache_ptr == nullptr || (reinterpret_cast<uintptr_t>(cache_ptr) & 15) == 0;
  const bool mma_ok =
      dtype != MVB_DTYPE_F32 && block_size % 16 == 0 && aligned && rows < ((int64_t)1 << 31);
  const int64_t max_ctx_tiles = ((int64_t)max_blocks * block_size + 15) / 16;
  const int khg16 = num_kv_heads * ((G + kMmaHeadGroup - 1) / kMmaHeadGroup);
  const bool stream_ok = mma_ok && num_seqs <= kStreamMaxSeqs &&
                         (int64_t)num_seqs * khg16 * max_ctx_tiles < ((int64_t)1 << 31);
  const int hg16 = (G + kMmaHeadGroup - 1) / kMmaHeadGroup;
  SchedLayout sl = sched_layout(num_seqs, num_kv_heads, hg16, G, max_blocks, block_size, head_dim,
                                sm_count_current());
  const bool sched_ok = mma_ok && sl.ok;
  int v = variant;
  // AUTO, from the batch x context sweep (bench.py --op sweep, 14/2/64 bf16):
  //  * contexts of at most kAutoShortTokens: one CTA per (sequence, KV head,
  //    head group), unsplit (5.6 us at 1-64 sequences of 128 tokens, where the
  //    persistent kernels' fixed cost is 8-12 us);
  //  * little work: 512-token split-K partitions of at most 2 CTAs per SM
  //    (15.5 us for 1 x 8192 tokens against 58 us streamed through the
  //    whole GPU);
  //  * else the stream kernel where it applies (fastest at configs 2-4), the
  //    scheduled kernel past its batch limit, CUDA cores for the rest.
  int64_t auto_pt = 0;
  if (v == MVB_DECODE_AUTO) {
    const int64_t max_ctx_tok = (int64_t)max_blocks * block_size;
    const int64_t split_ctas = (int64_t)num_seqs * khg16 * ((max_ctx_tok + kAutoPartitionTokens - 1) / kAutoPartitionTokens);
    if (mma_ok && max_ctx_tok <= kAutoShortTokens) {
      v = MVB_DECODE_MMA;
      auto_pt = max_ctx_tok > 0 ? max_ctx_tok : 16;
    } else if (mma_ok && split_ctas <= 2 * (int64_t)sm_count_current()) {
      v = MVB_DECODE_MMA;
      auto_pt = kAutoPartitionTokens;
    } else {
      v = stream_ok ? MVB_DECODE_STREAM : sched_ok ? MVB_DECODE_SCHED : MVB_DECODE_FMA;
    }
  }
  if (v != MVB_DECODE_FMA && v != MVB_DECODE_MMA && v != MVB_DECODE_STREAM && v != MVB_DECODE_SCHED)
    return MVB_ERR_VARIANT;
  if (v == MVB_DECODE_MMA && !mma_ok) return MVB_ERR_VARIANT;
  if (v == MVB_DECODE_STREAM && !stream_ok) return MVB_ERR_VARIANT;
  if (v == MVB_DECODE_SCHED && !sched_ok) return MVB_ERR_VARIANT;
  pl->sched = sl;

  if (v == MVB_DECODE_SCHED) {
    pl->variant = v;
    pl->part_tokens = 0;
    pl->num_parts = 0;
    pl->head_groups = hg16;
    pl->maxg = kMmaHeadGroup;
    pl->max_bids = 0;
    pl->max_warps = 0;
    pl->off_m = pl->off_l = pl->off_part = 0;
    pl->ws_bytes = sl.bytes;
    return MVB_OK;
  }

  if (v == MVB_DECODE_STREAM) {
    // One contiguous tile range per warp; workspace = one 32-byte cut-unit
    // descriptor and two partial-state slots per warp of the largest grid the
    // GPU can hold.
    const int nw = stream_warps_per_cta(head_dim);
    const int smem = stream_smem_bytes(head_dim, num_seqs);
    int per_sm = smem_per_sm_current() / (smem + 1024);
    if (per_sm > 2048 / (nw * 32)) per_sm = 2048 / (nw * 32);
    if (per_sm < 1) per_sm = 1;
    pl->variant = v;
    pl->part_tokens = 0;
    pl->num_parts = 0;
    pl->head_groups = (G + kMmaHeadGroup - 1) / kMmaHeadGroup;
    pl->maxg = kMmaHeadGroup;
    pl->max_bids = 0;
    pl->max_warps = per_sm * sm_count_current() * nw;
    pl->off_m = pl->off_l = 0;
    pl->off_part = round_up((int64_t)pl->max_warps * 32, 256);
    // the per-step schedule (MVB_DECODE_SCHEDULE_READY): header, tile prefix,
    // servable kv_len, one row per tile, one 144-byte record and one 32-byte
    // fixup descriptor per warp
    pl->off_shdr = round_up(pl->off_part + (int64_t)pl->max_warps * 2 * 16 * (head_dim + 2) * 4, 256);
    pl->off_spre = pl->off_shdr + 256;
    pl->off_sctx = round_up(pl->off_spre + ((int64_t)num_seqs + 1) * 4, 256);
    pl->off_srows = round_up(pl->off_sctx + (int64_t)num_seqs * 4, 256);
    pl->off_srec = round_up(pl->off_srows + (int64_t)num_seqs * khg16 * max_ctx_tiles * 4, 256);
    pl->off_sdesc = round_up(pl->off_srec + (int64_t)pl->max_warps * 144, 256);
    pl->ws_bytes = pl->off_sdesc + (int64_t)pl->max_warps * 32;
    return MVB_OK;
  }
  pl->max_warps = 0;
  pl->off_part = 0;

  int maxg;
  if (v == MVB_DECODE_MMA)
    maxg = kMmaHeadGroup;
  else
    maxg = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
  const int head_groups = (G + maxg - 1) / maxg;

  const int64_t max_ctx = (int64_t)max_blocks * block_size;
  int64_t pt;
  if (partition_tokens > 0) {
    pt = partition_tokens;
  } else if (auto_pt > 0) {
    pt = auto_pt;
  } else {
    const int64_t ctas = (int64_t)num_seqs * num_kv_heads * head_groups;
    if (max_ctx <= kUnsplitMaxTokens && ctas >= 2 * (int64_t)sm_count_current())
      pt = max_ctx;
    else
      pt = kAutoPartitionTokens;
  }
  pt = round_up(pt < 16 ? 16 : pt, 16);
  if (v == MVB_DECODE_MMA && pt > kMmaMaxPartitionTokens) pt = kMmaMaxPartitionTokens;
  if (pt > (int64_t)1 << 30) pt = (int64_t)1 << 30;
  int64_t parts = max_ctx > 0 ? (max_ctx + pt - 1) / pt : 1;
  if (parts < 1) parts = 1;
  if ((int64_t)num_seqs * parts >= ((int64_t)1 << 31)) return MVB_ERR_INVALID_ARG;

  pl->variant = v;
  pl->part_tokens = (int)pt;
  pl->num_parts = (int)parts;
  pl->head_groups = head_groups;
  pl->maxg = maxg;
  pl->max_bids = (int)((pt + block_size - 1) / block_size + 2);
  if (parts > 1) {
    const int64_t n = (int64_t)num_seqs * num_heads * parts;
    const int64_t o_bytes = round_up(n * head_dim * 4, 256);
    const int64_t ml_bytes = round_up(n * 4, 256);
    pl->off_m = o_bytes;
    pl->off_l = o_bytes + ml_bytes;
    pl->ws_bytes = o_bytes + 2 * ml_bytes;
  } else {
    pl->off_m = pl->off_l = 0;
    pl->ws_bytes = 0;
  }
  return MVB_OK;
}

// ---- TMA tensor maps over a pool tensor viewed as [rows, head_dim] ---------
struct MapEntry {
  const void* ptr;
  int64_t rows;
  int head_dim;
  int dtype;
  CUtensorMap map;
};
std::mutex g_map_mu;
MapEntry g_maps[64];
int g_map_count = 0, g_map_next = 0;

bool pool_tensor_map(const void* base, int64_t rows, int head_dim, int dtype, CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (int i = 0; i < g_map_count; ++i) {
    const MapEntry& e = g_maps[i];
    if (e.ptr == base && e.rows == rows && e.head_dim == head_dim && e.dtype == dtype) {
      *out = e.map;
      return true;
    }
  }
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
  const cuuint32_t box[2] = {64, 16};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(&map, dtype == MVB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
         2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  MapEntry& slot = g_maps[g_map_next];
  slot.ptr = base;
  slot.rows = rows;
  slot.head_dim = head_dim;
  slot.dtype = dtype;
  slot.map = map;
  g_map_next = (g_map_next + 1) % 64;
  if (g_map_count < 64) ++g_map_count;
  *out = map;
  return true;
}

bool aligned_to(const void* p, int64_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Bounded-wait test hook (mvb_test_decode_wait_timeout); thread-local so a
// test call on one thread never reaches another thread's launches.
thread_local int g_hold_warp = -1, g_hold_tile = -1, g_wait_limit = kWaitSpinLimit;

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" {

int mvb_abi_version(void) { return kAbiVersion; }

const char* mvb_status_string(int status) {
  switch (status) {
    case MVB_OK: return "ok";
    case MVB_ERR_INVALID_ARG: return "invalid argument (shape, size or stride)";
    case MVB_ERR_DTYPE: return "unsupported dtype";
    case MVB_ERR_HEAD_DIM: return "head_dim not supported (only 64, 128)";
    case MVB_ERR_BLOCK_SIZE: return "block_size must be a positive power of 2";
    case MVB_ERR_ALIGNMENT: return "pointer or stride not aligned to the vector width";
    case MVB_ERR_CUDA: return "CUDA runtime error";
    case MVB_ERR_WORKSPACE: return "split-K workspace missing or too small";
    case MVB_ERR_TENSOR_MAP: return "cuTensorMapEncodeTiled failed";
    case MVB_ERR_VARIANT: return "requested decode variant cannot run on these inputs";
    case MVB_ERR_HEADS: return "num_heads must be a multiple of num_kv_heads";
    default: return "unknown status";
  }
}

int mvb_kv_cache_write(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                       const void* value, int64_t value_stride_token, int64_t value_stride_head,
                       void* key_cache, void* value_cache, const int64_t* slot_mapping,
                       int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                       int32_t block_size, int32_t num_blocks, int32_t dtype,
                       uint32_t* slot_claims, uint32_t epoch, int32_t* error_flags, void* stream) {
  mvb::NvtxRange nvtx_range("mvb_kv_cache_write");
  if (dtype != MVB_DTYPE_F32 && dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16)
    return MVB_ERR_DTYPE;
  if (block_size <= 0) return MVB_ERR_BLOCK_SIZE;
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_blocks <= 0)
    return MVB_ERR_INVALID_ARG;
  if (num_tokens == 0) return MVB_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping || !error_flags)
    return MVB_ERR_INVALID_ARG;
  if (slot_claims != nullptr && epoch == 0) return MVB_ERR_INVALID_ARG;
  const int es = elem_size(dtype);
  if (!aligned_to(key, es) || !aligned_to(value, es) || !aligned_to(key_cache, es) ||
      !aligned_to(value_cache, es))
    return MVB_ERR_ALIGNMENT;
  const cudaError_t e = launch_kv_write(
      key, key_stride_token * es, key_stride_head * es, value, value_stride_token * es,
      value_stride_head * es, key_cache, value_cache, slot_mapping, num_tokens, num_kv_heads,
      head_dim * es, es, block_size, (int64_t)num_blocks * block_size, slot_claims, epoch,
      error_flags, static_cast<cudaStream_t>(stream), sm_count_current());
  return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
}

int mvb_paged_decode_plan(int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                          int32_t head_dim, int32_t block_size, int32_t num_blocks,
                          int32_t max_blocks_per_seq, int32_t dtype, int32_t variant,
                          int32_t partition_tokens, const void* cache_ptr, int32_t* variant_out,
                          int32_t* partition_tokens_out, int32_t* num_partitions_out,
                          int64_t* workspace_bytes_out, int32_t* launches_out) {
  Plan pl;
  variant &= ~(MVB_DECODE_AFTER_WRITE | MVB_DECODE_SCHEDULE_READY);  // launch-ordering hints: no effect on the plan
  const int st = make_plan(num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                           max_blocks_per_seq, dtype, variant, partition_tokens, cache_ptr, &pl);
  if (st != MVB_OK) return st;
  if (variant_out) *variant_out = pl.variant;
  if (partition_tokens_out) *partition_tokens_out = pl.part_tokens;
  if (num_partitions_out) *num_partitions_out = pl.num_parts;
  if (workspace_bytes_out) *workspace_bytes_out = pl.ws_bytes;
  if (launches_out) {
    // kernels one mvb_paged_decode call launches (without MVB_DECODE_SCHEDULE_READY)
    if (pl.variant == MVB_DECODE_SCHED)
      *launches_out = 2;  // schedule + decode
    else if (pl.variant == MVB_DECODE_STREAM)
      *launches_out = 2;  // + the fixup
    else
      *launches_out = pl.num_parts > 1 ? 2 : 1;  // + the split-K reduction
  }
  return MVB_OK;
}

int mvb_paged_decode(const void* query, int64_t q_stride_seq, int64_t q_stride_head,
                     const void* key_cache, const void* value_cache, const int64_t* block_table,
                     int64_t block_table_stride, int32_t max_blocks_per_seq,
                     const int32_t* kv_len, void* out, int64_t out_stride_seq,
                     int64_t out_stride_head, int32_t num_seqs, int32_t num_heads,
                     int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                     int32_t num_blocks, float scale, int32_t dtype, int32_t variant,
                     int32_t partition_tokens, void* workspace, int64_t workspace_bytes,
                     int32_t* error_flags, void* stream) {
  mvb::NvtxRange nvtx_range("mvb_paged_decode");
  Plan pl;
  const bool after_write = (variant & MVB_DECODE_AFTER_WRITE) != 0;
  const bool sched_ready = (variant & MVB_DECODE_SCHEDULE_READY) != 0;
  variant &= ~(MVB_DECODE_AFTER_WRITE | MVB_DECODE_SCHEDULE_READY);
  const int st = make_plan(num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                           max_blocks_per_seq, dtype, variant, partition_tokens, key_cache, &pl);
  if (st != MVB_OK) return st;
  if (num_seqs == 0) return MVB_OK;
  if (!query || !key_cache || !value_cache || !block_table || !kv_len || !out || !error_flags)
    return MVB_ERR_INVALID_ARG;
  if (max_blocks_per_seq > 0 && block_table_stride < max_blocks_per_seq) return MVB_ERR_INVALID_ARG;
  if (pl.variant != MVB_DECODE_FMA && !aligned_to(value_cache, 16)) return MVB_ERR_VARIANT;

  const int es = elem_size(dtype);
  // Query loads: 4-byte pairs in the MMA kernel, 16-byte vectors in the FMA kernel.
  const int64_t qa = pl.variant == MVB_DECODE_FMA ? 16 : 4;
  if (!aligned_to(query, qa) || (q_stride_seq * es) % qa != 0 || (q_stride_head * es) % qa != 0)
    return MVB_ERR_ALIGNMENT;
  if (pl.variant == MVB_DECODE_FMA && (!aligned_to(key_cache, 16) || !aligned_to(value_cache, 16)))
    return MVB_ERR_ALIGNMENT;
  if (!aligned_to(out, es)) return MVB_ERR_ALIGNMENT;
  if (pl.ws_bytes > 0) {
    if (workspace == nullptr || workspace_bytes < pl.ws_bytes || !aligned_to(workspace, 256))
      return MVB_ERR_WORKSPACE;
  }

  DecodeArgs a;
  a.q = query;
  a.q_s0 = q_stride_seq;
  a.q_s1 = q_stride_head;
  a.kc = key_cache;
  a.vc = value_cache;
  a.bt = block_table;
  a.bt_s0 = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.kv_len = kv_len;
  a.out = out;
  a.o_s0 = out_stride_seq;
  a.o_s1 = out_stride_head;
  a.num_seqs = num_seqs;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.G = num_heads / num_kv_heads;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.head_groups = pl.head_groups;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.part_tokens = pl.part_tokens;
  a.num_parts = pl.num_parts;
  char* ws = static_cast<char*>(workspace);
  a.part_o = pl.num_parts > 1 ? reinterpret_cast<float*>(ws) : nullptr;
  a.part_m = pl.num_parts > 1 ? reinterpret_cast<float*>(ws + pl.off_m) : nullptr;
  a.part_l = pl.num_parts > 1 ? reinterpret_cast<float*>(ws + pl.off_l) : nullptr;
  a.err = error_flags;
  a.early_inputs = after_write ? 1 : 0;  // honoured by the stream kernel
  a.hold_warp = g_hold_warp;
  a.hold_tile = g_hold_tile;
  a.wait_limit = g_wait_limit;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (pl.variant == MVB_DECODE_SCHED) {
    const int64_t rows = (int64_t)num_blocks * num_kv_heads * block_size;
    CUtensorMap tmk, tmv;
    if (!pool_tensor_map(key_cache, rows, head_dim, dtype, &tmk) ||
        !pool_tensor_map(value_cache, rows, head_dim, dtype, &tmv))
      return MVB_ERR_TENSOR_MAP;
    if (!sched_ready) {
      // build the schedule first; the decode then waits for it before reading anything
      e = launch_decode_schedule(a, head_dim, pl.sched, workspace, after_write, s);
      if (e != cudaSuccess) return MVB_ERR_CUDA;
      a.early_inputs = 0;
    }
    e = launch_decode_sched(tmk, tmv, a, dtype, head_dim, pl.sched, workspace, s);
    return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
  }
  if (pl.variant == MVB_DECODE_STREAM) {
    const int64_t rows = (int64_t)num_blocks * num_kv_heads * block_size;
    CUtensorMap tmk, tmv;
    if (!pool_tensor_map(key_cache, rows, head_dim, dtype, &tmk) ||
        !pool_tensor_map(value_cache, rows, head_dim, dtype, &tmv))
      return MVB_ERR_TENSOR_MAP;
    StreamSchedPtrs sp = stream_sched_ptrs(pl, ws);
    e = launch_decode_stream(tmk, tmv, a, dtype, head_dim, reinterpret_cast<int*>(ws),
                             reinterpret_cast<float*>(ws + pl.off_part), pl.max_warps,
                             sm_count_current(), sched_ready ? &sp : nullptr, s);
    return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
  }
  if (pl.variant == MVB_DECODE_MMA) {
    const int64_t rows = (int64_t)num_blocks * num_kv_heads * block_size;
    CUtensorMap tmk, tmv;
    if (!pool_tensor_map(key_cache, rows, head_dim, dtype, &tmk) ||
        !pool_tensor_map(value_cache, rows, head_dim, dtype, &tmv))
      return MVB_ERR_TENSOR_MAP;
    e = launch_decode_mma(tmk, tmv, a, dtype, head_dim, pl.max_bids, s);
  } else {
    e = launch_decode_fma(a, dtype, head_dim, pl.maxg, s);
  }
  if (e != cudaSuccess) return MVB_ERR_CUDA;
  if (pl.num_parts > 1) {
    e = launch_decode_reduce(a, dtype, head_dim, s);
    if (e != cudaSuccess) return MVB_ERR_CUDA;
  }
  return MVB_OK;
}

int mvb_paged_decode_schedule(const int32_t* kv_len, const int64_t* block_table, int64_t block_table_stride,
                              int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                              int32_t block_size, int32_t num_blocks, int32_t max_blocks_per_seq, int32_t dtype,
                              int32_t variant, int32_t flags, void* workspace, int64_t workspace_bytes,
                              int32_t* error_flags, void* stream) {
  mvb::NvtxRange nvtx_range("mvb_paged_decode_schedule");
  Plan pl;
  variant &= ~(MVB_DECODE_AFTER_WRITE | MVB_DECODE_SCHEDULE_READY);
  const int st = make_plan(num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                           max_blocks_per_seq, dtype, variant, 0, nullptr, &pl);
  if (st != MVB_OK) return st;
  if ((flags & ~MVB_DECODE_AFTER_WRITE) != 0) return MVB_ERR_INVALID_ARG;
  if (num_seqs == 0) return MVB_OK;
  if (pl.variant != MVB_DECODE_SCHED && pl.variant != MVB_DECODE_STREAM) return MVB_OK;  // nothing per step
  if (!kv_len || !block_table || !error_flags) return MVB_ERR_INVALID_ARG;
  if (max_blocks_per_seq > 0 && block_table_stride < max_blocks_per_seq) return MVB_ERR_INVALID_ARG;
  if (workspace == nullptr || workspace_bytes < pl.ws_bytes || !aligned_to(workspace, 256))
    return MVB_ERR_WORKSPACE;
  DecodeArgs a = {};
  a.kv_len = kv_len;
  a.bt = block_table;
  a.bt_s0 = block_table_stride;
  a.num_seqs = num_seqs;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.G = num_heads / num_kv_heads;
  a.head_groups = pl.head_groups;
  a.block_size = block_size;
  a.max_blocks = max_blocks_per_seq;
  a.num_blocks = num_blocks;
  a.err = error_flags;
  const bool wait_at_end = (flags & MVB_DECODE_AFTER_WRITE) != 0;
  cudaError_t e;
  if (pl.variant == MVB_DECODE_SCHED) {
    e = launch_decode_schedule(a, head_dim, pl.sched, workspace, wait_at_end, static_cast<cudaStream_t>(stream));
  } else {
    e = launch_decode_stream_schedule(a, dtype, head_dim, pl.max_warps, sm_count_current(),
                                      stream_sched_ptrs(pl, static_cast<char*>(workspace)), wait_at_end,
                                      static_cast<cudaStream_t>(stream));
  }
  return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
}

int mvb_paged_prefill(const void* query, int64_t q_stride_tok, int64_t q_stride_head, const void* key,
                      int64_t k_stride_tok, int64_t k_stride_head, const void* value, int64_t v_stride_tok,
                      int64_t v_stride_head, const void* key_cache, const void* value_cache,
                      const int64_t* block_table, int64_t block_table_rows, int64_t block_table_stride,
                      int32_t max_blocks_per_seq, const int64_t* seq_rows, const int64_t* cached_len,
                      const int64_t* query_len, int32_t num_chunks, int32_t total_q, void* out,
                      int64_t out_stride_tok, int64_t out_stride_head, int32_t num_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t block_size, int32_t num_blocks, float scale, int32_t dtype,
                      int32_t* error_flags, void* stream) {
  mvb::NvtxRange nvtx_range("mvb_paged_prefill");
  if (dtype != MVB_DTYPE_BF16 && dtype != MVB_DTYPE_F16) return MVB_ERR_DTYPE;
  if (head_dim != 64 && head_dim != 128) return MVB_ERR_HEAD_DIM;
  if (!is_pow2(block_size)) return MVB_ERR_BLOCK_SIZE;
  if (num_chunks < 0 || total_q < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      max_blocks_per_seq < 0 || block_table_rows < 0)
    return MVB_ERR_INVALID_ARG;
  if (num_heads % num_kv_heads != 0) return MVB_ERR_HEADS;
  if (num_chunks > mvb::kPrefillMaxSeqsHost) return MVB_ERR_INVALID_ARG;
  if (num_chunks == 0 || total_q == 0) return MVB_OK;
  if (!query || !key_cache || !value_cache || !block_table || !seq_rows || !cached_len || !query_len || !out ||
      !error_flags)
    return MVB_ERR_INVALID_ARG;
  if ((key == nullptr) != (value == nullptr)) return MVB_ERR_INVALID_ARG;
  if (max_blocks_per_seq > 0 && block_table_stride < max_blocks_per_seq) return MVB_ERR_INVALID_ARG;
  const int64_t rows = (int64_t)num_blocks * num_kv_heads * block_size;
  if (rows * head_dim >= ((int64_t)1 << 62)) return MVB_ERR_INVALID_ARG;
  const int es = elem_size(dtype);
  // 16-byte copies of pool and chunk rows, 4-byte query pairs, element output stores
  if (!aligned_to(key_cache, 16) || !aligned_to(value_cache, 16)) return MVB_ERR_ALIGNMENT;
  if (key != nullptr &&
      (!aligned_to(key, 16) || !aligned_to(value, 16) || (k_stride_tok * es) % 16 || (k_stride_head * es) % 16 ||
       (v_stride_tok * es) % 16 || (v_stride_head * es) % 16))
    return MVB_ERR_ALIGNMENT;
  if (!aligned_to(query, 4) || (q_stride_tok * es) % 4 || (q_stride_head * es) % 4) return MVB_ERR_ALIGNMENT;
  if (!aligned_to(out, es)) return MVB_ERR_ALIGNMENT;
  mvb::PrefillArgs a;
  a.q = query;
  a.q_s0 = q_stride_tok;
  a.q_s1 = q_stride_head;
  a.k = key;
  a.k_s0 = k_stride_tok;
  a.k_s1 = k_stride_head;
  a.v = value;
  a.v_s0 = v_stride_tok;
  a.v_s1 = v_stride_head;
  a.kc = key_cache;
  a.vc = value_cache;
  a.bt = block_table;
  a.bt_rows = block_table_rows;
  a.bt_s0 = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.seq_rows = seq_rows;
  a.cached = cached_len;
  a.qlen = query_len;
  a.n = num_chunks;
  a.total_q = total_q;
  a.out = out;
  a.o_s0 = out_stride_tok;
  a.o_s1 = out_stride_head;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.G = num_heads / num_kv_heads;
  a.head_groups = (a.G + mvb::kPrefillHeadsHost - 1) / mvb::kPrefillHeadsHost;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = error_flags;
  const cudaError_t e = launch_prefill(a, dtype, head_dim, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
}

}  // extern "C"

extern "C" int mvb_test_decode_wait_timeout(
    const void* query, int64_t q_stride_seq, int64_t q_stride_head, const void* key_cache,
    const void* value_cache, const int64_t* block_table, int64_t block_table_stride, int32_t max_blocks_per_seq,
    const int32_t* kv_len, void* out, int64_t out_stride_seq, int64_t out_stride_head, int32_t num_seqs,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
    float scale, int32_t dtype, void* workspace, int64_t workspace_bytes, int32_t* error_flags, void* stream,
    int32_t hold_warp, int32_t hold_tile, int32_t wait_limit, int32_t variant) {
  if (hold_warp < 0 || hold_tile < 0 || wait_limit <= 0 || wait_limit > kWaitSpinLimit) return MVB_ERR_INVALID_ARG;
  if (variant != MVB_DECODE_STREAM && variant != MVB_DECODE_SCHED) return MVB_ERR_VARIANT;
  g_hold_warp = hold_warp;
  g_hold_tile = hold_tile;
  g_wait_limit = wait_limit;
  const int st = mvb_paged_decode(query, q_stride_seq, q_stride_head, key_cache, value_cache, block_table,
                                  block_table_stride, max_blocks_per_seq, kv_len, out, out_stride_seq,
                                  out_stride_head, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                                  num_blocks, scale, dtype, variant, 0, workspace, workspace_bytes,
                                  error_flags, stream);
  g_hold_warp = -1;
  g_hold_tile = -1;
  g_wait_limit = kWaitSpinLimit;
  return st;
}
