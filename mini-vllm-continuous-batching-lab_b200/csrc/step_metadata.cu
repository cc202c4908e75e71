// mvb_build_step_metadata: the per-step attention metadata on the device.
//
// Replaces the per-token host loops of ModelInputBuilder.build
// (mini_vllm/engine/input_builder.py:48-196) for the tensors the attention path
// consumes: for a step of S sequences (prefill chunks first, then decodes) with
// block lists B_s, cached_len_before c_s and query lengths q_s,
//   positions[t]    = c_s + i                      (token i of sequence s)
//   slot_mapping[t] = B_s[p / BS] * BS + p % BS    (input_builder.py:202-221)
//   tables[s][j]    = B_s[j] for j < |B_s|, else -1 (input_builder.py:238-256)
//   kv_len_after[s] = c_s + q_s
// B_s is read at blocks[block_starts[s] .. + block_counts[s]): the step's lists
// concatenated, or the rows of a padded [S, W] table (starts s * W) that an
// engine keeps as arrays.  The kernel fills every output in one launch (one
// thread per table entry, token and sequence).  A position whose logical block is not in B_s
// (the reference raises "Block not allocated") sets MVB_DEV_TABLE_SHORT and
// gets slot -1.
#include "mvb_common.cuh"

namespace mvb {
namespace {

struct StepArgs {
  const int64_t* blocks;      // block ids
  const int64_t* blk_start;   // [S] first entry of B_s in blocks
  const int64_t* blk_count;   // [S] |B_s|
  const int64_t* cached;      // [S]
  const int64_t* tok_off;     // [S + 1] exclusive prefix of q_s
  int num_seqs;
  int64_t num_tokens;
  int max_blocks;
  int block_size;
  int64_t* positions;
  int64_t* slots;
  int64_t* tables;
  int32_t* kv_len;
  int* err;
};

__global__ void __launch_bounds__(256) step_metadata_kernel(const StepArgs a) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t n_table = (int64_t)a.num_seqs * a.max_blocks;
  const int64_t total = n_table + a.num_tokens + a.num_seqs;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n_table) {  // padded block table entry
      const int s = (int)(i / a.max_blocks), j = (int)(i - (int64_t)s * a.max_blocks);
      const int64_t b0 = __ldg(a.blk_start + s), n = __ldg(a.blk_count + s);
      a.tables[i] = j < n ? __ldg(a.blocks + b0 + j) : -1;
    } else if (i < n_table + a.num_tokens) {  // token: position and slot
      const int64_t t = i - n_table;
      int lo = 0, hi = a.num_seqs;  // the last s with tok_off[s] <= t
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(a.tok_off + mid) <= t)
          lo = mid;
        else
          hi = mid;
      }
      const int64_t p = __ldg(a.cached + lo) + (t - __ldg(a.tok_off + lo));
      const int64_t b0 = __ldg(a.blk_start + lo), n = __ldg(a.blk_count + lo);
      const int64_t lb = p / a.block_size;
      a.positions[t] = p;
      if (p < 0 || lb >= n) {
        atomicOr(a.err, MVB_DEV_TABLE_SHORT);
        a.slots[t] = -1;
      } else {
        a.slots[t] = __ldg(a.blocks + b0 + lb) * a.block_size + (p - lb * a.block_size);
      }
    } else {  // sequence: kv_len_after
      const int s = (int)(i - n_table - a.num_tokens);
      a.kv_len[s] = (int32_t)(__ldg(a.cached + s) + __ldg(a.tok_off + s + 1) - __ldg(a.tok_off + s));
    }
  }
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int mvb_build_step_metadata(const int64_t* blocks, const int64_t* block_starts,
                                       const int64_t* block_counts, const int64_t* cached_len,
                                       const int64_t* token_offsets,
                                       int32_t num_seqs, int64_t num_tokens, int32_t max_blocks,
                                       int32_t block_size, int64_t* positions, int64_t* slot_mapping,
                                       int64_t* block_tables, int32_t* kv_len_after, int32_t* error_flags,
                                       void* stream) {
  mvb::NvtxRange nvtx_range("mvb_build_step_metadata");
  if (block_size <= 0) return MVB_ERR_BLOCK_SIZE;
  if (num_seqs < 0 || num_tokens < 0 || max_blocks < 0) return MVB_ERR_INVALID_ARG;
  if (num_seqs == 0) return MVB_OK;
  if (!block_starts || !block_counts || !cached_len || !token_offsets || !kv_len_after || !error_flags ||
      (max_blocks > 0 && (!block_tables || !blocks)) || (num_tokens > 0 && (!positions || !slot_mapping)))
    return MVB_ERR_INVALID_ARG;
  StepArgs a;
  a.blocks = blocks;
  a.blk_start = block_starts;
  a.blk_count = block_counts;
  a.cached = cached_len;
  a.tok_off = token_offsets;
  a.num_seqs = num_seqs;
  a.num_tokens = num_tokens;
  a.max_blocks = max_blocks;
  a.block_size = block_size;
  a.positions = positions;
  a.slots = slot_mapping;
  a.tables = block_tables;
  a.kv_len = kv_len_after;
  a.err = error_flags;
  if (ensure_kernel_attrs(step_metadata_kernel, 0) != cudaSuccess) return MVB_ERR_CUDA;
  const int64_t total = (int64_t)num_seqs * max_blocks + num_tokens + num_seqs;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + 255) / 256, cap = (int64_t)sms * 8;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  return launch_pdl(step_metadata_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), a) ==
                 cudaSuccess
             ? MVB_OK
             : MVB_ERR_CUDA;
}
