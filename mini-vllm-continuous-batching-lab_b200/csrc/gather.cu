// mvb_paged_gather: logical -> physical gather of cached K/V into contiguous
// [total_tokens, KH, D] tensors (the prefill path's prefix read).
//
// Replaces the reference's Triton _gather_prefix_kv_kernel and its wrapper
// gather_prefix_kv (mini_vllm/attention/paged_attention_gpu.py:329-433), whose
// index maps were built by a Python loop over every prefix token, and restates
// gather_paged_kv (mini_vllm/cache/cache_read.py:19-84) for a batch of
// sequences: out[off_i + p] = cache[block_table[row_i][p / BS], :, p % BS, :]
// for p < n_i, where n_i = out_offsets[i + 1] - out_offsets[i].
//
// It is an HBM copy (2 x read + 2 x write of T * KH * D elements), so the
// kernel moves 16-byte vectors, one per thread and step of a grid-stride loop
// sized to a few waves of resident threads.  A token whose logical block lies
// past the table (IndexError in gather_paged_kv) or whose block id is outside
// [0, num_blocks) (-1 padding, where the Triton kernel left the output
// unwritten) gets zero rows and an error bit.
#include "mvb_common.cuh"

namespace mvb {
namespace {

struct GatherArgs {
  const uint4* kc;
  const uint4* vc;
  const int64_t* bt;
  int64_t bt_s0;
  int64_t bt_rows;
  int max_blocks;
  const int64_t* rows;     // [num_seqs] block-table row of each sequence
  const int64_t* offsets;  // [num_seqs + 1] exclusive prefix of the token counts
  uint4* ko;
  uint4* vo;
  int num_seqs;
  int64_t total_chunks;    // total_tokens * KH * CH
  int kh;
  int ch;                  // 16-byte chunks per (token, KV head) row
  int block_size;
  int num_blocks;
  int* err;
};

__global__ void __launch_bounds__(256) paged_gather_kernel(const GatherArgs a) {
  grid_dependency_wait();  // the cache may have been written by the previous kernel
  grid_launch_dependents();
  const int64_t per_token = (int64_t)a.kh * a.ch;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int bad = 0;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < a.total_chunks; c += stride) {
    const int64_t t = c / per_token;
    const int r = (int)(c - t * per_token);
    const int kvh = r / a.ch, chunk = r - kvh * a.ch;
    // sequence of output token t: the last i with offsets[i] <= t
    int lo = 0, hi = a.num_seqs;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(a.offsets + mid) <= t)
        lo = mid;
      else
        hi = mid;
    }
    const int64_t o0 = __ldg(a.offsets + lo);
    const int64_t p = t - o0;
    const int64_t blk = p / a.block_size;
    const int64_t row = __ldg(a.rows + lo);
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (p < 0 || t >= __ldg(a.offsets + lo + 1)) {
      bad |= MVB_DEV_KV_LEN;  // offsets are not an increasing prefix starting at 0
    } else if (row < 0 || row >= a.bt_rows) {
      bad |= MVB_DEV_BLOCK_ID;
    } else if (blk >= a.max_blocks) {
      bad |= MVB_DEV_TABLE_SHORT;
    } else {
      const int64_t bid = __ldg(a.bt + row * a.bt_s0 + blk);
      if (bid < 0 || bid >= a.num_blocks) {
        bad |= MVB_DEV_BLOCK_ID;
      } else {
        const int64_t src = ((bid * a.kh + kvh) * a.block_size + (p - blk * a.block_size)) * a.ch + chunk;
        kv = __ldg(a.kc + src);
        vv = __ldg(a.vc + src);
      }
    }
    a.ko[c] = kv;
    a.vo[c] = vv;
  }
  if (bad) atomicOr(a.err, bad);
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int mvb_paged_gather(const void* key_cache, const void* value_cache, const int64_t* block_table,
                                int64_t block_table_rows, int64_t block_table_stride, int32_t max_blocks_per_seq,
                                const int64_t* seq_rows,
                                const int64_t* out_offsets, void* key_out, void* value_out, int32_t num_seqs,
                                int64_t total_tokens, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                int32_t num_blocks, int32_t dtype, int32_t* error_flags, void* stream) {
  if (dtype != MVB_DTYPE_F32 && dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16) return MVB_ERR_DTYPE;
  if (head_dim <= 0) return MVB_ERR_HEAD_DIM;
  if (block_size <= 0) return MVB_ERR_BLOCK_SIZE;
  if (num_seqs < 0 || total_tokens < 0 || num_kv_heads <= 0 || num_blocks <= 0 || max_blocks_per_seq < 0 ||
      block_table_rows < 0)
    return MVB_ERR_INVALID_ARG;
  if (total_tokens == 0 || num_seqs == 0) return MVB_OK;
  if (!key_cache || !value_cache || !block_table || !seq_rows || !out_offsets || !key_out || !value_out ||
      !error_flags)
    return MVB_ERR_INVALID_ARG;
  if (max_blocks_per_seq > 0 && block_table_stride < max_blocks_per_seq) return MVB_ERR_INVALID_ARG;
  const int64_t row_bytes = (int64_t)head_dim * (dtype == MVB_DTYPE_F32 ? 4 : 2);
  if (row_bytes % 16 != 0) return MVB_ERR_HEAD_DIM;  // rows move as 16-byte vectors
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!aligned(key_cache) || !aligned(value_cache) || !aligned(key_out) || !aligned(value_out))
    return MVB_ERR_ALIGNMENT;

  GatherArgs a;
  a.kc = static_cast<const uint4*>(key_cache);
  a.vc = static_cast<const uint4*>(value_cache);
  a.bt = block_table;
  a.bt_s0 = block_table_stride;
  a.bt_rows = block_table_rows;
  a.max_blocks = max_blocks_per_seq;
  a.rows = seq_rows;
  a.offsets = out_offsets;
  a.ko = static_cast<uint4*>(key_out);
  a.vo = static_cast<uint4*>(value_out);
  a.num_seqs = num_seqs;
  a.kh = num_kv_heads;
  a.ch = (int)(row_bytes / 16);
  a.total_chunks = total_tokens * num_kv_heads * a.ch;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.err = error_flags;

  cudaError_t e = ensure_kernel_attrs(paged_gather_kernel, 0);
  if (e != cudaSuccess) return MVB_ERR_CUDA;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (a.total_chunks + 255) / 256;
  const int64_t cap = (int64_t)sms * 8;  // 8 resident 256-thread CTAs per SM, one wave
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  e = launch_pdl(paged_gather_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), a);
  return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
}
