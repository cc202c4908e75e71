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
// It is an HBM copy (2 x read + 2 x write of T * KH * D elements): 16-byte
// vectors, four per lane in flight, over a grid-stride loop of one wave of
// resident CTAs.  A token whose logical block lies
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

// Chunk c of the output is (token t, KV head, 16-byte chunk) with
// c = (t * KH + kvh) * CH + chunk.  A warp moves U * 32 consecutive chunks per
// step: it finds the sequence of its first token once (32-ary ballot search
// over the offsets), each lane steps forward only across sequence boundaries,
// and all U loads of K and V are in flight before the stores.  POW2: KH, CH and
// the block size are powers of two, so the index math is shifts and masks.
constexpr int kGatherUnroll = 4;

__device__ __forceinline__ int gather_find_sequence(const GatherArgs& a, int64_t t, int lane) {
  int lo = 0, hi = a.num_seqs;  // the last i with offsets[i] <= t (offsets[0] <= t assumed; checked later)
  while (hi - lo > 1) {
    const int step = (hi - lo + 31) >> 5;
    const int probe = lo + lane * step;
    const bool le = probe < hi && __ldg(a.offsets + probe) <= t;
    const unsigned m = __ballot_sync(0xffffffffu, le) | 1u;
    lo += (31 - __clz(m)) * step;
    hi = min(hi, lo + step);
  }
  return lo;
}

constexpr int kGatherCtasPerSm = 4;  // 256 threads x <= 64 registers

template <bool POW2>
__global__ void __launch_bounds__(256, kGatherCtasPerSm) paged_gather_kernel(const GatherArgs a) {
  grid_dependency_wait();  // the cache may have been written by the previous kernel
  grid_launch_dependents();
  constexpr int U = kGatherUnroll;
  const int lane = threadIdx.x & 31;
  const int per_token = a.kh * a.ch;
  const int sh_tok = POW2 ? __ffs(per_token) - 1 : 0, sh_ch = POW2 ? __ffs(a.ch) - 1 : 0;
  const int sh_bs = POW2 ? __ffs(a.block_size) - 1 : 0;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t step = (((int64_t)gridDim.x * blockDim.x) >> 5) * (U * 32);
  int bad = 0;
  // Source chunk of each of this lane's U output chunks in the step at `base`
  // (-1: a zero row).  Warp-uniform `base`: the search is warp-collective.
  auto resolve = [&](int64_t base, int64_t (&src)[U]) {
    const int64_t t0 = POW2 ? (base >> sh_tok) : base / per_token;
    const int s0 = gather_find_sequence(a, t0, lane);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      src[u] = -1;
      const int64_t c = base + u * 32 + lane;
      if (c >= a.total_chunks) continue;
      const int r = (int)(c - t0 * per_token);  // < U * 32 + per_token
      const int dt = POW2 ? (r >> sh_tok) : r / per_token;
      const int rem = r - dt * per_token;
      const int kvh = POW2 ? (rem >> sh_ch) : rem / a.ch;
      const int chunk = rem - kvh * a.ch;
      const int64_t t = t0 + dt;
      int s = s0;
      while (s + 1 < a.num_seqs && t >= __ldg(a.offsets + s + 1)) ++s;
      const int64_t o0 = __ldg(a.offsets + s);
      const int64_t row = __ldg(a.rows + s);
      if (t < o0 || t >= __ldg(a.offsets + s + 1)) {
        bad |= MVB_DEV_KV_LEN;  // offsets are not an increasing prefix starting at 0
        continue;
      }
      if (row < 0 || row >= a.bt_rows) {
        bad |= MVB_DEV_BLOCK_ID;
        continue;
      }
      const int p = (int)(t - o0);  // a position inside one sequence
      const int blk = POW2 ? (p >> sh_bs) : p / a.block_size;
      if (blk >= a.max_blocks) {
        bad |= MVB_DEV_TABLE_SHORT;
        continue;
      }
      const int64_t bid = __ldg(a.bt + row * a.bt_s0 + blk);
      if (bid < 0 || bid >= a.num_blocks) {
        bad |= MVB_DEV_BLOCK_ID;
        continue;
      }
      src[u] = ((bid * a.kh + kvh) * a.block_size + (p - blk * a.block_size)) * a.ch + chunk;
    }
  };
  // Software pipeline: the next step's addresses are resolved (its metadata
  // loads in flight) while this step's K/V loads are in flight.
  int64_t base = warp0 * (U * 32);
  int64_t cur[U];
  if (base < a.total_chunks) resolve(base, cur);
  for (; base < a.total_chunks; base += step) {
    uint4 kv[U], vv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      kv[u] = make_uint4(0, 0, 0, 0);
      vv[u] = make_uint4(0, 0, 0, 0);
      if (cur[u] >= 0) {  // read once: streaming (evict-first) loads
        kv[u] = __ldcs(a.kc + cur[u]);
        vv[u] = __ldcs(a.vc + cur[u]);
      }
    }
    const int64_t next = base + step;
    if (next < a.total_chunks) resolve(next, cur);  // cur is free once the loads are issued
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = base + u * 32 + lane;
      if (c < a.total_chunks) {  // streaming stores: the outputs are consumed by the next kernel
        __stcs(a.ko + c, kv[u]);
        __stcs(a.vo + c, vv[u]);
      }
    }
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
  mvb::NvtxRange nvtx_range("mvb_paged_gather");
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

  auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
  const bool p2 = pow2(a.kh) && pow2(a.ch) && pow2(a.block_size);
  auto kern = p2 ? paged_gather_kernel<true> : paged_gather_kernel<false>;
  cudaError_t e = ensure_kernel_attrs(kern, 0);
  if (e != cudaSuccess) return MVB_ERR_CUDA;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per_cta = 256 * kGatherUnroll;
  const int64_t want = (a.total_chunks + per_cta - 1) / per_cta;
  const int64_t cap = (int64_t)sms * kGatherCtasPerSm;  // one wave of resident CTAs
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  e = launch_pdl(kern, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), a);
  return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
}
