// mvb_paged_decode_noalloc: the split-K paged decode without a caller workspace.
//
// Some callers cannot allocate device memory at decode time: a serving process
// that hands all free HBM to the KV pool at start-up and allows no allocation
// afterwards (a cudaMalloc mid-run would fail or fragment the pool), or a host
// binding (cgo, JNI, a C runtime) that has no device allocator of its own.
// This entry point keeps the flash-decoding partial states in a fixed,
// file-scope device array instead of a workspace the caller provides, and
// calls no cudaMalloc, cudaFree or allocating library routine.
//
// The array is kNoAllocScratchBytes (16 MiB).  Every GPU that loads this
// library holds one such array until the process exits.  Host code cannot use
// the array's name as a device address: the first call on a device looks the
// address up with cudaGetSymbolAddress (once per device, with that device
// current) and every launch receives that address.
#include <mutex>

#include "mvb_common.cuh"

namespace mvb {
namespace {

constexpr int64_t kNoAllocScratchBytes = (int64_t)16 << 20;

// Partial states (m, l, unnormalised O) of the split-K decode; every call
// shares it and writes each entry it later reads, so nothing needs clearing.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MVB_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return MVB_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return MVB_OK;
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_paged_decode_noalloc(
    const void* query, int64_t q_stride_seq, int64_t q_stride_head, const void* key_cache,
    const void* value_cache, const int64_t* block_table, int64_t block_table_stride,
    int32_t max_blocks_per_seq, const int32_t* kv_len, void* out, int64_t out_stride_seq,
    int64_t out_stride_head, int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t block_size, int32_t num_blocks, float scale, int32_t dtype,
    int32_t variant, int32_t partition_tokens, int32_t* error_flags, void* stream) {
  mvb::NvtxRange nvtx_range("mvb_paged_decode_noalloc");
  // The split-K family only: tensor-core kernel when eligible, else CUDA cores.
  variant &= ~MVB_DECODE_AFTER_WRITE;  // the split-K kernels read every input after the wait
  if (variant != MVB_DECODE_AUTO && variant != MVB_DECODE_FMA && variant != MVB_DECODE_MMA)
    return MVB_ERR_VARIANT;  // the stream and scheduled kernels, flags, unknown values
  int32_t v = variant, pt = 0, parts = 0;
  int64_t ws = 0;
  int st = MVB_ERR_VARIANT;
  if (variant == MVB_DECODE_AUTO || variant == MVB_DECODE_MMA)
    st = mvb_paged_decode_plan(num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                               max_blocks_per_seq, dtype, MVB_DECODE_MMA, partition_tokens, key_cache,
                               &v, &pt, &parts, &ws, nullptr);
  if (st == MVB_ERR_VARIANT && variant != MVB_DECODE_MMA)
    st = mvb_paged_decode_plan(num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                               max_blocks_per_seq, dtype, MVB_DECODE_FMA, partition_tokens, key_cache,
                               &v, &pt, &parts, &ws, nullptr);
  if (st != MVB_OK) return st;
  if (ws > mvb::kNoAllocScratchBytes) return MVB_ERR_WORKSPACE;
  void* scratch = nullptr;
  if (ws > 0) {
    st = mvb::noalloc_scratch(&scratch);
    if (st != MVB_OK) return st;
  }
  return mvb_paged_decode(query, q_stride_seq, q_stride_head, key_cache, value_cache, block_table,
                          block_table_stride, max_blocks_per_seq, kv_len, out, out_stride_seq,
                          out_stride_head, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                          num_blocks, scale, dtype, v, pt, scratch, ws, error_flags, stream);
}
