// KV-cache write: scatter new K/V rows into their physical pool slots.
//
// Semantics follow write_to_paged_cache (mini_vllm/cache/cache_write.py:25-74)
// and the Triton kernel it backs (mini_vllm/attention/paged_attention_gpu.py:32-87):
//     key_cache[slot / BS][h][slot % BS][:] = key[t][h][:]   (same for value)
// with slot == -1 skipped.  Unlike the Triton kernel this one bounds-checks the
// slot (the oracle raises IndexError there, cache_write.py:61-66) and honours
// the input's token/head strides, so V can be a strided view of a fused QKV
// output with no .contiguous() copy.
//
// Work decomposition: one thread per 16-byte chunk of one (token, head) row,
// K and V moved by the same thread, grid-stride over the flattened
// (token, head, chunk) space.  Pure HBM traffic: T*KH*D*esize read and
// written for each of K and V, plus 8 bytes of slot per token.
#include "mvb_common.cuh"

namespace mvb {

template <int VB>  // bytes moved per thread-iteration: 16 (uint4) or the element size
struct VecType;
template <> struct VecType<16> { using type = uint4; };
template <> struct VecType<4> { using type = uint32_t; };
template <> struct VecType<2> { using type = uint16_t; };

template <int VB>
__global__ void __launch_bounds__(256)
kv_write_kernel(const char* __restrict__ key, int64_t k_st, int64_t k_sh,
                const char* __restrict__ value, int64_t v_st, int64_t v_sh,
                char* __restrict__ kc, char* __restrict__ vc,
                const int64_t* __restrict__ slots, int num_tokens, int kh, int row_bytes,
                int block_size, int64_t total_slots, uint32_t* __restrict__ claims, uint32_t epoch,
                int* __restrict__ err) {
  using V = typename VecType<VB>::type;
  grid_dependency_wait();    // key/value/slots of the previous kernel are visible
  grid_launch_dependents();  // the decode that follows may be scheduled early
  const int chunks = row_bytes / VB;
  const int64_t items = (int64_t)num_tokens * kh * chunks;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(it % chunks);
    const int64_t th = it / chunks;
    const int h = (int)(th % kh);
    const int t = (int)(th / kh);
    const int64_t slot = __ldg(slots + t);
    if (slot == -1) continue;
    if (slot < -1 || slot >= total_slots) {
      if (h == 0 && c == 0) atomicOr(err, MVB_DEV_SLOT_RANGE);
      continue;
    }
    if (claims != nullptr && h == 0 && c == 0) {
      // Each call stamps its slots with a fresh epoch; finding our own epoch
      // already there means an earlier token of this call took the slot.
      if (atomicExch(claims + slot, epoch) == epoch) atomicOr(err, MVB_DEV_DUP_SLOT);
    }
    const int64_t blk = slot / block_size;
    const int64_t off = slot - blk * block_size;
    const int64_t dst = ((blk * kh + h) * block_size + off) * row_bytes + (int64_t)c * VB;
    const V kv = *reinterpret_cast<const V*>(key + t * k_st + h * k_sh + (int64_t)c * VB);
    const V vv = *reinterpret_cast<const V*>(value + t * v_st + h * v_sh + (int64_t)c * VB);
    *reinterpret_cast<V*>(kc + dst) = kv;
    *reinterpret_cast<V*>(vc + dst) = vv;
  }
}

// Host launcher (programmatic dependent launch); byte strides.  Returns a cudaError_t.
cudaError_t launch_kv_write(const void* key, int64_t k_st, int64_t k_sh, const void* value,
                            int64_t v_st, int64_t v_sh, void* kc, void* vc, const int64_t* slots,
                            int num_tokens, int kh, int row_bytes, int esize, int block_size,
                            int64_t total_slots, uint32_t* claims, uint32_t epoch, int* err,
                            cudaStream_t stream, int sm_count) {
  auto aligned16 = [](int64_t v) { return (v & 15) == 0; };
  const bool vec16 = aligned16((int64_t)(uintptr_t)key) && aligned16((int64_t)(uintptr_t)value) &&
                     aligned16((int64_t)(uintptr_t)kc) && aligned16((int64_t)(uintptr_t)vc) &&
                     aligned16(k_st) && aligned16(k_sh) && aligned16(v_st) && aligned16(v_sh) &&
                     (row_bytes % 16) == 0;
  const int vb = vec16 ? 16 : esize;
  const int64_t items = (int64_t)num_tokens * kh * (row_bytes / vb);
  int64_t blocks = (items + 255) / 256;
  const int64_t cap = (int64_t)sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const char* k = static_cast<const char*>(key);
  const char* v = static_cast<const char*>(value);
  char* kcc = static_cast<char*>(kc);
  char* vcc = static_cast<char*>(vc);
  cudaError_t e = vb == 16 ? ensure_kernel_attrs(kv_write_kernel<16>, 0)
                  : vb == 4 ? ensure_kernel_attrs(kv_write_kernel<4>, 0)
                            : ensure_kernel_attrs(kv_write_kernel<2>, 0);
  if (e != cudaSuccess) return e;
  switch (vb) {
    case 16:
      return launch_pdl(kv_write_kernel<16>, dim3((unsigned)blocks), dim3(256), 0, stream, k, k_st,
                        k_sh, v, v_st, v_sh, kcc, vcc, slots, num_tokens, kh, row_bytes, block_size,
                        total_slots, claims, epoch, err);
    case 4:
      return launch_pdl(kv_write_kernel<4>, dim3((unsigned)blocks), dim3(256), 0, stream, k, k_st,
                        k_sh, v, v_st, v_sh, kcc, vcc, slots, num_tokens, kh, row_bytes, block_size,
                        total_slots, claims, epoch, err);
    default:
      return launch_pdl(kv_write_kernel<2>, dim3((unsigned)blocks), dim3(256), 0, stream, k, k_st,
                        k_sh, v, v_st, v_sh, kcc, vcc, slots, num_tokens, kh, row_bytes, block_size,
                        total_slots, claims, epoch, err);
  }
}

}  // namespace mvb
