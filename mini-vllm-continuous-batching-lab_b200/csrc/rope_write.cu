// mvb_rope_kv_cache_write: rotary position embedding of the step's query and
// key rows fused with the paged KV-cache write of the rotated keys and the
// values — one pass over the fused QKV output instead of three.
//
// Equivalent, bit for bit, to the reference's per-layer sequence
// (mini_vllm/model_runner/qwen_runner.py:163-170):
//   q = rope(q, positions); k = rope(k, positions); write_kv_cache(k, v, slots)
// with rope from mini_vllm/model/rotary.py:47-85:
//   out = x * cos[pos] + rotate_half(x) * sin[pos],
//   rotate_half(x) = cat(-x[D/2:], x[:D/2]).
// Each of the three elementwise operations rounds to the tensor dtype, as the
// torch expression does, so the kernel rounds after each: the products
// x*cos and rot*sin are exact in float32 for 16-bit inputs and then rounded,
// the sum is a float32 add of the two rounded products, rounded again; float32
// inputs use correctly rounded float32 operations with no fused multiply-add.
// cos / sin are the caller's tables ([rows, D], the RotaryEmbedding cache), so
// the result does not depend on how they were computed.
//
// One warp per token and step; its lanes cover the token's (row, vector)
// items, row over the H query heads, the KH key heads and the KH value heads,
// a vector being VEC elements of the row's lower half and the matching VEC of
// its upper half (16 bytes each when every row stride, pointer and D/2 allows
// it, else one element).
#include "mvb_common.cuh"

namespace mvb {
namespace {

struct RopeArgs {
  const void* q;
  int64_t q_s0, q_s1;
  void* q_out;
  int64_t qo_s0, qo_s1;
  const void* k;
  int64_t k_s0, k_s1;
  void* k_out;  // optional rotated keys [T, KH, D] contiguous
  const void* v;
  int64_t v_s0, v_s1;
  const int64_t* pos;
  const void* cos;
  const void* sin;
  int64_t table_rows;
  void* kc;
  void* vc;
  const int64_t* slots;
  int num_tokens, num_heads, num_kv_heads, head_dim, block_size, num_blocks;
  uint32_t* claims;
  uint32_t epoch;
  int* err;
};

template <typename T> __device__ __forceinline__ float rnd(float x);
template <> __device__ __forceinline__ float rnd<float>(float x) { return x; }
template <> __device__ __forceinline__ float rnd<__half>(float x) { return __half2float(__float2half_rn(x)); }
template <> __device__ __forceinline__ float rnd<__nv_bfloat16>(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// x * c + r * s with the torch expression's three roundings.
template <typename T>
__device__ __forceinline__ T rope_elem(T x, T c, T r_neg_or_pos, T s) {
  const float a = rnd<T>(__fmul_rn(to_f32(x), to_f32(c)));
  const float b = rnd<T>(__fmul_rn(to_f32(r_neg_or_pos), to_f32(s)));
  return from_f32<T>(__fadd_rn(a, b));
}

template <typename T, int VEC>
struct Vec {
  T e[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ Vec<T, VEC> ld(const T* p) {
  Vec<T, VEC> v;
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(v.e) = *reinterpret_cast<const uint4*>(p);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v.e[i] = p[i];
  }
  return v;
}
template <typename T, int VEC>
__device__ __forceinline__ void st(T* p, const Vec<T, VEC>& v) {
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(v.e);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = v.e[i];
  }
}

constexpr int kRopeCtasPerSm = 4;  // 256 threads x <= 64 registers

template <typename T, int VEC>
__global__ void __launch_bounds__(256, kRopeCtasPerSm) rope_kv_write_kernel(const RopeArgs a) {
  grid_dependency_wait();  // q/k/v and positions may come from the previous kernel
  grid_launch_dependents();
  const int H = a.num_heads, KH = a.num_kv_heads, D = a.head_dim, half = D / 2;
  const int nvec = half / VEC;
  const int per_token = (H + 2 * KH) * nvec;  // (row, vector) items of one token
  const int lane = threadIdx.x & 31;
  const int64_t total_slots = (int64_t)a.num_blocks * a.block_size;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  // one warp per token and step: the token's slot, position and table rows are
  // read once; lanes cover its (row, vector) items
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < a.num_tokens; t += warps) {
    const int64_t slot = __ldg(a.slots + t);
    const int64_t p = __ldg(a.pos + t);
    const bool slot_ok = slot >= 0 && slot < total_slots;
    const bool pos_ok = p >= 0 && p < a.table_rows;
    if (lane == 0) {
      int bad = 0;
      if (slot >= total_slots || slot < -1) bad |= MVB_DEV_SLOT_RANGE;
      if (!pos_ok) bad |= MVB_DEV_POSITION;
      if (slot_ok && a.claims != nullptr && atomicExch(a.claims + slot, a.epoch) == a.epoch) bad |= MVB_DEV_DUP_SLOT;
      if (bad) atomicOr(a.err, bad);
    }
    const int64_t blk_row = slot_ok ? (slot / a.block_size) * KH : 0;  // first (block, kv head) row
    const int in_blk = slot_ok ? (int)(slot % a.block_size) : 0;
    const T* cs = static_cast<const T*>(a.cos) + (pos_ok ? p : 0) * D;
    const T* sn = static_cast<const T*>(a.sin) + (pos_ok ? p : 0) * D;
    for (int it = lane; it < per_token; it += 32) {
      const int row = it / nvec;
      const int d0 = (it - row * nvec) * VEC;
      if (row >= H + KH) {  // value row: copied as is
        if (!slot_ok) continue;
        const int kvh = row - H - KH;
        const T* src = static_cast<const T*>(a.v) + (int64_t)t * a.v_s0 + (int64_t)kvh * a.v_s1;
        T* dst = static_cast<T*>(a.vc) + ((blk_row + kvh) * a.block_size + in_blk) * (int64_t)D;
        st<T, VEC>(dst + d0, ld<T, VEC>(src + d0));
        st<T, VEC>(dst + half + d0, ld<T, VEC>(src + half + d0));
        continue;
      }
      if (!pos_ok) continue;
      const T* src = row < H ? static_cast<const T*>(a.q) + (int64_t)t * a.q_s0 + (int64_t)row * a.q_s1
                             : static_cast<const T*>(a.k) + (int64_t)t * a.k_s0 + (int64_t)(row - H) * a.k_s1;
      const Vec<T, VEC> xl = ld<T, VEC>(src + d0), xh = ld<T, VEC>(src + half + d0);
      const Vec<T, VEC> cl = ld<T, VEC>(cs + d0), ch = ld<T, VEC>(cs + half + d0);
      const Vec<T, VEC> sl = ld<T, VEC>(sn + d0), sh = ld<T, VEC>(sn + half + d0);
      Vec<T, VEC> ol, oh;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        ol.e[i] = rope_elem<T>(xl.e[i], cl.e[i], from_f32<T>(-to_f32(xh.e[i])), sl.e[i]);  // rot = -x_hi
        oh.e[i] = rope_elem<T>(xh.e[i], ch.e[i], xl.e[i], sh.e[i]);                        // rot = x_lo
      }
      if (row < H) {
        T* dst = static_cast<T*>(a.q_out) + (int64_t)t * a.qo_s0 + (int64_t)row * a.qo_s1;
        st<T, VEC>(dst + d0, ol);
        st<T, VEC>(dst + half + d0, oh);
        continue;
      }
      const int kvh = row - H;
      if (a.k_out != nullptr) {
        T* dst = static_cast<T*>(a.k_out) + ((int64_t)t * KH + kvh) * D;
        st<T, VEC>(dst + d0, ol);
        st<T, VEC>(dst + half + d0, oh);
      }
      if (slot_ok) {
        T* dst = static_cast<T*>(a.kc) + ((blk_row + kvh) * a.block_size + in_blk) * (int64_t)D;
        st<T, VEC>(dst + d0, ol);
        st<T, VEC>(dst + half + d0, oh);
      }
    }
  }
}

template <typename T>
int launch_rope(const RopeArgs& a, bool vec16, cudaStream_t stream) {
  constexpr int V16 = 16 / sizeof(T);
  auto kern = vec16 ? rope_kv_write_kernel<T, V16> : rope_kv_write_kernel<T, 1>;
  if (ensure_kernel_attrs(kern, 0) != cudaSuccess) return MVB_ERR_CUDA;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = ((int64_t)a.num_tokens + 7) / 8, cap = (int64_t)sms * kRopeCtasPerSm;  // one wave
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  return launch_pdl(kern, dim3(grid), dim3(256), 0, stream, a) == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int mvb_rope_kv_cache_write(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, void* query_out,
    int64_t qo_stride_token, int64_t qo_stride_head, const void* key, int64_t k_stride_token,
    int64_t k_stride_head, const void* value, int64_t v_stride_token, int64_t v_stride_head,
    const int64_t* positions, const void* cos_table, const void* sin_table, int64_t table_rows,
    void* key_cache, void* value_cache, const int64_t* slot_mapping, void* key_out, int32_t num_tokens,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
    int32_t dtype, uint32_t* slot_claims, uint32_t epoch, int32_t* error_flags, void* stream) {
  mvb::NvtxRange nvtx_range("mvb_rope_kv_cache_write");
  if (dtype != MVB_DTYPE_F32 && dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16) return MVB_ERR_DTYPE;
  if (head_dim <= 0 || head_dim % 2 != 0) return MVB_ERR_HEAD_DIM;
  if (block_size <= 0) return MVB_ERR_BLOCK_SIZE;
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || table_rows <= 0)
    return MVB_ERR_INVALID_ARG;
  if (num_tokens == 0) return MVB_OK;
  if (!query || !query_out || !key || !value || !positions || !cos_table || !sin_table || !key_cache ||
      !value_cache || !slot_mapping || !error_flags)
    return MVB_ERR_INVALID_ARG;
  if (slot_claims != nullptr && epoch == 0) return MVB_ERR_INVALID_ARG;
  const int es = dtype == MVB_DTYPE_F32 ? 4 : 2;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  auto al_s = [es](int64_t s) { return (s * es) % 16 == 0; };
  const bool vec16 = (head_dim / 2 * es) % 16 == 0 && al(query) && al(query_out) && al(key) && al(value) &&
                     al(cos_table) && al(sin_table) && al(key_cache) && al(value_cache) &&
                     (key_out == nullptr || al(key_out)) && al_s(q_stride_token) && al_s(q_stride_head) &&
                     al_s(qo_stride_token) && al_s(qo_stride_head) && al_s(k_stride_token) &&
                     al_s(k_stride_head) && al_s(v_stride_token) && al_s(v_stride_head);
  RopeArgs a;
  a.q = query;
  a.q_s0 = q_stride_token;
  a.q_s1 = q_stride_head;
  a.q_out = query_out;
  a.qo_s0 = qo_stride_token;
  a.qo_s1 = qo_stride_head;
  a.k = key;
  a.k_s0 = k_stride_token;
  a.k_s1 = k_stride_head;
  a.k_out = key_out;
  a.v = value;
  a.v_s0 = v_stride_token;
  a.v_s1 = v_stride_head;
  a.pos = positions;
  a.cos = cos_table;
  a.sin = sin_table;
  a.table_rows = table_rows;
  a.kc = key_cache;
  a.vc = value_cache;
  a.slots = slot_mapping;
  a.num_tokens = num_tokens;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.claims = slot_claims;
  a.epoch = epoch;
  a.err = error_flags;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == MVB_DTYPE_BF16) return launch_rope<__nv_bfloat16>(a, vec16, s);
  if (dtype == MVB_DTYPE_F16) return launch_rope<__half>(a, vec16, s);
  return launch_rope<float>(a, vec16, s);
}
