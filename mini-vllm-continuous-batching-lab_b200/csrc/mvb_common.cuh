// Shared device helpers for the B200 paged-attention kernels (sm_100a).
//
// Everything here is a thin wrapper around one PTX instruction: shared-memory
// address conversion, mbarrier init / arrive / bounded wait, the 2-D TMA tile
// load, ldmatrix and the m16n8k16 tensor-core MMA, plus element conversions.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <mutex>
#include <utility>

#include "mini_vllm_b200.h"

#include <nvtx3/nvToolsExt.h>  // include/ (the build passes -I include)

namespace mvb {

// Upper bound on the spins of one bounded mbarrier wait.  A try_wait returns
// after a hardware time slice, so this bounds one wait to well under a second
// on an idle pipeline and turns a lost TMA completion into MVB_DEV_TIMEOUT
// instead of a hung GPU.
constexpr int kWaitSpinLimit = 1 << 22;

// Decode arguments shared by the FMA and MMA kernels and the split-K
// reduction.  Strides are in elements.
struct DecodeArgs {
  const void* q;
  int64_t q_s0, q_s1;
  const void* kc;
  const void* vc;
  const int64_t* bt;
  int64_t bt_s0;
  int max_blocks;
  const int* kv_len;
  void* out;
  int64_t o_s0, o_s1;
  int num_seqs, num_heads, num_kv_heads, G, block_size, num_blocks;
  int head_groups;   // CTAs per KV head along grid.y (heads split into groups)
  float scale_log2;  // softmax scale * log2(e): logits live in the exp2 domain
  int part_tokens;   // tokens per split-K partition (multiple of 16)
  int num_parts;     // partitions per sequence along grid.x (1 = unsplit)
  float* part_o;     // [num_seqs][num_heads][num_parts][D] unnormalised sums
  float* part_m;     // [num_seqs][num_heads][num_parts] running max (log2 units)
  float* part_l;     // [num_seqs][num_heads][num_parts] sum of exp2(x - m)
  int* err;
  int early_inputs;  // read query / block table / kv_len before the grid-dependency wait
  // Test hook of the bounded waits: the load of local tile `hold_tile` of
  // stream warp `hold_warp` (stream kernel), or of tile number `hold_tile` of
  // consumer warp `hold_warp` (CTA * consumers + consumer; scheduled kernel), is
  // never issued, so the wait on it runs out after `wait_limit` try-waits and
  // reports MVB_DEV_TIMEOUT.
  // Production calls: hold_warp = -1, wait_limit = kWaitSpinLimit.
  int hold_warp, hold_tile;
  int wait_limit;
};

// Arguments of the paged prefill kernel (prefill_mma.cu): the chunks' queries,
// optionally their own K / V rows, the pool and the per-chunk metadata.
struct PrefillArgs {
  const void* q;
  int64_t q_s0, q_s1;
  const void* k;  // chunk rows [total_q, KH, D] (nullptr: the chunk is read from the pool)
  int64_t k_s0, k_s1;
  const void* v;
  int64_t v_s0, v_s1;
  const void* kc;  // pool [num_blocks, KH, BS, D]
  const void* vc;
  const int64_t* bt;
  int64_t bt_rows, bt_s0;
  int max_blocks;
  const int64_t* seq_rows;  // [n] block-table row of chunk i
  const int64_t* cached;    // [n] tokens already in the cache before chunk i
  const int64_t* qlen;      // [n] tokens of chunk i
  int n;
  int total_q;
  void* out;
  int64_t o_s0, o_s1;
  int num_heads, num_kv_heads, G, head_groups, block_size, num_blocks;
  float scale_log2;
  int* err;
};

// The stream kernel's per-step schedule inside its workspace (pointers; the
// layout is the plan's): header, tile prefix, servable kv_len, pool rows in
// stream order, one record and one fixup descriptor per stream warp.
struct StreamSchedPtrs {
  void* hdr;
  const int* pre;
  const int* ctx;
  const int* rows;
  const void* rec;
  const void* desc;
};

// Workspace layout of the scheduled decode (MVB_DECODE_SCHED): a 256-byte
// header, one 256-byte record per CTA, the piece descriptors, the pool rows of
// every tile, the list of sequences left out, the arrival counters of cut units
// and their partial states, each 256-byte aligned.
struct SchedLayout {
  int ctas;  // decode grid: one CTA per SM
  int mg;    // partial-state rows per piece: min(16, G)
  int nb;    // merge buffers between the consumer warps and the merger (0: no fit)
  bool ok;   // the shape fits the variant
  int64_t max_tiles, max_pieces;
  int64_t off_rec, off_desc, off_rows, off_bad, off_ucnt, off_part, bytes;
};

// ---------------------------------------------------------------------------
// element conversions
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Unpack one 16-byte vector of T into floats.
template <typename T, int VEC>
__device__ __forceinline__ void unpack16(const uint4& raw, float (&f)[VEC]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < VEC; ++i) f[i] = to_f32<T>(e[i]);
}

// 2^x with the hardware approximation; exp2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// shared memory, mbarrier and TMA
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// NVTX range over one C-ABI call (its launches and host work), visible in a
// profiler's timeline; without a profiler attached a push / pop costs a few ns.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel in the
// stream finishes; grid_dependency_wait() blocks until that kernel has
// completed and its memory is visible (it returns at once for a normal launch).
// grid_launch_dependents() lets the next such kernel be scheduled early.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on one phase of an mbarrier; false when the bound ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int limit = kWaitSpinLimit) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// L2 policy for data read exactly once (KV tiles): evict first, so the
// stream of K/V does not push small, re-read data (partial states, tables,
// outputs) out of L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 2-D TMA tile load (no multicast) completing on an mbarrier, with an L2
// cache policy.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// ldmatrix / mma.sync m16n8k16
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct Mma16816;

template <> struct Mma16816<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  // x rounded to the operand type, as a float
  static __device__ __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

template <> struct Mma16816<__half> {
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};

// One-time per-device kernel attributes: the dynamic shared memory the launch
// needs, and the maximum shared-memory carveout.  Every kernel of the library
// asks for the same (max-shared) L1/shared split, so consecutive launches —
// KV write, decode, split-K reduction or stream fixup — never make an SM drain
// to reconfigure its carveout between kernels.
// Records which (kernel, device) pairs already carry their attributes.
struct KernelAttrCache {
  const void* fn[256];
  int dev[256];
  int smem[256];
  int count;
};
inline KernelAttrCache& kernel_attr_cache() {
  static KernelAttrCache c = {};
  return c;
}
inline std::mutex& kernel_attr_mutex() {
  static std::mutex mu;
  return mu;
}

template <typename K>
cudaError_t ensure_kernel_attrs(K kern, int smem_bytes) {
  std::lock_guard<std::mutex> lock(kernel_attr_mutex());
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  KernelAttrCache& c = kernel_attr_cache();
  const void* fn = reinterpret_cast<const void*>(kern);
  int i = 0;
  while (i < c.count && !(c.fn[i] == fn && c.dev[i] == dev)) ++i;
  const bool known = i < c.count;
  if (known && c.smem[i] >= smem_bytes) return cudaSuccess;
  if (!known) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
  }
  if (smem_bytes > 48 * 1024) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
  }
  if (!known && c.count < 256) {
    c.fn[c.count] = fn;
    c.dev[c.count] = dev;
    c.smem[c.count] = smem_bytes;
    ++c.count;
  } else if (known) {
    c.smem[i] = smem_bytes;
  }
  return cudaSuccess;
}

// Launch `kern` with the programmatic stream-serialization attribute (the
// kernel must call grid_dependency_wait() before touching the previous
// kernel's outputs).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace mvb
