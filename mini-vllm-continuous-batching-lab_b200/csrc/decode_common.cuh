// Pieces shared by the two paged-decode kernels (FMA and MMA) and the split-K
// cross-partition reduction.
#pragma once

#include "mvb_common.cuh"

namespace mvb {

// Number of split-K partitions sequence `ctx` occupies.
__device__ __forceinline__ int seq_partitions(const DecodeArgs& a, int ctx) {
  return (ctx + a.part_tokens - 1) / a.part_tokens;
}

// A sequence whose kv_len cannot be served: kv_len < 1 (the reference raises
// ValueError, paged_attention_gpu.py:296-300) or more blocks than the table
// row holds (gather_paged_kv raises IndexError, cache_read.py:62-67).
// Returns the error bit, or 0 when the sequence is servable.
__device__ __forceinline__ int seq_error(const DecodeArgs& a, int ctx) {
  if (ctx < 1) return MVB_DEV_KV_LEN;
  const int64_t need = ((int64_t)ctx + a.block_size - 1) / a.block_size;
  if (need > a.max_blocks) return MVB_DEV_TABLE_SHORT;
  return 0;
}

// Called by every CTA of a bad sequence: partition 0 writes zeros for its
// heads (so the output is deterministic) and one thread raises the flag.
template <typename T>
__device__ void fail_sequence(const DecodeArgs& a, int seq, int part, int h0, int nh, int D,
                              int bit) {
  if (part != 0) return;
  if (threadIdx.x == 0) atomicOr(a.err, bit);
  T* out = static_cast<T*>(a.out);
  for (int e = threadIdx.x; e < nh * D; e += blockDim.x) {
    const int g = e / D, d = e - g * D;
    out[seq * a.o_s0 + (int64_t)(h0 + g) * a.o_s1 + d] = from_f32<T>(0.f);
  }
}

// Final store of one output element of a CTA: either the normalised result
// (the sequence fits one partition) or the partition's unnormalised partial.
template <typename T>
__device__ __forceinline__ void store_result(const DecodeArgs& a, int seq, int part, int nparts_seq,
                                             int h, int d, int D, float M, float L, float O) {
  if (nparts_seq == 1) {
    T* out = static_cast<T*>(a.out);
    out[seq * a.o_s0 + (int64_t)h * a.o_s1 + d] = from_f32<T>(O / L);
  } else {
    const int64_t pi = ((int64_t)seq * a.num_heads + h) * a.num_parts + part;
    a.part_o[pi * D + d] = O;
    if (d == 0) {
      a.part_m[pi] = M;
      a.part_l[pi] = L;
    }
  }
}

// Combine `nstate` online-softmax states held in shared memory into the CTA
// result.  State r for head g is (m[r*MG+g], l[r*MG+g], o[(r*MG+g)*D + :]);
// states that saw no token carry m = -inf, l = 0, o = 0 and drop out.
template <typename T, int D>
__device__ void merge_states(const DecodeArgs& a, int seq, int part, int nparts_seq, int h0,
                             int nh, int nstate, int MG, const float* sm_m, const float* sm_l,
                             const float* sm_o) {
  for (int e = threadIdx.x; e < nh * D; e += blockDim.x) {
    const int g = e / D, d = e - g * D;
    float M = -INFINITY;
    for (int r = 0; r < nstate; ++r) M = fmaxf(M, sm_m[r * MG + g]);
    float L = 0.f, O = 0.f;
    for (int r = 0; r < nstate; ++r) {
      const float w = fast_exp2(sm_m[r * MG + g] - M);
      L += sm_l[r * MG + g] * w;
      O += sm_o[(r * MG + g) * D + d] * w;
    }
    store_result<T>(a, seq, part, nparts_seq, h0 + g, d, D, M, L, O);
  }
}

}  // namespace mvb
