// Paged decode attention on CUDA cores (FP32 FMA) — the generic variant.
//
// One CTA per (sequence, KV head, head group, split-K partition).  The CTA's
// query heads (up to MAXG of the G heads that share the KV head) stay in
// registers; each KV token is read from HBM once per CTA and scored against
// all of them, so the GQA group costs one pass over K/V (the Triton kernel,
// paged_attention_gpu.py:162-249, reads K/V once per query head).
//
// Lane layout: a token row of D elements is split into LPT = D/VEC lanes, each
// holding one 16-byte vector; a warp therefore scores TPS = 32/LPT tokens at a
// time and every such lane group keeps its own online-softmax state (running
// max m, sum l, accumulator o) so no cross-group reduction is needed inside the
// loop.  Dot products are finished with LPT-wide xor shuffles.  At the end the
// NW*TPS states are merged through shared memory.
//
// This variant serves every dtype (fp32 included) and every power-of-two
// block size; the MMA variant (decode_mma.cu) is preferred for bf16/f16 with
// block_size % 16 == 0.
#include "decode_common.cuh"

namespace mvb {

template <typename T, int D, int MAXG, int NW>
__global__ void __launch_bounds__(NW * 32)
decode_fma_kernel(const DecodeArgs a) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LPT = D / VEC;
  constexpr int TPS = 32 / LPT;
  constexpr int NG = NW * TPS;
  constexpr int U = 4;  // tokens in flight per lane group per iteration
  static_assert(LPT >= 1 && LPT <= 32 && 32 % LPT == 0, "lane layout");

  extern __shared__ float fsm[];

  const int seq = blockIdx.x / a.num_parts;
  const int part = blockIdx.x - seq * a.num_parts;
  const int kvh = blockIdx.y / a.head_groups;
  const int hg = blockIdx.y - kvh * a.head_groups;
  const int h0 = kvh * a.G + hg * MAXG;
  const int nh = min(MAXG, a.G - hg * MAXG);

  const int ctx = __ldg(a.kv_len + seq);
  if (const int bad = seq_error(a, ctx)) {
    fail_sequence<T>(a, seq, part, h0, nh, D, bad);
    return;
  }
  const int t0 = part * a.part_tokens;
  if (t0 >= ctx) return;
  const int t1 = min(ctx, t0 + a.part_tokens);
  const int nparts_seq = seq_partitions(a, ctx);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp * TPS + lane / LPT;
  const int c = lane % LPT;

  float q[MAXG][VEC];
  {
    const T* qp = static_cast<const T*>(a.q) + seq * a.q_s0 + (int64_t)h0 * a.q_s1 + c * VEC;
#pragma unroll
    for (int g = 0; g < MAXG; ++g) {
      if (g < nh) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(qp + g * a.q_s1));
        unpack16<T, VEC>(raw, q[g]);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) q[g][i] = 0.f;
      }
    }
  }

  float m[MAXG], l[MAXG], acc[MAXG][VEC];
#pragma unroll
  for (int g = 0; g < MAXG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[g][i] = 0.f;
  }

  const T* kc = static_cast<const T*>(a.kc);
  const T* vc = static_cast<const T*>(a.vc);
  const int64_t* bt_row = a.bt + seq * a.bt_s0;

  for (int tb = t0; tb < t1; tb += NG * U) {
    uint4 kr[U], vr[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = tb + u * NG + grp;
      ok[u] = t < t1;
      kr[u] = make_uint4(0, 0, 0, 0);
      vr[u] = make_uint4(0, 0, 0, 0);
      if (ok[u]) {
        const int bi = t / a.block_size;
        const int64_t bid = __ldg(bt_row + bi);
        if (bid < 0 || bid >= a.num_blocks) {
          ok[u] = false;
          if (c == 0) atomicOr(a.err, MVB_DEV_BLOCK_ID);
        } else {
          const int64_t off =
              ((bid * a.num_kv_heads + kvh) * a.block_size + (t - bi * a.block_size)) * D + c * VEC;
          kr[u] = __ldg(reinterpret_cast<const uint4*>(kc + off));
          vr[u] = __ldg(reinterpret_cast<const uint4*>(vc + off));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kf[VEC], vf[VEC];
      unpack16<T, VEC>(kr[u], kf);
      unpack16<T, VEC>(vr[u], vf);
      float dot[MAXG];
#pragma unroll
      for (int g = 0; g < MAXG; ++g) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < VEC; ++i) s = fmaf(q[g][i], kf[i], s);
        dot[g] = s;
      }
#pragma unroll
      for (int o = LPT / 2; o > 0; o >>= 1) {
#pragma unroll
        for (int g = 0; g < MAXG; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], o);
      }
      if (ok[u]) {
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
          const float x = dot[g] * a.scale_log2;
          const float mn = fmaxf(m[g], x);
          const float al = fast_exp2(m[g] - mn);
          const float p = fast_exp2(x - mn);
          l[g] = fmaf(l[g], al, p);
#pragma unroll
          for (int i = 0; i < VEC; ++i) acc[g][i] = fmaf(acc[g][i], al, p * vf[i]);
          m[g] = mn;
        }
      }
    }
  }

  // ---- merge the NG lane-group states ----
  float* sm_m = fsm;
  float* sm_l = fsm + NG * MAXG;
  float* sm_o = fsm + 2 * NG * MAXG;
#pragma unroll
  for (int g = 0; g < MAXG; ++g) {
    if (c == 0) {
      sm_m[grp * MAXG + g] = m[g];
      sm_l[grp * MAXG + g] = l[g];
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) sm_o[(grp * MAXG + g) * D + c * VEC + i] = acc[g][i];
  }
  __syncthreads();
  merge_states<T, D>(a, seq, part, nparts_seq, h0, nh, NG, MAXG, sm_m, sm_l, sm_o);
}

// Dynamic shared memory of one FMA CTA.
template <typename T, int D, int MAXG, int NW>
constexpr int fma_smem_bytes() {
  constexpr int NG = NW * (32 / (D / (16 / (int)sizeof(T))));
  return (2 * NG * MAXG + NG * MAXG * D) * (int)sizeof(float);
}

template <typename T, int D, int MAXG>
cudaError_t launch_fma_t(const DecodeArgs& a, cudaStream_t stream) {
  constexpr int NW = 4;
  constexpr int smem = fma_smem_bytes<T, D, MAXG, NW>();
  static_assert(smem <= 48 * 1024, "FMA merge scratch must fit the default smem window");
  const cudaError_t e = ensure_kernel_attrs(decode_fma_kernel<T, D, MAXG, NW>, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)(a.num_seqs * a.num_parts), (unsigned)(a.num_kv_heads * a.head_groups));
  decode_fma_kernel<T, D, MAXG, NW><<<grid, NW * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_fma_d(const DecodeArgs& a, int maxg, cudaStream_t stream) {
  switch (maxg) {
    case 1: return launch_fma_t<T, D, 1>(a, stream);
    case 2: return launch_fma_t<T, D, 2>(a, stream);
    case 4: return launch_fma_t<T, D, 4>(a, stream);
    default: return launch_fma_t<T, D, 8>(a, stream);
  }
}

// Launch the FMA decode.  `maxg` is the head-group size (1, 2, 4 or 8) the
// caller used to size a.head_groups.
cudaError_t launch_decode_fma(const DecodeArgs& a, int dtype, int head_dim, int maxg,
                              cudaStream_t stream) {
  if (dtype == MVB_DTYPE_BF16)
    return head_dim == 64 ? launch_fma_d<__nv_bfloat16, 64>(a, maxg, stream)
                          : launch_fma_d<__nv_bfloat16, 128>(a, maxg, stream);
  if (dtype == MVB_DTYPE_F16)
    return head_dim == 64 ? launch_fma_d<__half, 64>(a, maxg, stream)
                          : launch_fma_d<__half, 128>(a, maxg, stream);
  return head_dim == 64 ? launch_fma_d<float, 64>(a, maxg, stream)
                        : launch_fma_d<float, 128>(a, maxg, stream);
}

// ---------------------------------------------------------------------------
// split-K cross-partition reduction (flash-decoding second stage)
// ---------------------------------------------------------------------------
// One warp per (sequence, query head).  Combines the partition states written
// by either decode kernel:  M = max_p m_p,  L = sum_p l_p 2^(m_p - M),
//   out = sum_p o_p 2^(m_p - M) / L.
// Sequences that fit one partition were finished by the decode kernel.
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_reduce_kernel(const DecodeArgs a) {
  constexpr int DPL = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pair = (int64_t)blockIdx.x * 4 + warp;
  if (pair >= (int64_t)a.num_seqs * a.num_heads) return;
  const int seq = (int)(pair / a.num_heads);
  const int h = (int)(pair - (int64_t)seq * a.num_heads);
  const int ctx = __ldg(a.kv_len + seq);
  if (seq_error(a, ctx)) return;
  const int np = seq_partitions(a, ctx);
  if (np <= 1) return;
  const int64_t base = ((int64_t)seq * a.num_heads + h) * a.num_parts;

  float M = -INFINITY;
  for (int p = lane; p < np; p += 32) M = fmaxf(M, a.part_m[base + p]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
  for (int p = lane; p < np; p += 32) L += a.part_l[base + p] * fast_exp2(a.part_m[base + p] - M);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);

  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  for (int p = 0; p < np; ++p) {
    const float w = fast_exp2(a.part_m[base + p] - M);
    const float* src = a.part_o + (base + p) * D + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = fmaf(src[i], w, acc[i]);
  }
  const float inv = 1.f / L;
  T* out = static_cast<T*>(a.out) + seq * a.o_s0 + (int64_t)h * a.o_s1 + lane * DPL;
#pragma unroll
  for (int i = 0; i < DPL; ++i) out[i] = from_f32<T>(acc[i] * inv);
}

template <typename T>
cudaError_t launch_reduce_t(const DecodeArgs& a, int head_dim, cudaStream_t stream) {
  const int64_t pairs = (int64_t)a.num_seqs * a.num_heads;
  const unsigned blocks = (unsigned)((pairs + 3) / 4);
  cudaError_t e = head_dim == 64 ? ensure_kernel_attrs(decode_reduce_kernel<T, 64>, 0)
                                 : ensure_kernel_attrs(decode_reduce_kernel<T, 128>, 0);
  if (e != cudaSuccess) return e;
  if (head_dim == 64)
    decode_reduce_kernel<T, 64><<<blocks, 128, 0, stream>>>(a);
  else
    decode_reduce_kernel<T, 128><<<blocks, 128, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_decode_reduce(const DecodeArgs& a, int dtype, int head_dim,
                                 cudaStream_t stream) {
  if (dtype == MVB_DTYPE_BF16) return launch_reduce_t<__nv_bfloat16>(a, head_dim, stream);
  if (dtype == MVB_DTYPE_F16) return launch_reduce_t<__half>(a, head_dim, stream);
  return launch_reduce_t<float>(a, head_dim, stream);
}

}  // namespace mvb
