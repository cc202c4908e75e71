// Paged decode attention staged by TMA into shared memory and computed on the
// tensor cores (bf16 / f16, block_size a multiple of 16).
//
// One CTA per (sequence, KV head, head group of <= 16, split-K partition).
// The CTA's tokens are cut into 16-token tiles; warp w takes tiles w, w+NW, ...
// and runs its own STAGES-deep ring: lane 0 issues two 2-D TMA tile loads per
// tile (K and V, each 16 rows x D of one KV head inside one pool block, 128-byte
// swizzled) that complete on the stage's mbarrier, all 32 lanes wait on it,
// compute, and lane 0 refills the stage.  No CTA-wide barrier is taken inside
// the token loop.
//
// Math per tile (mma.sync m16n8k16, fp32 accumulate):
//   S[g][t] = Q[g][:] . K[t][:]        A = Q (16 rows = query heads of the
//                                      group, zero padded), B = K^T via ldmatrix
//   online softmax over t per head in the exp2 domain (quad shuffles)
//   O[g][:] += P[g][t] V[t][:]          A = P straight from the S accumulators
//                                      (FlashAttention-2 register reuse),
//                                      B = V via ldmatrix.trans
// Each warp keeps its own (m, l, O) state; the NW states are merged through
// shared memory at the end, then either normalised into `out` or written as a
// split-K partial for decode_reduce_kernel.
//
// Tokens past kv_len inside the last tile are masked to -inf before the max
// and their V rows are zeroed in shared memory, because the pool comes from
// torch.empty (mini_vllm/cache/pool.py:8-13) and 0 * NaN would poison the sum.
#include "decode_common.cuh"

namespace mvb {

constexpr int kTile = 16;  // tokens per pipeline stage

template <int D> struct MmaGeom {
  static constexpr int SUB = D / 64;                // 64-column (128-byte) panels per row
  static constexpr int PANEL_BYTES = kTile * 128;   // one swizzled 16 x 64 panel
  static constexpr int TILE_BYTES = SUB * PANEL_BYTES;  // one K (or V) tile
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int KC = D / 16;                 // k-steps of Q K^T
  static constexpr int NO = D / 8;                  // n-tiles of P V
};

// Byte offset of 16-byte chunk `ch` (along D) of tile row `r`, under the TMA
// 128-byte swizzle: inside each 1 KiB atom the chunk index is XOR-ed with r%8.
__device__ __forceinline__ uint32_t swz(int r, int ch) {
  return (uint32_t)((ch >> 3) * (kTile * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t ld_u32(const void* p) {
  return __ldg(reinterpret_cast<const unsigned int*>(p));
}

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
}

template <typename T, int D, int NW, int STAGES>
__global__ void __launch_bounds__(NW * 32)
decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const DecodeArgs a) {
  using Geo = MmaGeom<D>;
  using MMA = Mma16816<T>;
  static_assert(NW * 16 * D * 4 + 2 * NW * 16 * 4 <= NW * STAGES * Geo::STAGE_BYTES,
                "merge scratch aliases the stage ring");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NW * STAGES * Geo::STAGE_BYTES);
  int* bids = reinterpret_cast<int*>(bars + NW * STAGES);

  const int seq = blockIdx.x / a.num_parts;
  const int part = blockIdx.x - seq * a.num_parts;
  const int kvh = blockIdx.y / a.head_groups;
  const int hg = blockIdx.y - kvh * a.head_groups;
  const int h0 = kvh * a.G + hg * 16;
  const int nh = min(16, a.G - hg * 16);

  const int ctx = __ldg(a.kv_len + seq);
  if (const int bad = seq_error(a, ctx)) {
    fail_sequence<T>(a, seq, part, h0, nh, D, bad);
    return;
  }
  const int t0 = part * a.part_tokens;
  if (t0 >= ctx) return;
  const int t1 = min(ctx, t0 + a.part_tokens);
  const int nparts_seq = seq_partitions(a, ctx);
  const int ntiles = (t1 - t0 + kTile - 1) / kTile;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- this partition's block ids, validated once into shared memory ----
  const int bfirst = t0 / a.block_size;
  const int nb = (t1 - 1) / a.block_size - bfirst + 1;
  {
    const int64_t* bt_row = a.bt + seq * a.bt_s0 + bfirst;
    for (int i = threadIdx.x; i < nb; i += NW * 32) {
      const int64_t b = __ldg(bt_row + i);
      int v = -1;
      if (b >= 0 && b < a.num_blocks)
        v = (int)b;
      else
        atomicOr(a.err, MVB_DEV_BLOCK_ID);
      bids[i] = v;
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(bars + warp * STAGES + s), 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  __syncthreads();

  // TMA row (pool row index = (block * KH + kvh) * BS + offset) of tile i, or
  // -1 when the tile's block id was rejected.
  auto tile_row = [&](int i) -> int {
    const int tok = t0 + i * kTile;
    const int bi = tok / a.block_size;
    const int bid = bids[bi - bfirst];
    if (bid < 0) return -1;
    return (bid * a.num_kv_heads + kvh) * a.block_size + (tok - bi * a.block_size);
  };
  // Lane 0 only: start the loads of this warp's local tile j into its stage.
  auto issue = [&](int j) {
    const int s = j % STAGES;
    const uint32_t bar = smem_u32(bars + warp * STAGES + s);
    const int row = tile_row(warp + NW * j);
    if (row < 0) {
      mbar_arrive(bar);  // complete the phase with no bytes: the tile is skipped
      return;
    }
    mbar_arrive_expect_tx(bar, Geo::STAGE_BYTES);
    const uint32_t dk = smem_u32(ring + (warp * STAGES + s) * Geo::STAGE_BYTES);
    const uint32_t dv = dk + Geo::TILE_BYTES;
#pragma unroll
    for (int p = 0; p < Geo::SUB; ++p) {
      tma_load_2d(dk + p * Geo::PANEL_BYTES, &tmk, p * 64, row, bar);
      tma_load_2d(dv + p * Geo::PANEL_BYTES, &tmv, p * 64, row, bar);
    }
  };

  const int my_tiles = warp < ntiles ? (ntiles - 1 - warp) / NW + 1 : 0;
  if (lane == 0) {
    const int n0 = my_tiles < STAGES ? my_tiles : STAGES;
    for (int j = 0; j < n0; ++j) issue(j);
  }

  // ---- query fragments (A operand, rows = heads of the group) ----
  const int g0 = lane >> 2, qd = lane & 3;
  uint32_t qa[Geo::KC][4];
  {
    const T* qp = static_cast<const T*>(a.q) + seq * a.q_s0 + (int64_t)h0 * a.q_s1;
    const bool r0 = g0 < nh, r1 = g0 + 8 < nh;
#pragma unroll
    for (int kc = 0; kc < Geo::KC; ++kc) {
      const int d = kc * 16 + 2 * qd;
      qa[kc][0] = r0 ? ld_u32(qp + g0 * a.q_s1 + d) : 0u;
      qa[kc][1] = r1 ? ld_u32(qp + (g0 + 8) * a.q_s1 + d) : 0u;
      qa[kc][2] = r0 ? ld_u32(qp + g0 * a.q_s1 + d + 8) : 0u;
      qa[kc][3] = r1 ? ld_u32(qp + (g0 + 8) * a.q_s1 + d + 8) : 0u;
    }
  }

  float o[Geo::NO][4];
#pragma unroll
  for (int n = 0; n < Geo::NO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};

  int j = 0;
  bool failed = false;
  for (; j < my_tiles; ++j) {
    const int s = j % STAGES;
    const uint32_t bar = smem_u32(bars + warp * STAGES + s);
    const bool got = mbar_wait_bounded(bar, (uint32_t)((j / STAGES) & 1));
    if (__any_sync(0xffffffffu, !got)) {
      failed = true;
      break;
    }
    const int i = warp + NW * j;
    const int valid = min(kTile, t1 - (t0 + i * kTile));
    if (tile_row(i) >= 0) {
      const uint32_t kb = smem_u32(ring + (warp * STAGES + s) * Geo::STAGE_BYTES);
      const uint32_t vb = kb + Geo::TILE_BYTES;
      if (valid < kTile) {
        const int nchunk = (kTile - valid) * (D / 8);
        for (int e = lane; e < nchunk; e += 32) {
          const int r = valid + e / (D / 8), ch = e % (D / 8);
          st_shared_zero16(vb + (ch >> 3) * Geo::PANEL_BYTES + r * 128 + (ch & 7) * 16);
        }
        __syncwarp();
      }

      // S = Q K^T : s0 holds tokens 0-7, s1 tokens 8-15 of the tile.
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kc = 0; kc < Geo::KC; ++kc) {
        const int mi = lane >> 3;
        const int r = (lane & 7) + ((mi >> 1) << 3);
        const int ch = 2 * kc + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz(r, ch), b0, b1, b2, b3);
        MMA::run(s0, qa[kc], b0, b1);
        MMA::run(s1, qa[kc], b2, b3);
      }

      // Online softmax.  Thread rows: g0 (c0,c1) and g0+8 (c2,c3); its tokens:
      // 2qd, 2qd+1 (s0) and 8+2qd, 9+2qd (s1).
      float x[2][4] = {{s0[0], s0[1], s1[0], s1[1]}, {s0[2], s0[3], s1[2], s1[3]}};
      const int tk0 = 2 * qd;
      float p[2][4];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int tk = tk0 + (k & 1) + ((k >> 1) << 3);
          x[r][k] = tk < valid ? x[r][k] * a.scale_log2 : -INFINITY;
          mx = fmaxf(mx, x[r][k]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(mrow[r], mx);
        const float al = fast_exp2(mrow[r] - mn);
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          p[r][k] = fast_exp2(x[r][k] - mn);
          sum += p[r][k];
        }
        lrow[r] = fmaf(lrow[r], al, sum);
        mrow[r] = mn;
#pragma unroll
        for (int n = 0; n < Geo::NO; ++n) {
          o[n][2 * r] *= al;
          o[n][2 * r + 1] *= al;
        }
      }
      uint32_t pa[4];
      pa[0] = MMA::pack(p[0][0], p[0][1]);
      pa[1] = MMA::pack(p[1][0], p[1][1]);
      pa[2] = MMA::pack(p[0][2], p[0][3]);
      pa[3] = MMA::pack(p[1][2], p[1][3]);

      // O += P V
#pragma unroll
      for (int n = 0; n < Geo::NO; n += 2) {
        const int mi = lane >> 3;
        const int r = (lane & 7) + ((mi & 1) << 3);
        const int ch = n + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(vb + swz(r, ch), b0, b1, b2, b3);
        MMA::run(o[n], pa, b0, b1);
        MMA::run(o[n + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0 && j + STAGES < my_tiles) {
      fence_proxy_async_smem();  // our generic-proxy reads of the stage precede the TMA refill
      issue(j + STAGES);
    }
  }

  if (failed) {
    if (lane == 0) atomicOr(a.err, MVB_DEV_TIMEOUT);
    // Wait (bounded) for the loads this warp still has in flight, then drop
    // its state so the CTA finishes with a flagged, finite-shaped result.
    const int issued = min(my_tiles, j + STAGES);
    for (int jj = j; jj < issued; ++jj)
      mbar_wait_bounded(smem_u32(bars + warp * STAGES + jj % STAGES), (uint32_t)((jj / STAGES) & 1));
    mrow[0] = mrow[1] = -INFINITY;
    lrow[0] = lrow[1] = 0.f;
#pragma unroll
    for (int n = 0; n < Geo::NO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  }

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }

  // ---- merge the NW warp states (scratch aliases the drained ring) ----
  __syncthreads();
  float* sm_o = reinterpret_cast<float*>(smem);  // [NW][16][D]
  float* sm_m = sm_o + NW * 16 * D;              // [NW][16]
  float* sm_l = sm_m + NW * 16;                  // [NW][16]
#pragma unroll
  for (int n = 0; n < Geo::NO; ++n) {
    const int d = n * 8 + 2 * qd;
    sm_o[(warp * 16 + g0) * D + d] = o[n][0];
    sm_o[(warp * 16 + g0) * D + d + 1] = o[n][1];
    sm_o[(warp * 16 + g0 + 8) * D + d] = o[n][2];
    sm_o[(warp * 16 + g0 + 8) * D + d + 1] = o[n][3];
  }
  if (qd == 0) {
    sm_m[warp * 16 + g0] = mrow[0];
    sm_m[warp * 16 + g0 + 8] = mrow[1];
    sm_l[warp * 16 + g0] = lrow[0];
    sm_l[warp * 16 + g0 + 8] = lrow[1];
  }
  __syncthreads();
  merge_states<T, D>(a, seq, part, nparts_seq, h0, nh, NW, 16, sm_m, sm_l, sm_o);
}

// ---------------------------------------------------------------------------
// host launch
// ---------------------------------------------------------------------------
template <int D> struct MmaConfig;
template <> struct MmaConfig<64> {
  static constexpr int NW = 4, STAGES = 4;
};
template <> struct MmaConfig<128> {
  static constexpr int NW = 4, STAGES = 3;
};

template <int D>
constexpr int mma_smem_fixed() {
  return 1024 + MmaConfig<D>::NW * MmaConfig<D>::STAGES * (MmaGeom<D>::STAGE_BYTES + 8);
}

// Dynamic shared memory of one MMA CTA whose partition spans at most
// `max_bids` block-table entries.
int mma_smem_bytes(int head_dim, int max_bids) {
  const int fixed = head_dim == 64 ? mma_smem_fixed<64>() : mma_smem_fixed<128>();
  return fixed + 4 * max_bids;
}

template <typename T, int D>
cudaError_t launch_mma_t(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                         int max_bids, cudaStream_t stream) {
  constexpr int NW = MmaConfig<D>::NW, STAGES = MmaConfig<D>::STAGES;
  auto kern = decode_mma_kernel<T, D, NW, STAGES>;
  const int smem = mma_smem_bytes(D, max_bids);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static int granted[64] = {0};  // dynamic-smem opt-in already granted, per device
  if (dev >= 64 || granted[dev] < smem) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) granted[dev] = smem;
  }
  dim3 grid((unsigned)(a.num_seqs * a.num_parts), (unsigned)(a.num_kv_heads * a.head_groups));
  kern<<<grid, NW * 32, smem, stream>>>(tmk, tmv, a);
  return cudaGetLastError();
}

cudaError_t launch_decode_mma(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                              int dtype, int head_dim, int max_bids, cudaStream_t stream) {
  if (dtype == MVB_DTYPE_BF16)
    return head_dim == 64 ? launch_mma_t<__nv_bfloat16, 64>(tmk, tmv, a, max_bids, stream)
                          : launch_mma_t<__nv_bfloat16, 128>(tmk, tmv, a, max_bids, stream);
  return head_dim == 64 ? launch_mma_t<__half, 64>(tmk, tmv, a, max_bids, stream)
                        : launch_mma_t<__half, 128>(tmk, tmv, a, max_bids, stream);
}

}  // namespace mvb
