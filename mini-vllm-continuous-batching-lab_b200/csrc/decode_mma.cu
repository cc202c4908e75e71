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
#include "mma_tile.cuh"

namespace mvb {

template <typename T, int D, int NW, int STAGES>
__global__ void __launch_bounds__(NW * 32)
decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const DecodeArgs a) {
  using Geo = MmaGeom<D>;
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
  const uint64_t kv_policy = l2_policy_evict_first();
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
      tma_load_2d(dk + p * Geo::PANEL_BYTES, &tmk, p * 64, row, bar, kv_policy);
      tma_load_2d(dv + p * Geo::PANEL_BYTES, &tmv, p * 64, row, bar, kv_policy);
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
  load_q_frags<T, D>(a, seq, h0, nh, qa);

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
      attend_tile<T, D>(kb, kb + Geo::TILE_BYTES, valid, a.scale_log2, qa, o, mrow, lrow);
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
// Warps per CTA and pipeline stages per warp (overridable at build time for tuning sweeps).
#ifndef MVB_MMA64_NW
#define MVB_MMA64_NW 4
#endif
#ifndef MVB_MMA64_STAGES
#define MVB_MMA64_STAGES 4
#endif
#ifndef MVB_MMA128_NW
#define MVB_MMA128_NW 4
#endif
#ifndef MVB_MMA128_STAGES
#define MVB_MMA128_STAGES 3
#endif
template <int D> struct MmaConfig;
template <> struct MmaConfig<64> {
  static constexpr int NW = MVB_MMA64_NW, STAGES = MVB_MMA64_STAGES;
};
template <> struct MmaConfig<128> {
  static constexpr int NW = MVB_MMA128_NW, STAGES = MVB_MMA128_STAGES;
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
  const cudaError_t e = ensure_kernel_attrs(kern, smem);
  if (e != cudaSuccess) return e;
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
