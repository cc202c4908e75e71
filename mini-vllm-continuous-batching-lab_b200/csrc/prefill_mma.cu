// Paged prefill attention on the tensor cores (bf16 / f16): the causal
// attention of a batch of prefill chunks over each sequence's cached prefix and
// the chunk itself, read in place from the paged pool — no gathered copy of the
// prefix, no per-sequence host loop, no host synchronisation.
//
// Each chunk's query tokens are cut into 16-token tiles.  One CTA per (query
// tile, KV head, group of <= 8 query heads of that KV head):
//   * a producer warp stages the tile's KV range — positions [0, cached +
//     last row of the tile] — 16 positions at a time into an S-stage ring with
//     cp.async (16 bytes per lane and copy, 128-byte swizzled rows as the TMA
//     loads of the decode kernels write them).  Position p < cached comes from
//     the pool (block table -> block -> row); a chunk position comes from the
//     chunk's own key / value rows when they are given, else from the pool
//     (the runner writes the chunk into the cache first); positions past the
//     tile's causal end are zero-filled.  The copies of each stage complete on
//     its mbarrier (cp.async.mbarrier.arrive.noinc, one arrival per lane);
//   * consumer warp h holds the 16 query rows of head h0 + h (A operand of
//     mma.sync m16n8k16) and runs the same online softmax as the decode
//     (attend_tile_rows: each row masked at its own causal limit
//     cached + token), then normalises and writes its 16 x D output rows.
// The CTA finds its (sequence, tile) from a prefix over the chunks' tile
// counts that it computes itself from query_len, so the host only needs the
// tensors' shapes.
//
// Every wait is bounded (kWaitSpinLimit try-waits); a wait that runs out sets
// MVB_DEV_TIMEOUT and the warp leaves after its copies in flight have landed.
#include "mma_tile.cuh"

namespace mvb {

constexpr int kPrefillHeads = 8;       // consumer warps (query heads) per CTA
constexpr int kPrefillStages = 4;
constexpr int kPrefillMaxSeqs = 4096;  // chunks per launch (the CTA's tile prefix lives in shared memory)


__device__ __forceinline__ void cp_async_16_zfill(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <typename T, int D>
__global__ void __launch_bounds__((1 + kPrefillHeads) * 32)
prefill_mma_kernel(const PrefillArgs a) {
  using Geo = MmaGeom<D>;
  constexpr int S = kPrefillStages, KC = D / 16, NO = D / 8, CH = D / 8;  // 16-byte chunks per row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                                     // [S] stages
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Geo::STAGE_BYTES);  // [S]
  uint64_t* empty = full + S;                                               // [S]
  int* tpre = reinterpret_cast<int*>(empty + S);                            // [n + 1] tile prefix
  int* qpre = tpre + a.n + 1;                                               // [n + 1] token prefix
  __shared__ int s_tot[2][(1 + kPrefillHeads)];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NT = (1 + kPrefillHeads) * 32;
  grid_dependency_wait();  // query, chunk rows and the cache may come from the previous kernel
  grid_launch_dependents();

  // ---- tiles and tokens of every chunk, exclusive prefixes ----
  {
    const int per = (a.n + NT - 1) / NT;
    const int i0 = min(a.n, tid * per), i1 = min(a.n, i0 + per);
    int mt = 0, mq = 0;
    for (int i = i0; i < i1; ++i) {
      const int ql = (int)max((int64_t)0, __ldg(a.qlen + i));
      tpre[i] = (ql + kTile - 1) / kTile;
      qpre[i] = ql;
      mt += tpre[i];
      mq += ql;
    }
    int it = mt, iq = mq;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int vt = __shfl_up_sync(0xffffffffu, it, o), vq = __shfl_up_sync(0xffffffffu, iq, o);
      if (lane >= o) {
        it += vt;
        iq += vq;
      }
    }
    if (lane == 31) {
      s_tot[0][warp] = it;
      s_tot[1][warp] = iq;
    }
    __syncthreads();
    int bt_ = 0, bq = 0, Tt = 0, Tq = 0;
    for (int w = 0; w < 1 + kPrefillHeads; ++w) {
      if (w < warp) {
        bt_ += s_tot[0][w];
        bq += s_tot[1][w];
      }
      Tt += s_tot[0][w];
      Tq += s_tot[1][w];
    }
    int rt = bt_ + it - mt, rq = bq + iq - mq;
    for (int i = i0; i < i1; ++i) {
      const int t = tpre[i], q = qpre[i];
      tpre[i] = rt;
      qpre[i] = rq;
      rt += t;
      rq += q;
    }
    if (tid == 0) {
      tpre[a.n] = Tt;
      qpre[a.n] = Tq;
    }
    __syncthreads();
  }
  if (qpre[a.n] > a.total_q) {  // the chunks hold more tokens than query has rows: refuse
    if (blockIdx.x == 0 && blockIdx.y == 0 && tid == 0) atomicOr(a.err, MVB_DEV_BLOCK_ID);
    return;
  }
  const int x = blockIdx.x;
  if (x >= tpre[a.n]) return;  // the grid covers an upper bound of the tile count
  int lo = 0, hi = a.n;        // tpre[lo] <= x < tpre[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tpre[mid] <= x)
      lo = mid;
    else
      hi = mid;
  }
  const int ci = lo;
  const int t0 = (x - tpre[ci]) * kTile;  // first query token of the tile in its chunk
  const int qoff = qpre[ci];              // the chunk's first row in query / out / key / value
  const int ql = qpre[ci + 1] - qoff;
  const int nrow = min(kTile, ql - t0);
  const int64_t srow = __ldg(a.seq_rows + ci);
  const int cached = (int)__ldg(a.cached + ci);
  const int kvh = blockIdx.y / a.head_groups, hg = blockIdx.y - kvh * a.head_groups;
  const int h0 = kvh * a.G + hg * kPrefillHeads;
  const int nh = min(kPrefillHeads, a.G - hg * kPrefillHeads);
  T* const out = static_cast<T*>(a.out);

  // the tile's causal end: its last row attends positions [0, cached + t0 + nrow)
  const int kv_end = cached + t0 + nrow;
  const bool bad = cached < 0 || srow < 0 || srow >= a.bt_rows ||
                   (int64_t)(kv_end + a.block_size - 1) / a.block_size > a.max_blocks;
  if (bad) {  // a table too short for the chunk (or a bad row): zeros, and the flag
    for (int e = tid; e < nrow * nh * D; e += NT) {
      const int r = e / (nh * D), h = (e / D) % nh, d = e % D;
      out[(int64_t)(qoff + t0 + r) * a.o_s0 + (int64_t)(h0 + h) * a.o_s1 + d] = from_f32<T>(0.f);
    }
    if (tid == 0) atomicOr(a.err, MVB_DEV_TABLE_SHORT);
    return;
  }
  const int ntiles = (kv_end + kTile - 1) / kTile;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(full + s), 32);  // the producer's lanes (cp.async arrivals)
      mbar_init(smem_u32(empty + s), nh);  // the consumer warps
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ================================ producer ================================
    const T* kc = static_cast<const T*>(a.kc);
    const T* vc = static_cast<const T*>(a.vc);
    const T* kch = static_cast<const T*>(a.k);
    const T* vch = static_cast<const T*>(a.v);
    const int64_t* bt_row = a.bt + srow * a.bt_s0;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % S;
      if (j >= S && !mbar_wait_bounded(smem_u32(empty + st), (uint32_t)((j / S - 1) & 1))) {
        atomicOr(a.err, MVB_DEV_TIMEOUT);
        break;
      }
      const uint32_t kb = smem_u32(ring + st * Geo::STAGE_BYTES), vb = kb + Geo::TILE_BYTES;
      for (int c = lane; c < kTile * CH; c += 32) {
        const int r = c / CH, ch = c - r * CH;
        const int p = j * kTile + r;
        const T* ks = kc;  // any valid address for a zero fill
        const T* vs = vc;
        int bytes = 0;
        if (p < kv_end) {
          if (kch != nullptr && p >= cached) {
            const int64_t row = qoff + (p - cached);
            ks = kch + row * a.k_s0 + (int64_t)kvh * a.k_s1 + ch * 8;
            vs = vch + row * a.v_s0 + (int64_t)kvh * a.v_s1 + ch * 8;
            bytes = 16;
          } else {
            const int bi = p / a.block_size;
            const int64_t b = __ldg(bt_row + bi);
            if (b >= 0 && b < a.num_blocks) {
              const int64_t row = (b * a.num_kv_heads + kvh) * a.block_size + (p - bi * a.block_size);
              ks = kc + row * D + ch * 8;
              vs = vc + row * D + ch * 8;
              bytes = 16;
            } else if (ch == 0) {
              atomicOr(a.err, MVB_DEV_BLOCK_ID);
            }
          }
        }
        cp_async_16_zfill(kb + swz(r, ch), ks, bytes);
        cp_async_16_zfill(vb + swz(r, ch), vs, bytes);
      }
      cp_async_mbar_arrive_noinc(smem_u32(full + st));
    }
    cp_async_wait_all();  // nothing lands after the CTA has left
    return;
  }

  // ================================ consumers =================================
  const int h = warp - 1;
  if (h >= nh) return;
  const int g0 = lane >> 2, qd = lane & 3;
  // query fragments: rows = the tile's 16 tokens of head h0 + h (zero past the chunk)
  uint32_t qa[KC][4];
  {
    const T* qp = static_cast<const T*>(a.q) + (int64_t)(qoff + t0) * a.q_s0 + (int64_t)(h0 + h) * a.q_s1;
    const bool r0 = g0 < nrow, r1 = g0 + 8 < nrow;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      const int d = kc * 16 + 2 * qd;
      qa[kc][0] = r0 ? ld_u32(qp + (int64_t)g0 * a.q_s0 + d) : 0u;
      qa[kc][1] = r1 ? ld_u32(qp + (int64_t)(g0 + 8) * a.q_s0 + d) : 0u;
      qa[kc][2] = r0 ? ld_u32(qp + (int64_t)g0 * a.q_s0 + d + 8) : 0u;
      qa[kc][3] = r1 ? ld_u32(qp + (int64_t)(g0 + 8) * a.q_s0 + d + 8) : 0u;
    }
  }
  float o[NO][4];
#pragma unroll
  for (int nn = 0; nn < NO; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  // row r (token t0 + r) attends positions < cached + t0 + r + 1
  const int lim0 = cached + t0 + g0 + 1, lim1 = cached + t0 + g0 + 9;
  for (int j = 0; j < ntiles; ++j) {
    const int st = j % S;
    if (!mbar_wait_bounded(smem_u32(full + st), (uint32_t)((j / S) & 1))) {
      if (lane == 0) atomicOr(a.err, MVB_DEV_TIMEOUT);
      return;
    }
    const uint32_t kb = smem_u32(ring + st * Geo::STAGE_BYTES);
    attend_tile_rows<T, D>(kb, kb + Geo::TILE_BYTES, lim0 - j * kTile, lim1 - j * kTile, a.scale_log2, qa, o,
                           mrow, lrow);
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(empty + st));
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f, inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
  T* op = out + (int64_t)(qoff + t0) * a.o_s0 + (int64_t)(h0 + h) * a.o_s1;
#pragma unroll
  for (int nn = 0; nn < NO; ++nn) {
    const int d = nn * 8 + 2 * qd;
    if (g0 < nrow) {
      T* p = op + (int64_t)g0 * a.o_s0 + d;
      p[0] = from_f32<T>(o[nn][0] * inv0);
      p[1] = from_f32<T>(o[nn][1] * inv0);
    }
    if (g0 + 8 < nrow) {
      T* p = op + (int64_t)(g0 + 8) * a.o_s0 + d;
      p[0] = from_f32<T>(o[nn][2] * inv1);
      p[1] = from_f32<T>(o[nn][3] * inv1);
    }
  }
}

int prefill_smem_bytes(int head_dim, int n) {
  const int stage = head_dim == 64 ? MmaGeom<64>::STAGE_BYTES : MmaGeom<128>::STAGE_BYTES;
  return 1024 + kPrefillStages * stage + 2 * kPrefillStages * 8 + 2 * (n + 1) * 4;
}

template <typename T, int D>
cudaError_t launch_prefill_t(const PrefillArgs& a, cudaStream_t stream) {
  auto kern = prefill_mma_kernel<T, D>;
  const int smem = prefill_smem_bytes(D, a.n);
  cudaError_t e = ensure_kernel_attrs(kern, smem);
  if (e != cudaSuccess) return e;
  const int tiles_bound = (a.total_q + kTile - 1) / kTile + a.n;
  return launch_pdl(kern, dim3(tiles_bound, a.num_kv_heads * a.head_groups), dim3((1 + kPrefillHeads) * 32), smem,
                    stream, a);
}

cudaError_t launch_prefill(const PrefillArgs& a, int dtype, int head_dim, cudaStream_t stream) {
  if (dtype == MVB_DTYPE_BF16)
    return head_dim == 64 ? launch_prefill_t<__nv_bfloat16, 64>(a, stream)
                          : launch_prefill_t<__nv_bfloat16, 128>(a, stream);
  return head_dim == 64 ? launch_prefill_t<__half, 64>(a, stream) : launch_prefill_t<__half, 128>(a, stream);
}

}  // namespace mvb
