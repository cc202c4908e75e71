// Scheduled persistent paged decode (bf16 / f16, block_size a multiple of 16).
//
// Two kernels.
//
// decode_schedule_kernel (once per model step: kv_len and the block tables are
// the same for every layer of a step) cuts every unit — (sequence, KV head,
// head group of <= 16 query heads) — into pieces of at most `piece` 16-token
// tiles, split evenly (piece sizes of one unit differ by at most one tile),
// and lists the pieces ("chunks") longest first: units are bucketed by piece
// size, buckets in decreasing order, and the pieces of one unit are adjacent.
// `piece` is chosen from the step's total tile count so that there are about
// two chunks per CTA of the decode grid or more (4..32 tiles).
//
// decode_sched_kernel runs one CTA per SM over that list.  Each CTA takes its
// first chunk by index (blockIdx.x) and every further one from a global
// counter, so SMs that stream faster take more chunks and the last chunks
// handed out are the smallest: no per-warp static range, no random tail.
// Warp roles inside the CTA:
//   * fetcher (warp 0): takes the next chunk index, loads its descriptor, the
//     block ids of its tiles (validated, turned into pool rows) and the query
//     rows of its head group, and publishes them in one of 4 chunk slots.  It
//     is software-pipelined: while chunk k's block ids and query rows load,
//     chunk k+1's descriptor and the index after it are in flight;
//   * issuers (warps 1 .. NI): walk the published chunks and issue two 2-D TMA
//     tile loads (K and V, 16 rows x D, 128-byte swizzle) per tile into a
//     STAGES-deep ring (one full / one empty mbarrier per stage), in batches of
//     8 tiles, one per lane, the batches alternating between the issuer warps:
//     the bulk copies of one warp are accepted one after another (~60 ns each),
//     so a single issuing warp would cap the CTA near 8 tiles per microsecond;
//   * consumers (the next NC warps): tile j of the CTA's tile sequence goes to
//     consumer j % NC, which runs attend_tile (mma.sync m16n8k16, online
//     softmax, fp32 accumulate) and at the chunk end hands its state to the
//     merger.  Every stage thus has one consumer, which waits on its phases in
//     order (a parity wait is sound only while its waiter is at most one phase
//     away; consumers sharing stages drifted further apart than the ring).  A
//     chunk's tiles start on a multiple of NC of the sequence — the places
//     skipped are virtual tiles that pass through the ring without a load — so
//     tile i of a chunk always goes to consumer i % NC and the result does not
//     depend on timing;
//   * mergers (the last NM warps; chunk k is merger k % NM's): merge the NC
//     consumer states of the chunk.  A chunk
//     that holds a whole unit is normalised and written to `out`; a piece of a
//     longer unit writes its partial state (O, m, l per head row) and counts
//     itself in on the unit's arrival counter, and the last piece to arrive
//     merges all pieces in piece order (deterministic) and writes the unit.
// The consumers never wait for global memory, so the ring keeps streaming
// while the merger works.
//
// Every wait is bounded (DecodeArgs::wait_limit); a wait that runs out sets
// MVB_DEV_TIMEOUT and a CTA-wide abort flag that every other wait polls, the
// issuer then waits (bounded) for its loads in flight, and every role leaves.
// The work counters are then left dirty: the schedule must be rebuilt (the
// schedule kernel resets every counter it hands to the decode).
#include "mma_tile.cuh"

namespace mvb {

constexpr int kSchedMaxPiece = 32;  // tiles per chunk at most: one block id per fetcher lane
constexpr int kSchedMinPiece = 4;
constexpr int kSchedSlots = 4;      // chunk slots between the fetcher and the other roles
constexpr int kSchedIssueLanes = 8;  // tiles the issuer warp issues at once, one per lane
constexpr int kSchedBuildThreads = 1024;

// Workspace header (256 bytes at the start of the workspace).
struct SchedHeader {
  int n_chunks;
  int piece;        // tiles per chunk at most, as chosen
  int next;         // chunk hand-out counter (zero at rest)
  int done;         // CTAs whose fetcher saw the end of the list (zero at rest)
  int total_tiles;  // tiles of all units
  int pad[59];
};
static_assert(sizeof(SchedHeader) == 256, "header is 256 bytes");

// Chunk descriptor: two int4
//   {sequence, unit of the sequence (kvh * head_groups + hg), first tile, tiles}
//   {first chunk of the unit, pieces of the unit, kv_len, bad sequence flag}
// A bad sequence (kv_len < 1 or a block table too short) has one chunk of zero
// tiles per unit: its output rows are written as zeros.
struct SchedArgs {
  SchedHeader* hdr;
  const int4* desc;  // [max_chunks][2]
  int* ucnt;         // [max_chunks] arrival counters, indexed by a unit's first chunk
  float* part;       // [max_chunks][mg][D + 4] partial O (D), m, l
  int max_chunks;
  int mg;            // partial rows per chunk: min(16, G)
};

// ---------------------------------------------------------------------------
// schedule
// ---------------------------------------------------------------------------
__device__ __forceinline__ int sched_seq_error(int ctx, int block_size, int max_blocks) {
  if (ctx < 1) return MVB_DEV_KV_LEN;
  const int64_t need = ((int64_t)ctx + block_size - 1) / block_size;
  if (need > max_blocks) return MVB_DEV_TABLE_SHORT;
  return 0;
}

// One CTA.  wait_at_end: the previous kernel in the stream may still be running
// and writes none of this kernel's inputs (the KV write); the kernel computes
// first and waits for it only before exiting, so that a dependent of this
// kernel that waits for it also waits for that previous kernel.
__global__ void __launch_bounds__(kSchedBuildThreads)
decode_schedule_kernel(const int* __restrict__ kv_len, int num_seqs, int units_per_seq, int block_size,
                       int max_blocks, int ctas, SchedHeader* hdr, int4* desc, int* ucnt, int max_chunks,
                       int* err, int wait_at_end) {
  __shared__ int s_hist[kSchedMaxPiece + 1];
  __shared__ int s_base[kSchedMaxPiece + 1];
  __shared__ long long s_red[kSchedBuildThreads / 32];
  __shared__ int s_piece, s_overflow;
  if (!wait_at_end) grid_dependency_wait();
  grid_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid <= kSchedMaxPiece) s_hist[tid] = 0;

  // total tiles of all units
  long long tiles = 0;
  for (int s = tid; s < num_seqs; s += blockDim.x) {
    const int ctx = __ldg(kv_len + s);
    if (!sched_seq_error(ctx, block_size, max_blocks)) tiles += (ctx + kTile - 1) / kTile;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tiles += __shfl_xor_sync(0xffffffffu, tiles, o);
  if (lane == 0) s_red[warp] = tiles;
  __syncthreads();
  if (tid == 0) {
    long long t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_red[w];
    t *= units_per_seq;
    long long pc = (t + 2LL * ctas - 1) / (2LL * ctas);
    if (pc < kSchedMinPiece) pc = kSchedMinPiece;
    if (pc > kSchedMaxPiece) pc = kSchedMaxPiece;
    s_piece = (int)pc;
    hdr->piece = (int)pc;
    hdr->total_tiles = (int)(t < 0x7fffffffLL ? t : 0x7fffffffLL);
  }
  __syncthreads();
  const int piece = s_piece;

  // histogram of chunks by piece size (bucket 0: bad sequences)
  for (int s = tid; s < num_seqs; s += blockDim.x) {
    const int ctx = __ldg(kv_len + s);
    const bool bad = sched_seq_error(ctx, block_size, max_blocks) != 0;
    const int nt = bad ? 0 : (ctx + kTile - 1) / kTile;
    const int p = bad ? 1 : (nt + piece - 1) / piece;
    const int ps = bad ? 0 : (nt + p - 1) / p;
    atomicAdd(&s_hist[ps], p * units_per_seq);
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int b = kSchedMaxPiece; b >= 0; --b) {
      s_base[b] = run;
      run += s_hist[b];
    }
    s_overflow = run > max_chunks;
    if (s_overflow) {  // cannot happen with the host's bound; refuse rather than overrun
      atomicOr(err, MVB_DEV_SCHEDULE);
      run = 0;
    }
    hdr->n_chunks = run;
    hdr->next = 0;
    hdr->done = 0;
  }
  __syncthreads();
  const bool overflow = s_overflow != 0;

  // descriptors; within a bucket the order is arbitrary (it only affects which
  // CTA takes a chunk, never the arithmetic of any output)
  for (int s = tid; s < num_seqs; s += blockDim.x) {
    const int ctx = __ldg(kv_len + s);
    const int bad = sched_seq_error(ctx, block_size, max_blocks);
    if (bad) atomicOr(err, bad);
    if (overflow) continue;
    const int nt = bad ? 0 : (ctx + kTile - 1) / kTile;
    const int p = bad ? 1 : (nt + piece - 1) / piece;
    const int ps = bad ? 0 : (nt + p - 1) / p;
    const int c0 = atomicAdd(&s_base[ps], p * units_per_seq);
    for (int k = 0; k < units_per_seq; ++k) {
      const int first = c0 + k * p;
      ucnt[first] = 0;
      for (int i = 0; i < p; ++i) {
        const int b0 = (int)((int64_t)i * nt / p), b1 = (int)((int64_t)(i + 1) * nt / p);
        desc[2 * (first + i)] = make_int4(s, k, b0, b1 - b0);
        desc[2 * (first + i) + 1] = make_int4(first, p, ctx, bad ? 1 : 0);
      }
    }
  }
  if (wait_at_end) grid_dependency_wait();
}

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
// Per head dim: ring stages, consumer warps, merge buffers between the
// consumers and the mergers, issuer warps (the bulk copies one warp issues are
// accepted one after another, ~60 ns each, so a single warp caps a CTA near 8
// tiles per microsecond) and merger warps (under full streaming load each L2
// round trip of a merge — partial stores and fence, the arrival atomic, the
// other pieces' partials — takes 1-2 us, so one merger warp falls behind the
// ~7 split pieces a CTA streams at config 2).  The ring holds 128 KB in flight
// per SM; shared memory (ring + slots + NB buffers of NC states) sets NB.
// (Overridable at build time for tuning sweeps.)
#ifndef MVB_SCHED64_STAGES
#define MVB_SCHED64_STAGES 32
#endif
#ifndef MVB_SCHED64_NC
#define MVB_SCHED64_NC 8
#endif
#ifndef MVB_SCHED64_NB
#define MVB_SCHED64_NB 2
#endif
#ifndef MVB_SCHED64_NM
#define MVB_SCHED64_NM 2
#endif
#ifndef MVB_SCHED64_NI
#define MVB_SCHED64_NI 2
#endif
#ifndef MVB_SCHED128_STAGES
#define MVB_SCHED128_STAGES 16
#endif
#ifndef MVB_SCHED128_NC
#define MVB_SCHED128_NC 4
#endif
#ifndef MVB_SCHED128_NB
#define MVB_SCHED128_NB 2
#endif
#ifndef MVB_SCHED128_NM
#define MVB_SCHED128_NM 2
#endif
#ifndef MVB_SCHED128_NI
#define MVB_SCHED128_NI 2
#endif
template <int D> struct SchedConfig;
template <> struct SchedConfig<64> {
  static constexpr int STAGES = MVB_SCHED64_STAGES, NC = MVB_SCHED64_NC, NB = MVB_SCHED64_NB, NI = MVB_SCHED64_NI,
                       NM = MVB_SCHED64_NM;
};
template <> struct SchedConfig<128> {
  static constexpr int STAGES = MVB_SCHED128_STAGES, NC = MVB_SCHED128_NC, NB = MVB_SCHED128_NB,
                       NI = MVB_SCHED128_NI, NM = MVB_SCHED128_NM;
};

template <int D> struct SchedSmem {
  using Geo = MmaGeom<D>;
  static constexpr int STAGES = SchedConfig<D>::STAGES, NC = SchedConfig<D>::NC, NB = SchedConfig<D>::NB;
  static constexpr int NI = SchedConfig<D>::NI, NM = SchedConfig<D>::NM;
  static_assert(STAGES % NC == 0, "each stage belongs to one consumer");
  static_assert(STAGES % (NI * kSchedIssueLanes) == 0, "each stage belongs to one issuer");
  static_assert(NB % NM == 0, "each merge buffer belongs to one merger");
  static constexpr int THREADS = (1 + NI + NC + NM) * 32;  // fetcher, issuers, consumers, mergers
  static constexpr int QP = D + 8;  // query row pitch (elements): conflict-free fragment loads
  static constexpr int SLOT_BYTES = 32 + 4 * kSchedMaxPiece + 16 * QP * 2;
  // merge buffer: header (2 x int4), (m, l) [consumers][16], O [consumers][16][D]
  static constexpr int MB_ML = 32;
  static constexpr int MB_O = MB_ML + NC * 16 * 8;
  static constexpr int MB_BYTES = MB_O + NC * 16 * D * 4;
  static constexpr int RING = 0;
  static constexpr int SLOTS = RING + STAGES * Geo::STAGE_BYTES;
  static constexpr int MERGE = SLOTS + kSchedSlots * SLOT_BYTES;
  static constexpr int BARS = MERGE + NB * MB_BYTES;
  static constexpr int NBARS = 2 * STAGES + 2 * kSchedSlots + 2 * NB;
  static constexpr int STAGE_BAD = BARS + NBARS * 8;
  static constexpr int MISC = STAGE_BAD + STAGES * 4;
  static constexpr int BYTES = MISC + 16;
  static_assert(SLOTS % 16 == 0 && MERGE % 16 == 0 && MB_BYTES % 16 == 0 && BARS % 8 == 0, "alignment");
};

// Bounded wait that also gives up when another role has aborted the CTA.
__device__ __forceinline__ bool sched_wait(uint32_t bar, uint32_t parity, int limit, volatile int* abort_flag,
                                           int* err) {
  for (int i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31) == 31 && *abort_flag) return false;
  }
  *abort_flag = 1;
  atomicOr(err, MVB_DEV_TIMEOUT);
  return false;
}

// The same for all 32 lanes of a warp (true only when every lane got the phase).
__device__ __forceinline__ bool sched_wait_warp(uint32_t bar, uint32_t parity, int limit,
                                                volatile int* abort_flag, int* err) {
  const bool ok = sched_wait(bar, parity, limit, abort_flag, err);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// One arrival for a whole warp: __syncwarp orders every lane's shared-memory
// accesses before lane 0's arrive (release), as one arrival per lane would,
// at a thirty-second of the barrier traffic.
__device__ __forceinline__ void warp_arrive(uint32_t bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

template <typename T, int D>
__global__ void __launch_bounds__(SchedSmem<D>::THREADS, 1)
decode_sched_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                    const DecodeArgs a, const SchedArgs sa) {
  using Geo = MmaGeom<D>;
  using L = SchedSmem<D>;
  constexpr int KC = D / 16, NO = D / 8, QP = L::QP, PR = D + 4, NB = L::NB, NC = L::NC, STAGES = L::STAGES;
  constexpr int NI = L::NI, NM = L::NM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem + L::RING;
  uint8_t* slots = smem + L::SLOTS;
  uint8_t* merge = smem + L::MERGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  uint64_t* full = bars;                   // [STAGES] tile landed
  uint64_t* empty = bars + STAGES;         // [STAGES] tile consumed
  uint64_t* cfull = bars + 2 * STAGES;     // [slots] chunk published
  uint64_t* cempty = cfull + kSchedSlots;  // [slots] chunk read by the issuer and the consumers
  uint64_t* mfull = cempty + kSchedSlots;  // [NB] consumer states written
  uint64_t* mempty = mfull + NB;           // [NB] states read by the merger
  volatile int* stage_bad = reinterpret_cast<volatile int*>(smem + L::STAGE_BAD);
  volatile int* misc = reinterpret_cast<volatile int*>(smem + L::MISC);  // [0] abort flag

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), 1);  // the consuming warp
    }
    for (int c = 0; c < kSchedSlots; ++c) {
      mbar_init(smem_u32(cfull + c), 1);        // the fetcher warp
      mbar_init(smem_u32(cempty + c), NI + NC);  // the issuer and consumer warps
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(smem_u32(mfull + b), NC);  // the consumer warps
      mbar_init(smem_u32(mempty + b), 1);  // the merger warp
    }
    misc[0] = 0;
    fence_mbar_init();
  }
  __syncthreads();  // the only CTA-wide barrier
  grid_launch_dependents();
  volatile int* abort_flag = misc;
  const int limit = a.wait_limit;

  auto slot_desc = [&](int slot) { return reinterpret_cast<int4*>(slots + slot * L::SLOT_BYTES); };
  auto slot_rows = [&](int slot) { return reinterpret_cast<int*>(slots + slot * L::SLOT_BYTES + 32); };
  auto slot_q = [&](int slot) {
    return reinterpret_cast<T*>(slots + slot * L::SLOT_BYTES + 32 + 4 * kSchedMaxPiece);
  };
  auto mb_hdr = [&](int b) { return reinterpret_cast<int4*>(merge + b * L::MB_BYTES); };
  auto mb_ml = [&](int b) { return reinterpret_cast<float2*>(merge + b * L::MB_BYTES + L::MB_ML); };
  auto mb_o = [&](int b) { return reinterpret_cast<float*>(merge + b * L::MB_BYTES + L::MB_O); };

  if (warp == 0) {
    // ================================= fetcher =================================
    if (!a.early_inputs) grid_dependency_wait();
    bool waited = a.early_inputs == 0;
    const int4 stop = make_int4(0, 0, 0, -1);
    int idx = blockIdx.x;  // the first chunk by index; its descriptor is read before the chunk
                           // count (blockIdx.x < gridDim.x <= max_chunks: in bounds either way)
    int4 d0 = __ldcg(sa.desc + 2 * idx), d1 = __ldcg(sa.desc + 2 * idx + 1);
    const int n_chunks = __ldcg(&sa.hdr->n_chunks);
    bool have = idx < n_chunks;
    if (!have) {
      d0 = stop;
      d1 = make_int4(0, 0, 0, 0);
    }
    int idx_n = -1;  // the next chunk (from the second iteration on)
    bool aborted = false;
    for (int k = 0;; ++k) {
      const int slot = k % kSchedSlots;
      const int seq = d0.x, uk = d0.y, begin = d0.z, n = d0.w;
      const int kvh = uk / a.head_groups, hg = uk - kvh * a.head_groups;
      const int h0 = kvh * a.G + hg * 16, nh = min(16, a.G - hg * 16);
      // block id -> pool row of tile `lane` of the chunk
      int row = -1;
      if (lane < n) {
        const int tok = (begin + lane) * kTile;
        const int bi = tok / a.block_size;
        const int64_t b = __ldg(a.bt + (int64_t)seq * a.bt_s0 + bi);
        if (b >= 0 && b < a.num_blocks)
          row = ((int)b * a.num_kv_heads + kvh) * a.block_size + (tok - bi * a.block_size);
        else
          atomicOr(a.err, MVB_DEV_BLOCK_ID);
      }
      // query rows of the head group, 16 x D, zero past nh (4-byte words)
      constexpr int QW = 16 * D / 2 / 32;  // words per lane
      uint32_t qw[QW];
      const T* qbase = static_cast<const T*>(a.q) + (int64_t)seq * a.q_s0 + (int64_t)h0 * a.q_s1;
#pragma unroll
      for (int v = 0; v < QW; ++v) {
        const int e = lane + 32 * v, r = e / (D / 2), c = e - r * (D / 2);
        qw[v] = (n > 0 && r < nh) ? ld_u32(qbase + (int64_t)r * a.q_s1 + 2 * c) : 0u;
      }
      if (!waited) {  // the hand-out counter is reset by the previous decode
        grid_dependency_wait();
        waited = true;
      }
      // In flight during the publication below: on the first chunk the index of
      // the second; afterwards the next descriptor and the index after it.
      bool have_n = false;
      int4 n0 = stop, n1 = make_int4(0, 0, 0, 0);
      int t_nn = n_chunks;
      if (k == 0) {
        if (have && lane == 0) t_nn = (int)gridDim.x + atomicAdd(&sa.hdr->next, 1);
      } else {
        have_n = idx_n < n_chunks;
        if (have_n) {
          n0 = __ldcg(sa.desc + 2 * idx_n);
          n1 = __ldcg(sa.desc + 2 * idx_n + 1);
          if (lane == 0) t_nn = (int)gridDim.x + atomicAdd(&sa.hdr->next, 1);
        }
      }
      if (k >= kSchedSlots &&
          !sched_wait_warp(smem_u32(cempty + slot), (uint32_t)((k / kSchedSlots - 1) & 1), limit, abort_flag,
                           a.err)) {
        aborted = true;
        break;
      }
      if (lane == 0) {
        slot_desc(slot)[0] = d0;
        slot_desc(slot)[1] = make_int4(d1.x, d1.y, d1.z, idx);  // .w: the chunk's own index
      }
      slot_rows(slot)[lane] = row;
      uint32_t* qs = reinterpret_cast<uint32_t*>(slot_q(slot));
#pragma unroll
      for (int v = 0; v < QW; ++v) {
        const int e = lane + 32 * v, r = e / (D / 2), c = e - r * (D / 2);
        qs[r * (QP / 2) + c] = qw[v];
      }
      warp_arrive(smem_u32(cfull + slot), lane);
      if (!have) break;  // the end marker is published
      if (k == 0) {  // the second chunk's descriptor, and the third's index: the pipeline from here on
        idx = __shfl_sync(0xffffffffu, t_nn, 0);
        have = idx < n_chunks;
        d0 = have ? __ldcg(sa.desc + 2 * idx) : stop;
        d1 = have ? __ldcg(sa.desc + 2 * idx + 1) : make_int4(0, 0, 0, 0);
        int t = n_chunks;
        if (have && lane == 0) t = (int)gridDim.x + atomicAdd(&sa.hdr->next, 1);
        idx_n = __shfl_sync(0xffffffffu, t, 0);
      } else {
        idx = idx_n;
        have = have_n;
        d0 = n0;
        d1 = n1;
        idx_n = __shfl_sync(0xffffffffu, t_nn, 0);
      }
    }
    if (!aborted && lane == 0) {
      // the last CTA to reach the end of the list resets the counters
      const int prev = atomicAdd(&sa.hdr->done, 1);
      if (prev == (int)gridDim.x - 1) {
        atomicExch(&sa.hdr->next, 0);
        atomicExch(&sa.hdr->done, 0);
      }
    }
    return;
  }

  if (warp <= NI) {
    // ================================= issuers =================================
    // The tile sequence in batches of kSchedIssueLanes: batch j / kSchedIssueLanes
    // is issuer warp (j / kSchedIssueLanes) % NI's, one tile per lane.  Each lane
    // waits for its stage's previous tile to be consumed, then arms the stage's
    // barrier and issues the K and V loads.
    const int w = warp - 1;
    grid_dependency_wait();  // the cache is complete from here on
    if (w == 0 && lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
    }
    const uint64_t pol = l2_policy_evict_first();
    int j_base = 0, j_last = -1;  // the CTA's tile sequence; the end of this issuer's last batch
    for (int k = 0;; ++k) {
      const int slot = k % kSchedSlots;
      if (!sched_wait_warp(smem_u32(cfull + slot), (uint32_t)((k / kSchedSlots) & 1), limit, abort_flag, a.err))
        break;
      const int n = slot_desc(slot)[0].w;
      if (n < 0) break;
      const int* rows = slot_rows(slot);
      const int j_start = (j_base + NC - 1) / NC * NC, j_end = j_start + n;  // before j_start: virtual tiles
      bool ok = true;
      for (int j0 = j_base / kSchedIssueLanes * kSchedIssueLanes; j0 < j_end; j0 += kSchedIssueLanes) {
        if ((j0 / kSchedIssueLanes) % NI != w) continue;
        const int j = j0 + lane, st = j % STAGES;
        const bool mine = lane < kSchedIssueLanes && j >= j_base && j < j_end;
        bool got = true;
        if (mine && j >= STAGES)
          got = sched_wait(smem_u32(empty + st), (uint32_t)((j / STAGES - 1) & 1), limit, abort_flag, a.err);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        if (mine && !((int)blockIdx.x == a.hold_warp && j == a.hold_tile)) {  // test hook: never completes
          const int row = j < j_start ? -1 : rows[j - j_start];
          stage_bad[st] = row < 0;
          const uint32_t fb = smem_u32(full + st);
          if (row < 0) {
            mbar_arrive(fb);
          } else {
            mbar_arrive_expect_tx(fb, Geo::STAGE_BYTES);
            const uint32_t dk = smem_u32(ring + st * Geo::STAGE_BYTES);
#pragma unroll
            for (int p = 0; p < Geo::SUB; ++p) {
              tma_load_2d(dk + p * Geo::PANEL_BYTES, &tmk, p * 64, row, fb, pol);
              tma_load_2d(dk + Geo::TILE_BYTES + p * Geo::PANEL_BYTES, &tmv, p * 64, row, fb, pol);
            }
          }
        }
        j_last = min(j0 + kSchedIssueLanes, j_end) - 1;
      }
      if (!ok) break;
      j_base = j_end;
      warp_arrive(smem_u32(cempty + slot), lane);
    }
    // Wait (bounded, without the abort shortcut) for this issuer's loads still in
    // flight, the latest use of each of its stages, so no copy lands after the
    // CTA has left.
    for (int i = lane; i < STAGES; i += 32) {
      const int jj = j_last - i;
      if (jj < 0 || (jj / kSchedIssueLanes) % NI != w || ((int)blockIdx.x == a.hold_warp && jj == a.hold_tile))
        continue;
      mbar_wait_bounded(smem_u32(full + jj % STAGES), (uint32_t)((jj / STAGES) & 1), limit);
    }
    return;
  }

  if (warp < 1 + NI + NC) {
    // ================================ consumers ================================
    const int c = warp - 1 - NI;
    const int g0 = lane >> 2, qd = lane & 3;
    int j_base = 0;
    for (int k = 0;; ++k) {
      const int slot = k % kSchedSlots;
      if (!sched_wait_warp(smem_u32(cfull + slot), (uint32_t)((k / kSchedSlots) & 1), limit, abort_flag, a.err))
        return;
      const int4 d0 = slot_desc(slot)[0], d1 = slot_desc(slot)[1];
      const int n = d0.w;
      const int begin = d0.z, ctx = d1.z;
      uint32_t qa[KC][4];
      if (n > 0) {
        const uint32_t* qs = reinterpret_cast<const uint32_t*>(slot_q(slot));
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
          const int w = kc * 8 + qd;  // word column of element kc * 16 + 2 qd
          qa[kc][0] = qs[g0 * (QP / 2) + w];
          qa[kc][1] = qs[(g0 + 8) * (QP / 2) + w];
          qa[kc][2] = qs[g0 * (QP / 2) + w + 4];
          qa[kc][3] = qs[(g0 + 8) * (QP / 2) + w + 4];
        }
      }
      if (n >= 0) warp_arrive(smem_u32(cempty + slot), lane);  // descriptor and query are in registers

      float o[NO][4];
#pragma unroll
      for (int nn = 0; nn < NO; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
      float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
      // tile j of the sequence is this consumer's when j % NC == c; the chunk's
      // tiles start at j_start (a multiple of NC; before it, virtual tiles)
      const int j_start = (j_base + NC - 1) / NC * NC;
      const int j_end = n >= 0 ? j_start + n : j_base;  // the end marker has no tiles, virtual or real
      for (int jj = j_base + (c - j_base % NC + NC) % NC; jj < j_end; jj += NC) {
        const int st = jj % STAGES;
        if (!sched_wait_warp(smem_u32(full + st), (uint32_t)((jj / STAGES) & 1), limit, abort_flag, a.err))
          return;
        if (!stage_bad[st]) {
          const int i = jj - j_start;
          const int valid = min(kTile, ctx - (begin + i) * kTile);
          const uint32_t kb = smem_u32(ring + st * Geo::STAGE_BYTES);
          attend_tile<T, D>(kb, kb + Geo::TILE_BYTES, valid, a.scale_log2, qa, o, mrow, lrow);
          if (valid < kTile) fence_proxy_async_smem();  // V rows zeroed through the generic proxy
        }
        warp_arrive(smem_u32(empty + st), lane);
      }
      j_base = j_end;

      // ---- hand this consumer's state to the chunk's merger; at the end, the
      // end marker to every merger (chunks k .. k + NM - 1) ----
      for (int e = 0; e < (n < 0 ? NM : 1); ++e) {
        const int kk = k + e, b = kk % NB;
        if (kk >= NB &&
            !sched_wait_warp(smem_u32(mempty + b), (uint32_t)((kk / NB - 1) & 1), limit, abort_flag, a.err))
          return;
        if (n >= 0) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
            lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
          }
          const int nh = min(16, a.G - (d0.y % a.head_groups) * 16);
          float* mo = mb_o(b) + c * 16 * D;
#pragma unroll
          for (int nn = 0; nn < NO; ++nn) {
            const int d = nn * 8 + 2 * qd;
            if (g0 < nh) *reinterpret_cast<float2*>(mo + g0 * D + d) = make_float2(o[nn][0], o[nn][1]);
            if (g0 + 8 < nh) *reinterpret_cast<float2*>(mo + (g0 + 8) * D + d) = make_float2(o[nn][2], o[nn][3]);
          }
          if (qd == 0) {
            float2* mml = mb_ml(b) + c * 16;
            if (g0 < nh) mml[g0] = make_float2(mrow[0], lrow[0]);
            if (g0 + 8 < nh) mml[g0 + 8] = make_float2(mrow[1], lrow[1]);
          }
        }
        if (c == 0 && lane == 0) {
          mb_hdr(b)[0] = d0;
          mb_hdr(b)[1] = d1;
        }
        warp_arrive(smem_u32(mfull + b), lane);
      }
      if (n < 0) return;
    }
  }

  // ================================== mergers =================================
  // Merger m takes chunks k with k % NM == m, through its own buffers
  // b = k % NB (b % NM == m).  Lane l takes head row r = l / 4 (+ 8 on a second
  // pass for more than 8 heads) and column quarter l % 4 (CQ = D / 4 columns).
  {
    constexpr int CQ = D / 4;
    const int m = warp - (1 + NI + NC);
    const int rq = lane >> 2, cq = (lane & 3) * CQ;
    T* const outp = static_cast<T*>(a.out);
    for (int k = m;; k += NM) {
      const int b = k % NB;
      if (!sched_wait_warp(smem_u32(mfull + b), (uint32_t)((k / NB) & 1), limit, abort_flag, a.err)) return;
      const int4 d0 = mb_hdr(b)[0], d1 = mb_hdr(b)[1];
      if (d0.w < 0) return;  // end marker
      const int seq = d0.x, uk = d0.y;
      const int first = d1.x, p = d1.y, me = d1.w;
      const int kvh = uk / a.head_groups, hg = uk - kvh * a.head_groups;
      const int h0 = kvh * a.G + hg * 16, nh = min(16, a.G - hg * 16);
      // the NC consumer states of each row -> (M, L, O) of the chunk
      float Mr[2], Lr[2], Or[2][CQ];
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int r = rq + 8 * pass;
        Mr[pass] = -INFINITY;
        Lr[pass] = 0.f;
#pragma unroll
        for (int i = 0; i < CQ; ++i) Or[pass][i] = 0.f;
        if (r >= nh) continue;
        float2 ml[NC];
#pragma unroll
        for (int s = 0; s < NC; ++s) {
          ml[s] = mb_ml(b)[s * 16 + r];
          Mr[pass] = fmaxf(Mr[pass], ml[s].x);
        }
        if (Mr[pass] == -INFINITY) continue;  // no token (a bad sequence): zeros
#pragma unroll
        for (int s = 0; s < NC; ++s) {
          const float w = fast_exp2(ml[s].x - Mr[pass]);
          Lr[pass] = fmaf(ml[s].y, w, Lr[pass]);
          const float4* src = reinterpret_cast<const float4*>(mb_o(b) + (s * 16 + r) * D + cq);
#pragma unroll
          for (int i = 0; i < CQ / 4; ++i) {
            const float4 v = src[i];
            Or[pass][4 * i] = fmaf(v.x, w, Or[pass][4 * i]);
            Or[pass][4 * i + 1] = fmaf(v.y, w, Or[pass][4 * i + 1]);
            Or[pass][4 * i + 2] = fmaf(v.z, w, Or[pass][4 * i + 2]);
            Or[pass][4 * i + 3] = fmaf(v.w, w, Or[pass][4 * i + 3]);
          }
        }
      }
      warp_arrive(smem_u32(mempty + b), lane);  // the states are in registers: the buffer is free

      if (p == 1) {
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          const int r = rq + 8 * pass;
          if (r >= nh) continue;
          const float inv = Lr[pass] > 0.f ? 1.f / Lr[pass] : 0.f;
          T* po = outp + (int64_t)seq * a.o_s0 + (int64_t)(h0 + r) * a.o_s1 + cq;
#pragma unroll
          for (int i = 0; i < CQ; ++i) po[i] = from_f32<T>(Or[pass][i] * inv);
        }
        continue;
      }
      // a piece of a split unit: store the partial, count in; the last piece merges
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int r = rq + 8 * pass;
        if (r >= nh) continue;
        float* pp = sa.part + ((int64_t)me * sa.mg + r) * PR;
        float4* dst = reinterpret_cast<float4*>(pp + cq);
#pragma unroll
        for (int i = 0; i < CQ / 4; ++i)
          dst[i] = make_float4(Or[pass][4 * i], Or[pass][4 * i + 1], Or[pass][4 * i + 2], Or[pass][4 * i + 3]);
        if ((lane & 3) == 0) *reinterpret_cast<float2*>(pp + D) = make_float2(Mr[pass], Lr[pass]);
      }
      fence_acq_rel_gpu();  // this lane's partial is visible GPU-wide before the arrival
      __syncwarp();
      int arrived = 0;
      if (lane == 0) arrived = atomicAdd(sa.ucnt + first, 1);
      arrived = __shfl_sync(0xffffffffu, arrived, 0);
      if (arrived != p - 1) continue;
      fence_acq_rel_gpu();  // acquire side: the other pieces' partials
      // online merge of the pieces in piece order (deterministic), 4 at a time
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int r = rq + 8 * pass;
        if (r >= nh) continue;  // lane-divergent: no warp collectives below
        float M = -INFINITY, Lsum = 0.f, acc[CQ];
#pragma unroll
        for (int i = 0; i < CQ; ++i) acc[i] = 0.f;
        for (int i0 = 0; i0 < p; i0 += 4) {
          float2 ml[4];
          float4 ov[4][CQ / 4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int i = i0 + t < p ? i0 + t : p - 1;
            const float* pp = sa.part + ((int64_t)(first + i) * sa.mg + r) * PR;
            ml[t] = __ldcg(reinterpret_cast<const float2*>(pp + D));
#pragma unroll
            for (int v = 0; v < CQ / 4; ++v) ov[t][v] = __ldcg(reinterpret_cast<const float4*>(pp + cq) + v);
          }
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            if (i0 + t >= p) break;
            const float mn = fmaxf(M, ml[t].x);
            const float sa_ = fast_exp2(M - mn), sb = fast_exp2(ml[t].x - mn);
            Lsum = Lsum * sa_ + ml[t].y * sb;
#pragma unroll
            for (int v = 0; v < CQ / 4; ++v) {
              acc[4 * v] = acc[4 * v] * sa_ + ov[t][v].x * sb;
              acc[4 * v + 1] = acc[4 * v + 1] * sa_ + ov[t][v].y * sb;
              acc[4 * v + 2] = acc[4 * v + 2] * sa_ + ov[t][v].z * sb;
              acc[4 * v + 3] = acc[4 * v + 3] * sa_ + ov[t][v].w * sb;
            }
            M = mn;
          }
        }
        const float inv = 1.f / Lsum;
        T* po = outp + (int64_t)seq * a.o_s0 + (int64_t)(h0 + r) * a.o_s1 + cq;
#pragma unroll
        for (int i = 0; i < CQ; ++i) po[i] = from_f32<T>(acc[i] * inv);
      }
      __syncwarp();
      if (lane == 0) sa.ucnt[first] = 0;  // zero at rest for the next decode of this schedule
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

SchedLayout sched_layout(int num_seqs, int num_kv_heads, int head_groups, int G, int max_blocks,
                         int block_size, int head_dim, int ctas) {
  SchedLayout l = {};
  const int64_t units = (int64_t)num_seqs * num_kv_heads * head_groups;
  const int64_t max_tiles = ((int64_t)max_blocks * block_size + kTile - 1) / kTile;
  const int64_t per_unit = (max_tiles + kSchedMaxPiece - 1) / kSchedMaxPiece;
  // sum over units of ceil(tiles / piece) <= total / piece + units, and the
  // schedule's choice of piece keeps total / piece <= max(units * per_unit, 2 * ctas)
  int64_t mc = units * per_unit;
  if (mc < 2LL * ctas) mc = 2LL * ctas;
  mc += units;
  if (mc < 1) mc = 1;
  l.max_chunks = mc;
  l.mg = G < 16 ? G : 16;
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  l.off_desc = 256;
  l.off_ucnt = l.off_desc + up(mc * 32);
  l.off_part = l.off_ucnt + up(mc * 4);
  l.bytes = l.off_part + up(mc * l.mg * (head_dim + 4) * 4);
  return l;
}

int sched_smem_bytes(int head_dim) {
  return 1024 + (head_dim == 64 ? SchedSmem<64>::BYTES : SchedSmem<128>::BYTES);
}

cudaError_t launch_decode_schedule(const DecodeArgs& a, const SchedLayout& l, void* ws, int ctas, bool wait_at_end,
                                   cudaStream_t stream) {
  char* w = static_cast<char*>(ws);
  auto kern = decode_schedule_kernel;
  cudaError_t e = ensure_kernel_attrs(kern, 0);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(1), dim3(kSchedBuildThreads), 0, stream, a.kv_len, a.num_seqs,
                    a.num_kv_heads * a.head_groups, a.block_size, a.max_blocks, ctas,
                    reinterpret_cast<SchedHeader*>(w), reinterpret_cast<int4*>(w + l.off_desc),
                    reinterpret_cast<int*>(w + l.off_ucnt), (int)l.max_chunks, a.err, wait_at_end ? 1 : 0);
}

template <typename T, int D>
cudaError_t launch_sched_t(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                           const SchedLayout& l, void* ws, int ctas, cudaStream_t stream) {
  auto kern = decode_sched_kernel<T, D>;
  const int smem = 1024 + SchedSmem<D>::BYTES;
  cudaError_t e = ensure_kernel_attrs(kern, smem);
  if (e != cudaSuccess) return e;
  char* w = static_cast<char*>(ws);
  SchedArgs sa;
  sa.hdr = reinterpret_cast<SchedHeader*>(w);
  sa.desc = reinterpret_cast<const int4*>(w + l.off_desc);
  sa.ucnt = reinterpret_cast<int*>(w + l.off_ucnt);
  sa.part = reinterpret_cast<float*>(w + l.off_part);
  sa.max_chunks = (int)l.max_chunks;
  sa.mg = l.mg;
  return launch_pdl(kern, dim3(ctas), dim3(SchedSmem<D>::THREADS), smem, stream, tmk, tmv, a, sa);
}

cudaError_t launch_decode_sched(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a, int dtype,
                                int head_dim, const SchedLayout& l, void* ws, int ctas, cudaStream_t stream) {
  if (dtype == MVB_DTYPE_BF16)
    return head_dim == 64 ? launch_sched_t<__nv_bfloat16, 64>(tmk, tmv, a, l, ws, ctas, stream)
                          : launch_sched_t<__nv_bfloat16, 128>(tmk, tmv, a, l, ws, ctas, stream);
  return head_dim == 64 ? launch_sched_t<__half, 64>(tmk, tmv, a, l, ws, ctas, stream)
                        : launch_sched_t<__half, 128>(tmk, tmv, a, l, ws, ctas, stream);
}

}  // namespace mvb
