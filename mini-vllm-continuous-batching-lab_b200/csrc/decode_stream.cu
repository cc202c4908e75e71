// Persistent stream-K paged decode (bf16 / f16, block_size a multiple of 16).
//
// The decode's work is a stream of 16-token KV tiles: for every sequence s in
// order, for every (KV head, head group) unit of s, ceil(kv_len[s] / 16) tiles.
// The grid is sized to the number of CTAs the GPU holds at once, and the stream
// is cut into one contiguous range per WARP: equal ranges, or, with the
// per-step schedule, the cost-aware split (a range costs its tiles plus one
// tile per unit it enters), so the warps finish together and no second wave
// or ragged tail exists (one CTA per (sequence, KV head) leaves 1.15 waves on
// config 2).
//
// Each warp runs the TMA ring of decode_mma.cu over its range: lane 0 loads
// K and V tiles STAGES ahead (2-D tensor-map loads, 128-byte swizzle, one
// mbarrier per stage), all lanes run attend_tile (mma.sync m16n8k16, online
// softmax).  When the range crosses a unit boundary the warp flushes the unit:
//   * a unit that lies wholly inside the warp's range is normalised and
//     written to `out` directly;
//   * a unit cut by a range boundary is written as a partial state
//     (m, l, O per head row) to the warp's first or last slot.
// decode_stream_fixup_kernel then merges the partials of every cut unit (two
// warps per unit, each on half its head rows; contributors in warp order, so
// the result is deterministic).  It is launched as a programmatic dependent of
// the streaming kernel, so its CTAs are resident during the streaming
// kernel's tail.  Merging inside the streaming kernel (per warp or per CTA, by
// the last arriver) was measured and was slower: the arrivals and merges land
// on the critical path of the warps that finish last.
// The only CTA-wide synchronisation is the prologue, where the CTA scans
// kv_len into the per-sequence tile prefix it locates tiles with (or reads the
// schedule's); the warp that begins a cut unit leaves a descriptor of it for
// the fixup kernel (or the schedule holds it).
#include "mma_tile.cuh"

namespace mvb {

// Per-warp timeline, compiled in only with -DMVB_STREAM_TRACE: the trace build
// (lib/libmvb200_trace.so, made by build.build_trace(); bench.py --op trace
// loads it).  The product library holds none of it.  Each launch takes the
// next of kTraceLaunches slots (a per-warp arrival counter, so up to
// kTraceLaunches back-to-back launches after mvb_trace_clear() keep their own
// stamps), and lane 0 of a warp records %globaltimer (ns) at:
//   stream warp W: entry, first loads issued, first tile landed, loop end,
//                  end, and the landing of each of its first kTraceTiles tiles;
//   fixup warp gw (one with a cut unit): entry, wait returned, end.
#ifdef MVB_STREAM_TRACE
constexpr int kTraceLaunches = 8, kTraceWarps = 4096, kTraceFixWarps = 16384, kTraceTiles = 32;
__device__ int g_trace_wcnt[kTraceWarps];
__device__ int g_trace_fcnt[kTraceFixWarps];
__device__ unsigned long long g_trace_w[kTraceLaunches][kTraceWarps][5];
__device__ unsigned long long g_trace_t[kTraceLaunches][kTraceWarps][kTraceTiles];
__device__ unsigned long long g_trace_f[kTraceLaunches][kTraceFixWarps][3];
__device__ __forceinline__ unsigned long long trace_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define MVB_TRACE(...) __VA_ARGS__
#else
#define MVB_TRACE(...)
#endif

constexpr int kStreamRowBatch = 128;  // tiles whose pool rows a warp resolves at once
#ifndef MVB_STREAM_FIXUP_CB
#define MVB_STREAM_FIXUP_CB 4
#endif
#ifndef MVB_STREAM_FIXUP_SPLIT
#define MVB_STREAM_FIXUP_SPLIT 4
#endif
#ifndef MVB_STREAM_FIXUP_RP64
#define MVB_STREAM_FIXUP_RP64 2   // the warp fixup's head rows per pass, head_dim 64
#endif
#ifndef MVB_STREAM_FIXUP_RP128
#define MVB_STREAM_FIXUP_RP128 2  // ... head_dim 128
#endif
// The warp fixup's warps per cut unit, each merging its share of the unit's
// head rows: fewer rows per warp shorten the merge's serial work and cut its
// registers per contributor.  Config-2 decode with a schedule: 1 -> 2 warps
// per unit 34.1 -> 32.9 us, later 2 -> 4 warps (two head rows each) 31.5 ->
// 31.1 us; 8 warps, 8 contributors per batch, or two batches in flight
// (the next batch loaded before the current one is summed) were slower.
constexpr int kFixupWarpsPerUnit = MVB_STREAM_FIXUP_SPLIT;

// Per-step schedule of the stream kernel (MVB_DECODE_SCHEDULE_READY): what
// every layer of a model step would otherwise derive again from kv_len and the
// block tables, built once by decode_stream_schedule_kernel.
struct StreamSchedHeader {
  int total_tiles;
  int bits;       // MVB_DEV_* bits of the step's sequences and block ids
  int num_warps;  // the stream grid the schedule was cut for
  int pad[61];
};
static_assert(sizeof(StreamSchedHeader) == 256, "header is 256 bytes");
struct StreamRec {  // one per stream warp: its tile range and the pool rows of its first 32 tiles
  int4 h;           // {first tile, tiles, 0, 0}
  int rows[32];     // -1 past the range or for a bad block id
};
static_assert(sizeof(StreamRec) == 144, "record is 144 bytes");

struct StreamArgs {
  int4* desc;     // [num_warps][2] the cut unit each warp begins, for the fixup:
                  // {first tile, end tile, sequence, T_all}, {first head, heads, contributors, 0};
                  // first tile = -1 when the warp begins no cut unit
  float* part;    // [num_warps][2][16][D + 2] partial states (m, l, O[D] per row)
  int num_warps;  // gridDim.x * NW
  // the step's schedule (nullptr: the kernel derives its set-up from kv_len and the tables)
  const StreamSchedHeader* shdr;
  const int* spre;        // [Nd + 1] tile prefix per sequence (all its units)
  const int* sctx;        // [Nd] servable kv_len (0 = left out)
  const int* srows;       // [total_tiles] pool row of every tile, in stream order
  const StreamRec* srec;  // [num_warps]
  const int4* sdesc;      // [num_warps][2] the schedule's copy of `desc` (the fixup reads it)
};

// Warp whose range [R(w), R(w+1)), R(w) = floor(w * T / Wtot), holds global
// tile g: the largest w with R(w) <= g.
__device__ __forceinline__ int stream_warp_of(int g, int T, int Wtot) {
  return (int)(((int64_t)(g + 1) * Wtot + T - 1) / T) - 1;
}
__device__ __forceinline__ int stream_range_start(int w, int T, int Wtot) {
  return (int)((int64_t)w * T / Wtot);
}

// Cost-aware split.  A warp that enters a unit pays its flush, the lookup of
// the next unit and that unit's partial last tile besides the tiles (about one
// tile's time each: warps whose equal range touched two units ended 1.4 us
// later, three units 3.1 us later).  With F(g) = g + kStreamUnitCost * u(g),
// u(g) the index of the unit holding tile g (KHG units per sequence, counted
// over every sequence), warp w takes [b(w), b(w + 1)) with
//   b(w) = min{ g : F(g) * Wtot >= w * F(T) },   F(T) = T + kStreamUnitCost * KHG * Nd,
// and tile g belongs to warp floor(F(g) * Wtot / F(T)).  The schedule kernel
// cuts it when no sequence is left out (a left-out sequence would add cost
// without tiles) and F(T) >= 3 * Wtot (then every range holds a tile, so the
// contributors of a cut unit are consecutive warps); else, and without a
// schedule, the equal split R(w).
constexpr int kStreamUnitCost = 1;
// floor(a * b / c) for 0 <= a * b < 2^53 and c > 0: a double quotient
// corrected in integers (a 64-bit integer division is a long software routine)
__device__ __forceinline__ int64_t mul_div_floor(int64_t a, int64_t b, int64_t c) {
  const int64_t p = a * b;
  int64_t q = (int64_t)((double)p / (double)c);
  while (q * c > p) --q;
  while ((q + 1) * c <= p) ++q;
  return q;
}
struct StreamSplit {
  int T, KHG, Wtot;
  int64_t FT;  // F(T); 0: the equal split
};
__device__ __forceinline__ StreamSplit stream_split(int T, int KHG, int Nd, int Wtot, bool any_left_out) {
  StreamSplit sp;
  sp.T = T;
  sp.KHG = KHG;
  sp.Wtot = Wtot;
  const int64_t FT = (int64_t)T + (int64_t)kStreamUnitCost * KHG * Nd;
  sp.FT = !any_left_out && FT >= 3 * (int64_t)Wtot ? FT : 0;
  return sp;
}
// First tile of warp w's range; pre: the tile prefix per sequence (Nd + 1).
__device__ __forceinline__ int stream_split_start(const int* pre, int Nd, const StreamSplit& sp, int w) {
  if (sp.FT == 0) return stream_range_start(w, sp.T, sp.Wtot);
  const int64_t q = mul_div_floor(w, sp.FT, sp.Wtot);
  const int64_t target = q * sp.Wtot == (int64_t)w * sp.FT ? q : q + 1;  // ceil(w * F(T) / Wtot)
  const int64_t cu = (int64_t)kStreamUnitCost * sp.KHG;  // G(s) = pre[s] + cu * s: F at sequence s's first tile
  if (pre[Nd] + cu * Nd <= target) return pre[Nd];
  int lo = 0, hi = Nd;  // the last sequence s with G(s) <= target
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pre[mid] + cu * mid <= target)
      lo = mid;
    else
      hi = mid;
  }
  const int64_t off = target - (pre[lo] + cu * lo);
  const int ut = (pre[lo + 1] - pre[lo]) / sp.KHG;
  if (ut == 0) return pre[lo + 1];
  // within the sequence: F(pre[s] + x) = G(s) + x + cost * floor(x / ut)
  const int64_t k = off / (ut + kStreamUnitCost), t = off - k * (ut + kStreamUnitCost);
  const int64_t x = t >= ut ? (k + 1) * ut : k * ut + t;
  return (int)min((int64_t)pre[lo + 1], pre[lo] + x);
}
// Warp holding tile g, which is tile t of unit k of sequence s.
__device__ __forceinline__ int stream_split_warp_of(const int* pre, const StreamSplit& sp, int g, int s, int k) {
  if (sp.FT == 0) return stream_warp_of(g, sp.T, sp.Wtot);
  const int64_t F = (int64_t)g + (int64_t)kStreamUnitCost * ((int64_t)sp.KHG * s + k);
  return (int)min((int64_t)sp.Wtot - 1, mul_div_floor(F, sp.Wtot, sp.FT));
}

template <typename T, int D, int NW, int STAGES>
__global__ void __launch_bounds__(NW * 32)
decode_stream_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const DecodeArgs a, const StreamArgs sa) {
  using Geo = MmaGeom<D>;
  constexpr int KC = D / 16, NO = D / 8, ROW = D + 2;

  extern __shared__ uint8_t smem_raw[];
  __shared__ int warp_sums[NW];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NW * STAGES * Geo::STAGE_BYTES);
  int* stage_ok = reinterpret_cast<int*>(bars + NW * STAGES);  // [NW][STAGES]
  int* rows = stage_ok + NW * STAGES;                           // [NW][kStreamRowBatch]
  int* pre = rows + NW * kStreamRowBatch;                       // [Nd + 1] tile prefix per sequence
  int* ctxs = pre + a.num_seqs + 1;                             // [Nd] servable kv_len (0 = skipped)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Nd = a.num_seqs;
  const int KHG = a.num_kv_heads * a.head_groups;

  // Without early_inputs any input may come from the previous kernel in the
  // stream: wait for it first.  With it (the previous kernel is the KV write,
  // which writes only the cache) the set-up below reads query, block table and
  // kv_len at once, and only the first cache load waits.
  MVB_TRACE(const unsigned long long tr_entry = trace_now();)
  if (!a.early_inputs) grid_dependency_wait();
  grid_launch_dependents();    // the fixup kernel may be scheduled as CTAs retire

  const bool from_schedule = sa.srec != nullptr;
  int rec_row = -1;
  int4 rec_h = make_int4(0, 0, 0, 0);
  if (from_schedule) {
    rec_h = __ldcg(&(sa.srec + blockIdx.x * NW + warp)->h);
    // The step's schedule: the pool rows of this warp's first 32 tiles in one
    // read, the tile prefix and servable kv_len for locating units
    // (L2-resident: every layer of the step reads them).
    rec_row = __ldcg(&(sa.srec + blockIdx.x * NW + warp)->rows[lane]);
    for (int i = tid; i <= Nd; i += NW * 32) {
      pre[i] = __ldcg(sa.spre + i);
      if (i < Nd) ctxs[i] = __ldcg(sa.sctx + i);
    }
    __syncthreads();
    if (__ldcg(&sa.shdr->num_warps) != sa.num_warps) {  // cut for another grid: refuse
      if (tid == 0 && blockIdx.x == 0) atomicOr(a.err, MVB_DEV_SCHEDULE);
      if (lane == 0) sa.desc[2 * (blockIdx.x * NW + warp)] = make_int4(-1, 0, 0, 0);
      return;
    }
    if (blockIdx.x == 0) {  // rows of the sequences left out: zeros, and the step's error bits
      if (tid == 0) {
        const int bits = __ldcg(&sa.shdr->bits);
        if (bits) atomicOr(a.err, bits);
      }
      for (int i = warp; i < Nd; i += NW) {
        if (ctxs[i] != 0) continue;
        T* out = static_cast<T*>(a.out) + (int64_t)i * a.o_s0;
        for (int e = lane; e < a.num_heads * D; e += 32) out[(e / D) * a.o_s1 + e % D] = from_f32<T>(0.f);
      }
    }
  } else {
  // ---- prologue: tiles per sequence (all its units) and their exclusive prefix ----
  {
    constexpr int NT = NW * 32;
    const int per = (Nd + NT - 1) / NT;
    const int i0 = min(Nd, tid * per), i1 = min(Nd, i0 + per);
    int mine = 0;
    for (int i = i0; i < i1; ++i) {
      const int c = __ldg(a.kv_len + i);
      const int bad = seq_error(a, c);
      ctxs[i] = bad ? 0 : c;
      const int t = bad ? 0 : ((c + kTile - 1) / kTile) * KHG;
      pre[i] = t;
      mine += t;
      if (bad && blockIdx.x == 0) {
        atomicOr(a.err, bad);
        T* out = static_cast<T*>(a.out) + (int64_t)i * a.o_s0;
        for (int e = 0; e < a.num_heads * D; ++e) out[(e / D) * a.o_s1 + e % D] = from_f32<T>(0.f);
      }
    }
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    int run = incl - mine, total = 0;
    for (int w = 0; w < NW; ++w) {
      if (w < warp) run += warp_sums[w];
      total += warp_sums[w];
    }
    for (int i = i0; i < i1; ++i) {
      const int t = pre[i];
      pre[i] = run;
      run += t;
    }
    if (tid == 0) pre[Nd] = total;
    __syncthreads();
  }
  }

  const int T_all = pre[Nd];
  const int Wtot = sa.num_warps;
  const int W = blockIdx.x * NW + warp;
  // This warp's range: the record's with a schedule (the schedule kernel cut
  // the cost-aware split), else the equal split (the cost-aware split's
  // boundaries computed here made the launch 1.6 us slower at config 2).
  const StreamSplit split = stream_split(T_all, KHG, Nd, Wtot, /*any_left_out=*/true);
  const int r0 = from_schedule ? rec_h.x : stream_split_start(pre, Nd, split, W);
  const int r1 = from_schedule ? rec_h.x + rec_h.y : stream_split_start(pre, Nd, split, W + 1);
  const int n = r1 - r0;
  MVB_TRACE(int tr_slot = 0; const bool tr_on = lane == 0 && W < kTraceWarps;
            if (tr_on) {
              tr_slot = atomicAdd(&g_trace_wcnt[W], 1) % kTraceLaunches;
              g_trace_w[tr_slot][W][0] = tr_entry;
            })
  if (n <= 0) {  // no CTA-wide barrier follows
    if (lane == 0) sa.desc[2 * W] = make_int4(-1, 0, 0, 0);
    return;
  }

  uint64_t* mybars = bars + warp * STAGES;
  int* myok = stage_ok + warp * STAGES;
  int* myrows = rows + warp * kStreamRowBatch;
  uint8_t* myring = ring + warp * STAGES * Geo::STAGE_BYTES;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(mybars + s), 1);
    fence_mbar_init();
  }
  if (lane == 0 && warp == 0) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  __syncwarp();

  // global tile g -> sequence s, unit k of s, tile t of the unit
  auto locate = [&](int g, int& s, int& k, int& t) {
    int lo = 0, hi = Nd;  // pre[lo] <= g < pre[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pre[mid] <= g)
        lo = mid;
      else
        hi = mid;
    }
    s = lo;
    const int ut = (ctxs[s] + kTile - 1) / kTile;
    const int off = g - pre[s];
    k = off / ut;
    t = off - k * ut;
  };
  // All lanes: resolve the pool rows of tiles [j0, j0 + kStreamRowBatch) of this range.
  auto fill_rows = [&](int j0, int i0 = 0) {
    if (from_schedule) {
      for (int i = i0 + lane; i < kStreamRowBatch; i += 32) {
        const int j = j0 + i;
        myrows[i] = j < n ? __ldcg(sa.srows + r0 + j) : -1;
      }
      __syncwarp();
      return;
    }
    for (int i = i0 + lane; i < kStreamRowBatch; i += 32) {
      const int j = j0 + i;
      int row = -1;
      if (j < n) {
        int s, k, t;
        locate(r0 + j, s, k, t);
        const int kvh = k / a.head_groups;
        const int tok = t * kTile;
        const int bi = tok / a.block_size;
        const int64_t b = __ldg(a.bt + (int64_t)s * a.bt_s0 + bi);
        if (b >= 0 && b < a.num_blocks)
          row = ((int)b * a.num_kv_heads + kvh) * a.block_size + (tok - bi * a.block_size);
        else
          atomicOr(a.err, MVB_DEV_BLOCK_ID);
      }
      myrows[i] = row;
    }
    __syncwarp();
  };
  const uint64_t kv_policy = l2_policy_evict_first();
  // Lane 0: start the loads of local tile j into its stage.
  auto issue = [&](int j) {
    const int st = j % STAGES;
    const uint32_t bar = smem_u32(mybars + st);
    const int row = myrows[j % kStreamRowBatch];
    myok[st] = row >= 0;
    if (W == a.hold_warp && j == a.hold_tile) return;  // test hook: the stage never completes
    if (row < 0) {
      if (from_schedule) atomicOr(a.err, MVB_DEV_BLOCK_ID);  // resolved by the schedule: flag it per call
      mbar_arrive(bar);
      return;
    }
    mbar_arrive_expect_tx(bar, Geo::STAGE_BYTES);
    const uint32_t dk = smem_u32(myring + st * Geo::STAGE_BYTES);
#pragma unroll
    for (int p = 0; p < Geo::SUB; ++p) {
      tma_load_2d(dk + p * Geo::PANEL_BYTES, &tmk, p * 64, row, bar, kv_policy);
      tma_load_2d(dk + Geo::TILE_BYTES + p * Geo::PANEL_BYTES, &tmv, p * 64, row, bar, kv_policy);
    }
  };

  // The first 32 block ids only: the first loads are issued before the rest of
  // the batch is resolved (below).
  if (from_schedule) myrows[lane] = rec_row;
  for (int j = lane; j < 32 && !from_schedule; j += 32) {
    int row = -1;
    if (j < n) {
      int s, k, t;
      locate(r0 + j, s, k, t);
      const int kvh = k / a.head_groups;
      const int tok = t * kTile;
      const int bi = tok / a.block_size;
      const int64_t b = __ldg(a.bt + (int64_t)s * a.bt_s0 + bi);
      if (b >= 0 && b < a.num_blocks)
        row = ((int)b * a.num_kv_heads + kvh) * a.block_size + (tok - bi * a.block_size);
      else
        atomicOr(a.err, MVB_DEV_BLOCK_ID);
    }
    myrows[j] = row;
  }
  __syncwarp();

  const int g0 = lane >> 2, qd = lane & 3;
  uint32_t qa[KC][4], qa_next[KC][4];
  float o[NO][4] = {};
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  int u_start = 0, u_end = -1, u_seq = 0, u_k = 0, u_ctx = 0, h0 = 0, nh = 0;
  // head group of the next unit of this range, whose Q fragments are prefetched
  int n_h0 = 0, n_nh = 0;

  // Write the finished unit: normalised into `out` when this warp holds all of
  // it, else as a partial state for the fixup kernel.
  auto flush = [&]() {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
      lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
    }
    T* out = static_cast<T*>(a.out) + (int64_t)u_seq * a.o_s0;
    if (u_start >= r0 && u_end <= r1) {
      const float inv0 = 1.f / lrow[0], inv1 = 1.f / lrow[1];
#pragma unroll
      for (int nn = 0; nn < NO; ++nn) {
        const int d = nn * 8 + 2 * qd;
        if (g0 < nh) {
          T* p = out + (int64_t)(h0 + g0) * a.o_s1 + d;
          p[0] = from_f32<T>(o[nn][0] * inv0);
          p[1] = from_f32<T>(o[nn][1] * inv0);
        }
        if (g0 + 8 < nh) {
          T* p = out + (int64_t)(h0 + g0 + 8) * a.o_s1 + d;
          p[0] = from_f32<T>(o[nn][2] * inv1);
          p[1] = from_f32<T>(o[nn][3] * inv1);
        }
      }
      return;
    }
    const int slot = u_start < r0 ? 0 : 1;
    float* P = sa.part + ((int64_t)W * 2 + slot) * 16 * ROW;
    const bool row0 = g0 < nh, row1 = g0 + 8 < nh;  // rows past the group are padding
#pragma unroll
    for (int nn = 0; nn < NO; ++nn) {
      const int d = 2 + nn * 8 + 2 * qd;
      if (row0) *reinterpret_cast<float2*>(P + g0 * ROW + d) = make_float2(o[nn][0], o[nn][1]);
      if (row1) *reinterpret_cast<float2*>(P + (g0 + 8) * ROW + d) = make_float2(o[nn][2], o[nn][3]);
    }
    if (qd == 0) {
      if (row0) *reinterpret_cast<float2*>(P + g0 * ROW) = make_float2(mrow[0], lrow[0]);
      if (row1) *reinterpret_cast<float2*>(P + (g0 + 8) * ROW) = make_float2(mrow[1], lrow[1]);
    }
  };

  // Look up the unit holding global tile g (when g < r1) and prefetch its Q.
  auto prefetch_next = [&](int g) {
    if (g >= r1) return;
    int s, k, t;
    locate(g, s, k, t);
    const int kvh = k / a.head_groups, hg = k - kvh * a.head_groups;
    n_h0 = kvh * a.G + hg * 16;
    n_nh = min(16, a.G - hg * 16);
    load_q_frags<T, D>(a, s, n_h0, n_nh, qa_next);
  };

  prefetch_next(r0);  // the range's first unit (it may start before r0: locate handles it)
  if (a.early_inputs) grid_dependency_wait();  // the cache is complete from here on
  // The first wave in two halves: stage 0 of every warp now, the others when
  // the warp reaches its loop, so each warp's first tile is queued behind
  // fewer loads (config 2: -0.3 us).
  if (lane == 0 && n > 0) issue(0);
  MVB_TRACE(if (tr_on) g_trace_w[tr_slot][W][1] = trace_now();)
  fill_rows(0, 32);  // the rest of the first batch, while the first loads are in flight
  bool failed = false;
  int j = 0;
  for (; j < n; ++j) {
    const int g = r0 + j;
    if (g >= u_end) {  // warp-uniform: entering the prefetched unit
      if (j > 0) flush();
      {
        int s, k, t;
        locate(g, s, k, t);
        u_start = g - t;
        u_ctx = ctxs[s];
        u_seq = s;
        u_k = k;
      }
      u_end = u_start + (u_ctx + kTile - 1) / kTile;
      h0 = n_h0;
      nh = n_nh;
#pragma unroll
      for (int kc = 0; kc < KC; ++kc)
#pragma unroll
        for (int e = 0; e < 4; ++e) qa[kc][e] = qa_next[kc][e];
      prefetch_next(u_end);
#pragma unroll
      for (int nn = 0; nn < NO; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
      mrow[0] = mrow[1] = -INFINITY;
      lrow[0] = lrow[1] = 0.f;
    }
    if (j == 0 && lane == 0)
      for (int jj = 1; jj < (n < STAGES ? n : STAGES); ++jj) issue(jj);
    const int st = j % STAGES;
    const bool got = mbar_wait_bounded(smem_u32(mybars + st), (uint32_t)((j / STAGES) & 1), a.wait_limit);
    MVB_TRACE(if (tr_on) {
      const unsigned long long t = trace_now();
      if (j == 0) g_trace_w[tr_slot][W][2] = t;
      if (j < kTraceTiles) g_trace_t[tr_slot][W][j] = t;
    })
    if (__any_sync(0xffffffffu, !got)) {
      failed = true;
      break;
    }
    if (myok[st]) {
      const int valid = min(kTile, u_ctx - (g - u_start) * kTile);
      const uint32_t kb = smem_u32(myring + st * Geo::STAGE_BYTES);
      attend_tile<T, D>(kb, kb + Geo::TILE_BYTES, valid, a.scale_log2, qa, o, mrow, lrow);
    }
    __syncwarp();
    if (j + STAGES < n) {
      if ((j + STAGES) % kStreamRowBatch == 0) fill_rows(j + STAGES);
      if (lane == 0) {
        fence_proxy_async_smem();
        issue(j + STAGES);
      }
    }
  }
  if (failed) {
    if (lane == 0) atomicOr(a.err, MVB_DEV_TIMEOUT);
    const int issued = min(n, j + STAGES);
    for (int jj = j; jj < issued; ++jj)
      mbar_wait_bounded(smem_u32(mybars + jj % STAGES), (uint32_t)((jj / STAGES) & 1), a.wait_limit);
    if (lane == 0) sa.desc[2 * W] = make_int4(-1, 0, 0, 0);
    return;  // the unit's output stays unwritten; the error flag reports it
  }
  MVB_TRACE(if (tr_on) g_trace_w[tr_slot][W][3] = trace_now();)
  flush();
  // A unit that starts in this range and ends past it was begun here: this
  // warp is its first contributor, and the fixup finds the unit through it.
  if (lane == 0 && !from_schedule) {  // (a schedule holds its own copy of the descriptors)
    const bool begins_cut = u_start >= r0 && u_end > r1;
    sa.desc[2 * W] = begins_cut ? make_int4(u_start, u_end, u_seq, T_all) : make_int4(-1, 0, 0, 0);
    if (begins_cut) {
      // contributors: warps W .. the warp of the unit's last tile (every warp has
      // tiles), else one warp per tile
      const int nct = T_all >= Wtot ? stream_split_warp_of(pre, split, u_end - 1, u_seq, u_k) - W + 1
                                    : u_end - u_start;
      sa.desc[2 * W + 1] = make_int4(h0, nh, nct, 0);
    }
  }
  MVB_TRACE(if (tr_on) g_trace_w[tr_slot][W][4] = trace_now();)
}

// ---------------------------------------------------------------------------
// fixup, a few warps per unit: merge the partial states of every unit cut by
// a warp-range boundary (units cut into few pieces)
// ---------------------------------------------------------------------------
// kFixupWarpsPerUnit warps per warp w of the stream grid: when w begins a cut
// unit (its descriptor says which), each of them merges its share of the
// unit's head rows, RP rows per pass.  Lane c holds contributor c's (m, l) of each row; M and L come
// from warp reductions, and each lane accumulates its D/32 columns over the
// contributors with coefficients broadcast from the owning lane:
//   out[r][d] = sum_c O_c[r][d] 2^(m_c - M_r) / L_r.
// The O columns of the first CB contributors are requested together with the
// (m, l) values, so a pass over a unit cut into at most CB pieces costs one L2
// round trip after the descriptor's.  Contributors are the warps holding tiles
// of the unit, in warp order, so the result does not depend on timing: warps
// w..w_last when every warp has tiles (T_all >= warps), else (one tile per
// non-empty warp) the warps holding tiles us, us + 1, ...
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_stream_fixup_kernel(const DecodeArgs a, const StreamArgs sa) {
  constexpr int ROW = D + 2, DPL = D / 32;
  constexpr int RP = D == 64 ? MVB_STREAM_FIXUP_RP64 : MVB_STREAM_FIXUP_RP128;  // head rows per pass
  constexpr int CB = MVB_STREAM_FIXUP_CB;      // contributors per batch of O loads (divides 32)
  constexpr int SPLIT = kFixupWarpsPerUnit;    // warps per cut unit, each on its share of the head rows
  MVB_TRACE(const unsigned long long tr_entry = trace_now();)
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int w_first = gw / SPLIT, part_of = gw - w_first * SPLIT;
  const int Wtot = sa.num_warps;
  // The descriptor in one round trip: with a schedule its copy there, written
  // before the stream kernel ran, so it is read while that kernel finishes and
  // warps without a unit leave at once; else the stream kernel's, after it.
  if (sa.sdesc == nullptr) grid_dependency_wait();
  if (w_first >= Wtot) return;
  const int4* dsrc = sa.sdesc != nullptr ? sa.sdesc : sa.desc;
  const int4 d0 = __ldcg(dsrc + 2 * w_first);
  const int4 d1 = __ldcg(dsrc + 2 * w_first + 1);
  if (d0.x < 0) return;
  if (sa.sdesc != nullptr) grid_dependency_wait();  // the streaming kernel's partials are visible
  MVB_TRACE(int tr_slot = 0; const bool tr_on = lane == 0 && gw < kTraceFixWarps;
            if (tr_on) {
              tr_slot = atomicAdd(&g_trace_fcnt[gw], 1) % kTraceLaunches;
              g_trace_f[tr_slot][gw][0] = tr_entry;
              g_trace_f[tr_slot][gw][1] = trace_now();
            })
  const int us = d0.x, ue = d0.y, seq = d0.z, T_all = d0.w, h0 = d1.x, nrows = d1.y, nct = d1.z;
  const bool dense = T_all >= Wtot;
  auto contributor = [&](int c) { return dense ? w_first + c : stream_warp_of(us + c, T_all, Wtot); };
  // w_first keeps the unit in its "last" slot (1), later contributors in slot 0
  auto row_ptr = [&](int w, int r) -> const float* {
    return sa.part + ((int64_t)w * 2 + (w == w_first ? 1 : 0)) * 16 * ROW + r * ROW;
  };
  T* out = static_cast<T*>(a.out) + (int64_t)seq * a.o_s0;
  // this warp's head rows [r_lo, r_hi) of the unit
  const int rows_per = (nrows + SPLIT - 1) / SPLIT;
  const int r_lo = min(nrows, part_of * rows_per), r_hi = min(nrows, r_lo + rows_per);

  for (int rb = r_lo; rb < r_hi; rb += RP) {
    float x[CB][RP][DPL];  // O columns of contributors c0 .. c0 + CB - 1 (0 past the last)
    auto load_batch = [&](int c0) {
#pragma unroll
      for (int c = 0; c < CB; ++c) {
        const int w = c0 + c < nct ? contributor(c0 + c) : -1;
#pragma unroll
        for (int r = 0; r < RP; ++r)
#pragma unroll
          for (int i = 0; i < DPL; ++i)
            x[c][r][i] = w >= 0 && rb + r < r_hi ? __ldcg(row_ptr(w, rb + r) + 2 + lane + 32 * i) : 0.f;
      }
    };
    float2 ml[RP];  // (m, l) of contributor c32 + lane
    bool ok;        // ... which exists
    auto load_ml = [&](int c32) {
      const int w = c32 + lane < nct ? contributor(c32 + lane) : -1;
      ok = w >= 0;
#pragma unroll
      for (int r = 0; r < RP; ++r)
        ml[r] = ok && rb + r < r_hi ? __ldcg(reinterpret_cast<const float2*>(row_ptr(w, rb + r)))
                                     : make_float2(-INFINITY, 0.f);
    };
    load_batch(0);  // in flight during the (m, l) pass
    load_ml(0);
    // M_r = max_c m_c and L_r = sum_c l_c 2^(m_c - M_r), 32 contributors per step
    float M[RP], L[RP];
#pragma unroll
    for (int r = 0; r < RP; ++r) M[r] = -INFINITY, L[r] = 0.f;
    for (int c32 = 0;;) {
#pragma unroll
      for (int r = 0; r < RP; ++r) {
        float bm = ml[r].x;
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, sh));
        const float nm = fmaxf(M[r], bm);
        float sum = ok ? ml[r].y * fast_exp2(ml[r].x - nm) : 0.f;
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, sh);
        L[r] = L[r] * fast_exp2(M[r] - nm) + sum;
        M[r] = nm;
      }
      c32 += 32;
      if (c32 >= nct) break;
      load_ml(c32);
    }
    float inv[RP], cf[RP];  // cf: coefficient of contributor cf_base + lane
#pragma unroll
    for (int r = 0; r < RP; ++r) inv[r] = 1.f / L[r];
    auto coeffs = [&]() {
#pragma unroll
      for (int r = 0; r < RP; ++r) cf[r] = ok ? fast_exp2(ml[r].x - M[r]) * inv[r] : 0.f;
    };
    if (nct > 32) load_ml(0);  // the pass above left a later group of contributors in ml
    coeffs();
    int cf_base = 0;
    float acc[RP][DPL];
#pragma unroll
    for (int r = 0; r < RP; ++r)
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[r][i] = 0.f;
    for (int c0 = 0;; c0 += CB) {
      if (c0 - cf_base >= 32) {  // next group of 32 contributors
        cf_base += 32;
        load_ml(cf_base);
        coeffs();
      }
#pragma unroll
      for (int c = 0; c < CB; ++c)
#pragma unroll
        for (int r = 0; r < RP; ++r) {
          const float wt = __shfl_sync(0xffffffffu, cf[r], c0 - cf_base + c);
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[r][i] = fmaf(x[c][r][i], wt, acc[r][i]);
        }
      if (c0 + CB >= nct) break;
      load_batch(c0 + CB);
    }
#pragma unroll
    for (int r = 0; r < RP; ++r)
      if (rb + r < r_hi) {
        T* po = out + (int64_t)(h0 + rb + r) * a.o_s1;
#pragma unroll
        for (int i = 0; i < DPL; ++i) po[lane + 32 * i] = from_f32<T>(acc[r][i]);
      }
  }
  MVB_TRACE(if (tr_on) g_trace_f[tr_slot][gw][2] = trace_now();)
}

// ---------------------------------------------------------------------------
// fixup, one CTA per unit: the same merge for units cut into many pieces
// ---------------------------------------------------------------------------
// One CTA of kFixupWarps warps per kFixupWarps warps of the stream grid: for
// each of them that begins a cut unit (its descriptor says which), the whole
// CTA merges every head row of that unit, RP rows per pass:
//   out[r][d] = sum_c O_c[r][d] 2^(m_c - M_r) / L_r,
//   M_r = max_c m_c,  L_r = sum_c l_c 2^(m_c - M_r).
// The contributors are split into kFixupWarps contiguous shares.  Each warp
// loads its share's (m, l) (lane c: contributor c of the share) together with
// the O columns of its first CB contributors, reduces its share's max and sum,
// and the CTA combines the shares' (max, sum) pairs in shared memory; each warp
// then accumulates its share's columns with coefficients broadcast from the
// owning lanes, and the shares' sums are added in shared memory.  A unit cut
// into at most kFixupWarps * CB pieces costs one L2 round trip after the
// descriptor's; a long unit cut into ~30 pieces (32 K-token contexts) two.
// Contributors are the warps holding tiles of the unit, in warp order (w..w_last
// when every warp has tiles, T_all >= warps; else, with one tile per non-empty
// warp, the warps holding tiles us, us + 1, ...), and the summation order is
// fixed, so the result does not depend on timing.
constexpr int kFixupWarps = 4;
// Average pieces per unit above which the CTA fixup is used (the warp fixup
// merges CB = 4 pieces per L2 round trip).
constexpr int kFixupCtaPiecesPerUnit = 8;

template <typename T, int D>
__global__ void __launch_bounds__(kFixupWarps * 32) decode_stream_fixup_cta_kernel(const DecodeArgs a,
                                                                                  const StreamArgs sa) {
  constexpr int ROW = D + 2, DPL = D / 32, FW = kFixupWarps;
  constexpr int RP = D == 64 ? 8 : 4;  // head rows per pass
  constexpr int CB = 4;                // contributors per batch of O loads (divides 32)
  __shared__ float s_m[FW][RP], s_l[FW][RP];
  __shared__ float s_acc[FW][RP][D];
  __shared__ int4 s_desc[FW][2];
  grid_dependency_wait();  // the streaming kernel's partials and descriptors are visible
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Wtot = sa.num_warps;
  if (threadIdx.x < 2 * FW) {  // the FW descriptors of this CTA's stream warps, in one round trip
    const int w = blockIdx.x * FW + (threadIdx.x >> 1);
    s_desc[threadIdx.x >> 1][threadIdx.x & 1] = w < Wtot ? __ldcg((sa.sdesc != nullptr ? sa.sdesc : sa.desc) + 2 * w + (threadIdx.x & 1))
                                                         : make_int4(-1, 0, 0, 0);
  }
  __syncthreads();
  for (int q = 0; q < FW; ++q) {
    const int4 d0 = s_desc[q][0];
    if (d0.x < 0) continue;  // CTA-uniform
    const int4 d1 = s_desc[q][1];
    const int w_first = blockIdx.x * FW + q;
    const int us = d0.x, ue = d0.y, seq = d0.z, T_all = d0.w, h0 = d1.x, nrows = d1.y, nct = d1.z;
    const bool dense = T_all >= Wtot;
    auto contributor = [&](int c) { return dense ? w_first + c : stream_warp_of(us + c, T_all, Wtot); };
    // w_first keeps the unit in its "last" slot (1), later contributors in slot 0
    auto row_ptr = [&](int w, int r) -> const float* {
      return sa.part + ((int64_t)w * 2 + (w == w_first ? 1 : 0)) * 16 * ROW + r * ROW;
    };
    // this warp's share of the contributors: [c_lo, c_hi)
    const int share = (nct + FW - 1) / FW;
    const int c_lo = min(nct, warp * share), c_hi = min(nct, c_lo + share);
    T* out = static_cast<T*>(a.out) + (int64_t)seq * a.o_s0;

    for (int rb = 0; rb < nrows; rb += RP) {
      float x[CB][RP][DPL];  // O columns of contributors c0 .. c0 + CB - 1 of the share (0 past its end)
      auto load_batch = [&](int c0) {
  #pragma unroll
        for (int c = 0; c < CB; ++c) {
          const int w = c0 + c < c_hi ? contributor(c0 + c) : -1;
  #pragma unroll
          for (int r = 0; r < RP; ++r)
  #pragma unroll
            for (int i = 0; i < DPL; ++i)
              x[c][r][i] = w >= 0 && rb + r < nrows ? __ldcg(row_ptr(w, rb + r) + 2 + lane + 32 * i) : 0.f;
        }
      };
      float2 ml[RP];  // (m, l) of contributor c32 + lane
      bool ok;        // ... which exists
      auto load_ml = [&](int c32) {
        const int w = c32 + lane < c_hi ? contributor(c32 + lane) : -1;
        ok = w >= 0;
  #pragma unroll
        for (int r = 0; r < RP; ++r)
          ml[r] = ok && rb + r < nrows ? __ldcg(reinterpret_cast<const float2*>(row_ptr(w, rb + r)))
                                       : make_float2(-INFINITY, 0.f);
      };
      load_batch(c_lo);  // in flight during the (m, l) pass
      load_ml(c_lo);
      // the share's max and sum per row, 32 contributors per step
      float M[RP], L[RP];
  #pragma unroll
      for (int r = 0; r < RP; ++r) M[r] = -INFINITY, L[r] = 0.f;
      for (int c32 = c_lo; c32 < c_hi;) {
  #pragma unroll
        for (int r = 0; r < RP; ++r) {
          float bm = ml[r].x;
  #pragma unroll
          for (int sh = 16; sh > 0; sh >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, sh));
          const float nm = fmaxf(M[r], bm);
          float sum = ok && nm > -INFINITY ? ml[r].y * fast_exp2(ml[r].x - nm) : 0.f;
  #pragma unroll
          for (int sh = 16; sh > 0; sh >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, sh);
          L[r] = (M[r] > -INFINITY ? L[r] * fast_exp2(M[r] - nm) : 0.f) + sum;
          M[r] = nm;
        }
        c32 += 32;
        if (c32 >= c_hi) break;
        load_ml(c32);
      }
      if (lane == 0) {
  #pragma unroll
        for (int r = 0; r < RP; ++r) s_m[warp][r] = M[r], s_l[warp][r] = L[r];
      }
      __syncthreads();
      // the unit's max and sum per row, shares in a fixed order
      float inv[RP];
  #pragma unroll
      for (int r = 0; r < RP; ++r) {
        float gm = -INFINITY;
  #pragma unroll
        for (int q = 0; q < FW; ++q) gm = fmaxf(gm, s_m[q][r]);
        float gl = 0.f;
  #pragma unroll
        for (int q = 0; q < FW; ++q)
          if (s_m[q][r] > -INFINITY) gl += s_l[q][r] * fast_exp2(s_m[q][r] - gm);
        M[r] = gm;
        inv[r] = 1.f / gl;
      }
      float acc[RP][DPL];
  #pragma unroll
      for (int r = 0; r < RP; ++r)
  #pragma unroll
        for (int i = 0; i < DPL; ++i) acc[r][i] = 0.f;
      if (c_lo < c_hi) {
        // coefficient 2^(m_c - M) / L of contributor cf_base + lane
        float cf[RP];
        int cf_base = c_lo;
        auto coeffs = [&]() {
  #pragma unroll
          for (int r = 0; r < RP; ++r) cf[r] = ok ? fast_exp2(ml[r].x - M[r]) * inv[r] : 0.f;
        };
        if (c_hi - c_lo > 32) load_ml(c_lo);  // the pass above left a later group in ml
        coeffs();
        for (int c0 = c_lo;; c0 += CB) {
          if (c0 - cf_base >= 32) {  // next group of 32 contributors
            cf_base += 32;
            load_ml(cf_base);
            coeffs();
          }
  #pragma unroll
          for (int c = 0; c < CB; ++c)
  #pragma unroll
            for (int r = 0; r < RP; ++r) {
              const float wt = __shfl_sync(0xffffffffu, cf[r], c0 - cf_base + c);
  #pragma unroll
              for (int i = 0; i < DPL; ++i) acc[r][i] = fmaf(x[c][r][i], wt, acc[r][i]);
            }
          if (c0 + CB >= c_hi) break;
          load_batch(c0 + CB);
        }
      }
  #pragma unroll
      for (int r = 0; r < RP; ++r)
  #pragma unroll
        for (int i = 0; i < DPL; ++i) s_acc[warp][r][lane + 32 * i] = acc[r][i];
      __syncthreads();
      for (int e = threadIdx.x; e < RP * D; e += FW * 32) {
        const int r = e / D, col = e - r * D;
        if (rb + r < nrows) {
          float v = 0.f;
  #pragma unroll
          for (int q = 0; q < FW; ++q) v += s_acc[q][r][col];
          out[(int64_t)(h0 + rb + r) * a.o_s1 + col] = from_f32<T>(v);
        }
      }
      __syncthreads();  // s_m / s_acc are reused by the next pass
    }
  }  // q
}


// ---------------------------------------------------------------------------
// per-step schedule of the stream kernel
// ---------------------------------------------------------------------------
constexpr int kStreamSchedThreads = 512;

__device__ __forceinline__ int stream_sched_seq_error(int ctx, int block_size, int max_blocks) {
  if (ctx < 1) return MVB_DEV_KV_LEN;
  if (((int64_t)ctx + block_size - 1) / block_size > max_blocks) return MVB_DEV_TABLE_SHORT;
  return 0;
}

// One launch of C CTAs per model step.  Every CTA scans kv_len into the tile
// prefix (shared memory; tiles of a left-out sequence are 0), then resolves the
// pool rows of its 1/C share of the tile stream and the records of its 1/C
// share of the stream warps.  wait_at_end: as decode_schedule_kernel.
__global__ void __launch_bounds__(kStreamSchedThreads)
decode_stream_schedule_kernel(const int* __restrict__ kv_len, const int64_t* __restrict__ bt, int64_t bt_s0,
                              int num_seqs, int num_kv_heads, int head_groups, int block_size, int max_blocks,
                              int num_blocks, int G, int num_warps, StreamSchedHeader* hdr, int* spre, int* sctx,
                              int* srows, StreamRec* srec, int4* sdesc, int* err, int wait_at_end) {
  extern __shared__ int spre_s[];  // [num_seqs + 1]
  constexpr int NT = kStreamSchedThreads, NWP = NT / 32;
  __shared__ int s_red[2][NWP];
  if (!wait_at_end) grid_dependency_wait();
  grid_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ups = num_kv_heads * head_groups;
  const int per = (num_seqs + NT - 1) / NT;
  const int i0 = min(num_seqs, tid * per), i1 = min(num_seqs, i0 + per);
  int my_t = 0, my_bits = 0;
  for (int i = i0; i < i1; ++i) {
    const int ctx = __ldg(kv_len + i);
    const int e = stream_sched_seq_error(ctx, block_size, max_blocks);
    const int t = e ? 0 : (ctx + kTile - 1) / kTile * ups;
    spre_s[i] = t;
    my_t += t;
    my_bits |= e;
    if (blockIdx.x == 0) sctx[i] = e ? 0 : ctx;
  }
  int it = my_t, ob = my_bits;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, it, o);
    if (lane >= o) it += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ob |= __shfl_xor_sync(0xffffffffu, ob, o);
  if (lane == 31) s_red[0][warp] = it;
  if (lane == 0) s_red[1][warp] = ob;
  __syncthreads();
  int base = 0, T = 0, bits = 0;
  for (int w = 0; w < NWP; ++w) {
    if (w < warp) base += s_red[0][w];
    T += s_red[0][w];
    bits |= s_red[1][w];
  }
  int run = base + it - my_t;
  for (int i = i0; i < i1; ++i) {
    const int t = spre_s[i];
    spre_s[i] = run;
    run += t;
  }
  if (tid == 0) spre_s[num_seqs] = T;
  __syncthreads();
  if (blockIdx.x == 0)
    for (int i = tid; i <= num_seqs; i += NT) spre[i] = spre_s[i];
  // the unit holding stream tile g: sequence s, unit k of it, its first tile us and its tiles ut
  auto unit_of = [&](int g, int& s, int& k, int& us, int& ut) {
    int lo = 0, hi = num_seqs;  // spre_s[lo] <= g < spre_s[hi]: lo has tiles
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (spre_s[mid] <= g)
        lo = mid;
      else
        hi = mid;
    }
    s = lo;
    ut = (spre_s[lo + 1] - spre_s[lo]) / ups;
    k = (g - spre_s[lo]) / ut;
    us = spre_s[lo] + k * ut;
  };
  // pool row of stream tile g (-1 for a bad block id)
  auto row_of = [&](int g, int& bad) -> int {
    int s, k, us, ut;
    unit_of(g, s, k, us, ut);
    const int kvh = k / head_groups;
    const int tok = (g - us) * kTile;
    const int bi = tok / block_size;
    const int64_t b = __ldg(bt + (int64_t)s * bt_s0 + bi);
    if (b >= 0 && b < num_blocks) return ((int)b * num_kv_heads + kvh) * block_size + (tok - bi * block_size);
    bad = MVB_DEV_BLOCK_ID;
    return -1;
  };
  int my_bad = 0;
  const int C = gridDim.x;
  const int g0 = (int)((int64_t)blockIdx.x * T / C), g1 = (int)((int64_t)(blockIdx.x + 1) * T / C);
  for (int g = g0 + tid; g < g1; g += NT) srows[g] = row_of(g, my_bad);
  const int w0 = (int)((int64_t)blockIdx.x * num_warps / C), w1 = (int)((int64_t)(blockIdx.x + 1) * num_warps / C);
  const StreamSplit split = stream_split(T, ups, num_seqs, num_warps, bits != 0);
  for (int e = tid; e < (w1 - w0) * 32; e += NT) {
    const int W = w0 + e / 32, j = e % 32;
    const int r0 = stream_split_start(spre_s, num_seqs, split, W);
    const int r1 = stream_split_start(spre_s, num_seqs, split, W + 1);
    if (j == 0) {
      srec[W].h = make_int4(r0, r1 - r0, 0, 0);
      // the fixup's descriptor of the unit this warp begins and its range
      // cuts, as the decode kernel would write it
      int4 d0 = make_int4(-1, 0, 0, 0), d1 = make_int4(0, 0, 0, 0);
      if (r1 > r0) {
        int s, k, us, ut;
        unit_of(r1 - 1, s, k, us, ut);
        if (us >= r0 && us + ut > r1) {
          const int kvh = k / head_groups, hg = k - kvh * head_groups;
          const int nct = T >= num_warps ? stream_split_warp_of(spre_s, split, us + ut - 1, s, k) - W + 1 : ut;
          d0 = make_int4(us, us + ut, s, T);
          d1 = make_int4(kvh * G + hg * 16, min(16, G - hg * 16), nct, 0);
        }
      }
      sdesc[2 * W] = d0;
      sdesc[2 * W + 1] = d1;
    }
    srec[W].rows[j] = r0 + j < r1 ? row_of(r0 + j, my_bad) : -1;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) my_bad |= __shfl_xor_sync(0xffffffffu, my_bad, o);
  if (lane == 0 && (my_bad | (blockIdx.x == 0 && tid == 0 ? bits : 0))) atomicOr(err, my_bad | bits);
  if (blockIdx.x == 0 && tid == 0) {
    hdr->total_tiles = T;
    hdr->num_warps = num_warps;
    // every CTA's block-id errors are reported by the CTA itself; the header
    // carries the sequence errors, OR-ed in again by each decode
    hdr->bits = bits;
  }
  if (wait_at_end) grid_dependency_wait();
}

// ---------------------------------------------------------------------------
// host launch
// ---------------------------------------------------------------------------
// Warps per CTA and pipeline stages per warp (overridable at build time for
// tuning sweeps).  head_dim 64: one CTA of 16 warps per SM (128 registers a
// thread fill the register file) with 2 stages each; against 3 CTAs of 4 warps
// with 4 stages, the SM holds 32 tile loads in flight instead of 48 (a smaller
// first wave, so the first tiles land sooner) and runs 16 warps instead of 12
// (config-2 decode with a schedule 35.3 -> 33.9 us, config 3 94.5 -> 92.1 us).
// head_dim 128 keeps 4 warps x 3 stages (8 warps x 2 stages: config 4 +1.7 %).
#ifndef MVB_STREAM64_NW
#define MVB_STREAM64_NW 16
#endif
#ifndef MVB_STREAM64_STAGES
#define MVB_STREAM64_STAGES 2
#endif
#ifndef MVB_STREAM128_NW
#define MVB_STREAM128_NW 4
#endif
#ifndef MVB_STREAM128_STAGES
#define MVB_STREAM128_STAGES 3
#endif
template <int D> struct StreamConfig;
template <> struct StreamConfig<64> {
  static constexpr int NW = MVB_STREAM64_NW, STAGES = MVB_STREAM64_STAGES;
};
template <> struct StreamConfig<128> {
  static constexpr int NW = MVB_STREAM128_NW, STAGES = MVB_STREAM128_STAGES;
};

int stream_warps_per_cta(int head_dim) {
  return head_dim == 64 ? StreamConfig<64>::NW : StreamConfig<128>::NW;
}

int stream_smem_bytes(int head_dim, int num_seqs) {
  const int nw = stream_warps_per_cta(head_dim);
  const int stages = head_dim == 64 ? StreamConfig<64>::STAGES : StreamConfig<128>::STAGES;
  const int stage_bytes = head_dim == 64 ? MmaGeom<64>::STAGE_BYTES : MmaGeom<128>::STAGE_BYTES;
  return 1024 + nw * stages * (stage_bytes + 8 + 4) + nw * kStreamRowBatch * 4 +
         (2 * num_seqs + 1) * 4;
}

// CTAs of the stream grid: the CTAs the GPU holds at once, capped by the
// warps the workspace covers.  The per-step schedule is cut for this grid.
template <typename T, int D>
cudaError_t stream_ctas_t(int num_seqs, int max_warps, int sm_count, int* ctas_out) {
  constexpr int NW = StreamConfig<D>::NW, STAGES = StreamConfig<D>::STAGES;
  auto kern = decode_stream_kernel<T, D, NW, STAGES>;
  const int smem = stream_smem_bytes(D, num_seqs);
  cudaError_t e = ensure_kernel_attrs(kern, smem);
  if (e != cudaSuccess) return e;
  // Resident CTAs per SM, queried once per (device, shared-memory size): the
  // query costs microseconds of host time, and this runs once per layer-step.
  static std::mutex occ_mu;
  static int occ_dev[16], occ_smem[16], occ_val[16], occ_n = 0;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(occ_mu);
    for (int i = 0; i < occ_n; ++i)
      if (occ_dev[i] == dev && occ_smem[i] == smem) per_sm = occ_val[i];
    if (per_sm == 0) {
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NW * 32, smem);
      if (e != cudaSuccess) return e;
      if (per_sm < 1) per_sm = 1;
      const int slot = occ_n < 16 ? occ_n++ : (dev + smem) & 15;
      occ_dev[slot] = dev;
      occ_smem[slot] = smem;
      occ_val[slot] = per_sm;
    }
  }
  int ctas = per_sm * sm_count;
  if (ctas * NW > max_warps) ctas = max_warps / NW;
  if (ctas < 1) return cudaErrorInvalidConfiguration;
  *ctas_out = ctas;
  return cudaSuccess;
}

template <typename T, int D>
cudaError_t launch_stream_t(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                            int* scratch, float* part, int max_warps, int sm_count, const StreamSchedPtrs* sp,
                            cudaStream_t stream) {
  constexpr int NW = StreamConfig<D>::NW, STAGES = StreamConfig<D>::STAGES;
  auto kern = decode_stream_kernel<T, D, NW, STAGES>;
  const int smem = stream_smem_bytes(D, a.num_seqs);
  int ctas = 0;
  cudaError_t e = stream_ctas_t<T, D>(a.num_seqs, max_warps, sm_count, &ctas);
  if (e != cudaSuccess) return e;
  e = ensure_kernel_attrs(decode_stream_fixup_kernel<T, D>, 0);
  if (e != cudaSuccess) return e;
  e = ensure_kernel_attrs(decode_stream_fixup_cta_kernel<T, D>, 0);
  if (e != cudaSuccess) return e;
  StreamArgs sa = {};
  sa.desc = reinterpret_cast<int4*>(scratch);
  sa.part = part;
  sa.num_warps = ctas * NW;
  if (sp != nullptr) {
    sa.shdr = static_cast<const StreamSchedHeader*>(sp->hdr);
    sa.spre = sp->pre;
    sa.sctx = sp->ctx;
    sa.srows = sp->rows;
    sa.srec = static_cast<const StreamRec*>(sp->rec);
    sa.sdesc = static_cast<const int4*>(sp->desc);
  }
  e = launch_pdl(kern, dim3(ctas), dim3(NW * 32), smem, stream, tmk, tmv, a, sa);
  if (e != cudaSuccess) return e;
  // Stream warps per unit = the pieces an average unit is cut into: few (many
  // short sequences) -> one warp per unit; many (a few long sequences) -> the
  // warps of a CTA share a unit's pieces.
  const int64_t units = (int64_t)a.num_seqs * a.num_kv_heads * a.head_groups;
  const unsigned fixup_ctas = (unsigned)((sa.num_warps + 3) / 4);
  if ((int64_t)sa.num_warps > kFixupCtaPiecesPerUnit * units)
    return launch_pdl(decode_stream_fixup_cta_kernel<T, D>, dim3(fixup_ctas), dim3(kFixupWarps * 32), 0, stream, a,
                      sa);
  return launch_pdl(decode_stream_fixup_kernel<T, D>, dim3((sa.num_warps * kFixupWarpsPerUnit + 3) / 4), dim3(128), 0,
                    stream, a, sa);
}

cudaError_t launch_decode_stream(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                                 int dtype, int head_dim, int* scratch, float* part, int max_warps,
                                 int sm_count, const StreamSchedPtrs* sp, cudaStream_t stream) {
  if (dtype == MVB_DTYPE_BF16)
    return head_dim == 64
               ? launch_stream_t<__nv_bfloat16, 64>(tmk, tmv, a, scratch, part, max_warps, sm_count, sp, stream)
               : launch_stream_t<__nv_bfloat16, 128>(tmk, tmv, a, scratch, part, max_warps, sm_count, sp, stream);
  return head_dim == 64
             ? launch_stream_t<__half, 64>(tmk, tmv, a, scratch, part, max_warps, sm_count, sp, stream)
             : launch_stream_t<__half, 128>(tmk, tmv, a, scratch, part, max_warps, sm_count, sp, stream);
}

cudaError_t launch_decode_stream_schedule(const DecodeArgs& a, int dtype, int head_dim, int max_warps, int sm_count,
                                          const StreamSchedPtrs& sp, bool wait_at_end, cudaStream_t stream) {
  int ctas = 0;
  cudaError_t e;
  if (dtype == MVB_DTYPE_BF16)
    e = head_dim == 64 ? stream_ctas_t<__nv_bfloat16, 64>(a.num_seqs, max_warps, sm_count, &ctas)
                       : stream_ctas_t<__nv_bfloat16, 128>(a.num_seqs, max_warps, sm_count, &ctas);
  else
    e = head_dim == 64 ? stream_ctas_t<__half, 64>(a.num_seqs, max_warps, sm_count, &ctas)
                       : stream_ctas_t<__half, 128>(a.num_seqs, max_warps, sm_count, &ctas);
  if (e != cudaSuccess) return e;
  const int num_warps = ctas * stream_warps_per_cta(head_dim);
  auto kern = decode_stream_schedule_kernel;
  const int smem = (a.num_seqs + 1) * 4;
  e = ensure_kernel_attrs(kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(sm_count), dim3(kStreamSchedThreads), smem, stream, a.kv_len, a.bt, a.bt_s0,
                    a.num_seqs, a.num_kv_heads, a.head_groups, a.block_size, a.max_blocks, a.num_blocks, a.G,
                    num_warps,
                    static_cast<StreamSchedHeader*>(sp.hdr), const_cast<int*>(sp.pre), const_cast<int*>(sp.ctx),
                    const_cast<int*>(sp.rows), static_cast<StreamRec*>(const_cast<void*>(sp.rec)),
                    static_cast<int4*>(const_cast<void*>(sp.desc)), a.err,
                    wait_at_end ? 1 : 0);
}

}  // namespace mvb

#ifdef MVB_STREAM_TRACE
// Trace build only (not part of the product ABI): zero the arrival counters
// and stamps, and copy the stamps out (host buffers of the arrays' sizes:
// [8][4096][5], [8][4096][32] and [8][16384][3] unsigned 64-bit).
extern "C" int mvb_trace_clear() {
  cudaError_t e = cudaSuccess;
  const void* syms[] = {&mvb::g_trace_wcnt, &mvb::g_trace_fcnt, &mvb::g_trace_w, &mvb::g_trace_t, &mvb::g_trace_f};
  const size_t sizes[] = {sizeof(mvb::g_trace_wcnt), sizeof(mvb::g_trace_fcnt), sizeof(mvb::g_trace_w),
                          sizeof(mvb::g_trace_t), sizeof(mvb::g_trace_f)};
  for (int i = 0; i < 5 && e == cudaSuccess; ++i) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, syms[i]);
    if (e == cudaSuccess) e = cudaMemset(p, 0, sizes[i]);
  }
  return (int)e;
}

extern "C" int mvb_trace_read(void* warps, void* tiles, void* fixups) {
  cudaError_t e = cudaMemcpyFromSymbol(warps, mvb::g_trace_w, sizeof(mvb::g_trace_w));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(tiles, mvb::g_trace_t, sizeof(mvb::g_trace_t));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(fixups, mvb::g_trace_f, sizeof(mvb::g_trace_f));
  return (int)e;
}
#endif
