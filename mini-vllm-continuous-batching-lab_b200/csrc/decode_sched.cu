// Scheduled persistent paged decode (bf16 / f16, block_size a multiple of 16).
//
// Two kernels.
//
// decode_schedule_kernel runs once per model step (kv_len and the block tables
// are the same for every layer of a step).  The decode's work is the stream of
// 16-token K/V tiles of every unit — (sequence, KV head, head group of <= 16
// query heads) — in sequence order.  The schedule cuts that stream into one
// contiguous range per CTA of the decode grid (one CTA per SM; the lengths
// differ by at most one tile) and writes, for each CTA:
//   * its pieces: the part of each unit its range covers.  A unit cut by a
//     range boundary has one piece in every CTA it spans.  The piece cut by the
//     range's end is processed first, the piece cut by its start second and the
//     whole units longest first, so the partial states of cut units are stored
//     early and merged while the CTAs stream their longest whole units;
//   * the pool row of each of its tiles, in processing order: the block-table
//     lookups of every layer of the step, done once;
//   * a 256-byte record at a fixed place: where its pieces and rows are, its
//     first two pieces and the first rows of every consumer warp, so that a
//     decode CTA issues its first loads after one read.
// Sequences with kv_len < 1 or a block table too short for kv_len are left out
// of the stream and listed apart; the decode writes zeros to their rows.
//
// decode_sched_kernel: one CTA per SM, NC consumer warps and one merger warp.
//   * consumer c takes tiles c, c + NC, c + 2 NC, ... of its CTA's range.  It
//     issues the TMA loads of its own tiles (K and V, 16 rows x D, 128-byte
//     swizzle, 2-D tensor maps) S tiles ahead into its own S-stage ring and runs
//     attend_tile (mma.sync m16n8k16, online softmax, fp32 accumulate).  When its
//     next tile lies in a later piece it hands its state for the piece to the
//     merger, through one of NB shared-memory buffers, and switches to the next
//     piece's query fragments, loaded one piece ahead.  Warps that issue their
//     own copies stream like the stream kernel's; a separate issuing warp caps
//     a CTA near 8 tiles per microsecond (the copies one warp issues are
//     accepted one after another, ~60 ns each);
//   * the merger combines the consumer states of each piece in consumer order.
//     A whole unit is normalised and written to `out`.  A cut piece is stored
//     as a partial state (O, m, l per head row) and counted in on the unit's
//     arrival counter; the last of the unit's pieces to arrive merges all of
//     them in CTA order and writes the unit.
// Which consumer and which CTA take which tile is fixed by the schedule, so the
// result does not depend on timing.
//
// Every wait is bounded (DecodeArgs::wait_limit); a wait that runs out sets
// MVB_DEV_TIMEOUT and a CTA-wide abort flag that every other wait polls; each
// consumer then waits (bounded) for its own loads in flight and every warp
// leaves.  An arrival counter may then be left dirty: the schedule must be
// rebuilt (the schedule kernel zeroes every counter).
#include "mma_tile.cuh"

namespace mvb {

constexpr int kSchedBuildThreads = 512;
constexpr int kSchedMaxSeqs = 16384;  // sequences the schedule kernel's prefix arrays hold
constexpr int kSchedMaxCtas = kSchedBuildThreads;
constexpr int kSchedRecRows = 44;     // first rows a CTA record carries (NC * S of the decode)
constexpr int kSchedSortMax = 256;    // a CTA's whole pieces are sorted longest first up to this many pieces

// Workspace header (256 bytes).
struct SchedHeader {
  int total_tiles;  // tiles of all units of good sequences
  int ctas;         // CTAs with work: min(grid, total_tiles)
  int n_bad;        // sequences left out (kv_len < 1, block table too short)
  int bad_bits;     // their error bits, OR-ed
  int pad[60];
};
static_assert(sizeof(SchedHeader) == 256, "header is 256 bytes");

// Piece descriptor: two int4
//   {sequence, unit of the sequence (kvh * head_groups + hg), first tile of the
//    piece in the unit, tiles}
//   {position of its first tile in the CTA's processing order, kv_len,
//    first CTA of a cut unit (-1: the piece is the whole unit),
//    (CTAs the cut unit spans << 1) | (1 when it starts at that CTA's range start)}
// Per-CTA record (256 bytes): {first piece, pieces, first tile position of the
// range, tiles}, the first two pieces, and the pool row of tile c + NC * i of
// the range at rows0[c * S + i] (-1 past the range).
struct SchedRec {
  int4 h;
  int4 p[2][2];
  int rows0[kSchedRecRows];
};
static_assert(sizeof(SchedRec) == 256, "record is 256 bytes");

struct SchedArgs {
  const SchedHeader* hdr;
  const SchedRec* rec;  // [grid]
  const int4* desc;     // [max_pieces][2]
  const int* rows;      // [max_tiles] pool rows by tile position
  const int* bad;       // [num_seqs] sequences left out, in order
  int* ucnt;            // [grid] arrival counters of cut units, by first CTA
  float* part;          // [2 * grid][mg][D + 4] partial states: O (D), m, l
  int mg;               // query heads per unit: min(16, G)
  int nb;               // merge buffers (1 or 2)
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

// Last i in [0, n) with v[i] <= x (v non-decreasing, v[0] <= x).
__device__ __forceinline__ int sched_last_le(const int* v, int n, int x) {
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (v[mid] <= x)
      lo = mid;
    else
      hi = mid;
  }
  return lo;
}

// One CTA per CTA of the decode grid; each scans kv_len itself (a few KB from
// L2) and writes its own record, pieces and rows.  wait_at_end: the previous
// kernel in the stream may still be running and writes none of this kernel's
// inputs (the KV write); the kernel computes first and waits for it only
// before exiting, so that a dependent of this kernel that waits for it also
// waits for that previous kernel.
__global__ void __launch_bounds__(kSchedBuildThreads)
decode_schedule_kernel(const int* __restrict__ kv_len, const int64_t* __restrict__ bt, int64_t bt_s0,
                       int num_seqs, int num_kv_heads, int head_groups, int block_size, int max_blocks,
                       int num_blocks, int nc, int stages, SchedHeader* hdr, SchedRec* rec, int4* desc,
                       int* rows, int* bad, int* ucnt, int* err, int wait_at_end) {
  extern __shared__ int sched_smem[];
  int* pseq = sched_smem;                 // [num_seqs + 1] first tile position of the sequence's units
  int* gseq = sched_smem + num_seqs + 1;  // [num_seqs + 1] good sequences before it
  constexpr int NT = kSchedBuildThreads, NWP = NT / 32;
  __shared__ int s_red[3][NWP];
  __shared__ int s_cnt[NWP];
  __shared__ int s_len[kSchedSortMax];
  if (!wait_at_end) grid_dependency_wait();
  grid_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ups = num_kv_heads * head_groups;
  const int c = blockIdx.x;

  // ---- tiles of each sequence (all its units), exclusive prefixes ----
  const int per = (num_seqs + NT - 1) / NT;
  const int i0 = min(num_seqs, tid * per), i1 = min(num_seqs, i0 + per);
  int my_t = 0, my_g = 0, my_bits = 0;
  for (int i = i0; i < i1; ++i) {
    const int ctx = __ldg(kv_len + i);
    const int e = sched_seq_error(ctx, block_size, max_blocks);
    const int t = e ? 0 : (ctx + kTile - 1) / kTile * ups;
    pseq[i] = t;
    gseq[i] = e ? 0 : 1;
    my_t += t;
    my_g += e ? 0 : 1;
    my_bits |= e;
  }
  int it = my_t, ig = my_g, ob = my_bits;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int vt = __shfl_up_sync(0xffffffffu, it, o), vg = __shfl_up_sync(0xffffffffu, ig, o);
    if (lane >= o) {
      it += vt;
      ig += vg;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ob |= __shfl_xor_sync(0xffffffffu, ob, o);
  if (lane == 31) {
    s_red[0][warp] = it;
    s_red[1][warp] = ig;
  }
  if (lane == 0) s_red[2][warp] = ob;
  __syncthreads();
  int base_t = 0, base_g = 0, T = 0, NG = 0, bits = 0;
  for (int w = 0; w < NWP; ++w) {
    if (w < warp) {
      base_t += s_red[0][w];
      base_g += s_red[1][w];
    }
    T += s_red[0][w];
    NG += s_red[1][w];
    bits |= s_red[2][w];
  }
  int run_t = base_t + it - my_t, run_g = base_g + ig - my_g;
  for (int i = i0; i < i1; ++i) {
    const int t = pseq[i], g = gseq[i];
    pseq[i] = run_t;
    gseq[i] = run_g;
    run_t += t;
    run_g += g;
  }
  if (tid == 0) {
    pseq[num_seqs] = T;
    gseq[num_seqs] = NG;
  }
  __syncthreads();

  const int Ce = T < (int)gridDim.x ? T : (int)gridDim.x;
  if (c == 0) {
    for (int i = tid; i < num_seqs; i += NT)
      if (gseq[i + 1] == gseq[i]) bad[i - gseq[i]] = i;
    if (tid == 0) {
      hdr->total_tiles = T;
      hdr->ctas = Ce;
      hdr->n_bad = num_seqs - NG;
      hdr->bad_bits = bits;
      if (bits) atomicOr(err, bits);
    }
  }
  if (tid == 0) ucnt[c] = 0;
  if (c >= Ce) {
    if (tid == 0) rec[c].h = make_int4(0, 0, 0, 0);
    if (wait_at_end) grid_dependency_wait();
    return;
  }

  auto R = [&](int x) { return (int)((int64_t)x * T / Ce); };
  // CTA whose range holds tile position x: the largest c with R(c) <= x
  auto cta_of = [&](int x) { return (int)(((int64_t)(x + 1) * Ce + T - 1) / T) - 1; };
  // the unit holding tile position x < T: sequence, unit of it, its tiles, its first position
  auto locate = [&](int x, int& s, int& k, int& t, int& p) {
    s = sched_last_le(pseq, num_seqs, x);  // pseq[s] <= x < pseq[s + 1]: s has tiles
    t = (pseq[s + 1] - pseq[s]) / ups;
    k = (x - pseq[s]) / t;
    p = pseq[s] + k * t;
  };
  auto good_unit = [&](int s, int k) { return gseq[s] * ups + k; };

  // pieces of the CTAs before this one (c < Ce <= NT: one range per thread)
  int cnt = 0;
  if (tid < c) {
    int s0, k0, t0, p0, s1, k1, t1, p1;
    locate(R(tid), s0, k0, t0, p0);
    locate(R(tid + 1) - 1, s1, k1, t1, p1);
    cnt = good_unit(s1, k1) - good_unit(s0, k0) + 1;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if (lane == 0) s_cnt[warp] = cnt;
  __syncthreads();
  int pbase = 0;
  for (int w = 0; w < NWP; ++w) pbase += s_cnt[w];

  const int r0 = R(c), r1 = R(c + 1), n = r1 - r0;
  int sa, ka, ta, pa, sb, kb, tb, pb;
  locate(r0, sa, ka, ta, pa);
  locate(r1 - 1, sb, kb, tb, pb);
  const int gua = good_unit(sa, ka);
  const int np = good_unit(sb, kb) - gua + 1;
  // Processing order: the piece cut by the range's end first (when there are
  // two pieces or more it starts inside the range), the piece cut by its start
  // second, then the whole units longest first (ties in unit order; in unit
  // order when there are more than kSchedSortMax pieces).
  const bool cut_s = pa < r0, cut_e = pb + tb > r1;
  const int len0 = min(pa + ta, r1) - r0, len_l = r1 - max(pb, r0);
  const int n_head = np == 1 ? 1 : (cut_e ? 1 : 0) + (cut_s ? 1 : 0);
  const int head_len = np == 1 ? len0 : (cut_e ? len_l : 0) + (cut_s ? len0 : 0);
  const bool sorted = np <= kSchedSortMax;
  auto unit_piece = [&](int i, int& s, int& k, int& P, int& ps, int& pe) {
    const int g = gua + i, gs = g / ups;
    s = sched_last_le(gseq, num_seqs, gs);  // the good sequence number gs
    k = g - gs * ups;
    const int t = (pseq[s + 1] - pseq[s]) / ups;
    P = pseq[s] + k * t;
    ps = max(P, r0);
    pe = min(P + t, r1);
  };
  if (sorted) {
    for (int i = tid; i < np; i += NT) {
      int s, k, P, ps, pe;
      unit_piece(i, s, k, P, ps, pe);
      s_len[i] = pe - ps;
    }
    __syncthreads();
  }
  auto is_head = [&](int i) { return np == 1 || (i == np - 1 && cut_e) || (i == 0 && cut_s); };
  if (tid == 0) rec[c].h = make_int4(pbase, np, r0, n);
  for (int i = tid; i < np; i += NT) {
    int s, k, P, ps, pe;
    unit_piece(i, s, k, P, ps, pe);
    const int len = pe - ps;
    int pos, v0;
    if (np == 1 || (i == np - 1 && cut_e)) {
      pos = 0;
      v0 = 0;
    } else if (i == 0 && cut_s) {
      pos = cut_e ? 1 : 0;
      v0 = cut_e ? len_l : 0;
    } else if (sorted) {
      int rank = 0, before = 0;
      for (int j = 0; j < np; ++j) {
        if (j == i || is_head(j)) continue;
        const int lj = s_len[j];
        if (lj > len || (lj == len && j < i)) {
          ++rank;
          before += lj;
        }
      }
      pos = n_head + rank;
      v0 = head_len + before;
    } else {
      pos = i - (cut_s ? 1 : 0) + n_head;
      v0 = head_len + ps - (r0 + (cut_s ? len0 : 0));
    }
    int c0 = -1, w = 0;
    const int t = (pseq[s + 1] - pseq[s]) / ups;
    if (P < r0 || P + t > r1) {
      c0 = cta_of(P);
      const int c1 = cta_of(P + t - 1);
      w = ((c1 - c0 + 1) << 1) | (P == R(c0) ? 1 : 0);
    }
    const int4 d0 = make_int4(s, k, ps - P, len);
    const int4 d1 = make_int4(v0, __ldg(kv_len + s), c0, w);
    desc[2 * (pbase + pos)] = d0;
    desc[2 * (pbase + pos) + 1] = d1;
    if (pos < 2) {
      rec[c].p[pos][0] = d0;
      rec[c].p[pos][1] = d1;
    }
  }
  __syncthreads();  // this CTA's descriptors are visible to all its threads

  // pool rows, one warp per piece
  for (int pos = warp; pos < np; pos += NWP) {
    const int4 d0 = __ldcg(desc + 2 * (pbase + pos)), d1 = __ldcg(desc + 2 * (pbase + pos) + 1);
    const int s = d0.x, kvh = d0.y / head_groups, t0 = d0.z, len = d0.w, v0 = d1.x;
    for (int i = lane; i < len; i += 32) {
      const int tok = (t0 + i) * kTile;
      const int bi = tok / block_size;
      const int64_t b = __ldg(bt + (int64_t)s * bt_s0 + bi);
      int row = -1;
      if (b >= 0 && b < num_blocks)
        row = ((int)b * num_kv_heads + kvh) * block_size + (tok - bi * block_size);
      else
        atomicOr(err, MVB_DEV_BLOCK_ID);
      const int j = v0 + i;
      rows[r0 + j] = row;
      const int ii = j / nc;
      if (ii < stages) rec[c].rows0[(j - ii * nc) * stages + ii] = row;
    }
  }
  for (int e = tid; e < nc * stages; e += NT) {
    const int cc = e / stages, ii = e - cc * stages;
    if (cc + nc * ii >= n) rec[c].rows0[e] = -1;
  }
  if (wait_at_end) grid_dependency_wait();
}

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
// Per head dim: consumer warps and ring stages per consumer.  The CTA keeps
// NC * S tiles in flight (176 KB at D 64, 192 KB at D 128); the decode is bound
// by the bytes in flight (40 stages of 4 KB stream ~12 % slower than 44).  The
// registers a thread may use follow from the warps one SM sub-partition holds:
// 12 warps (3 per sub-partition) get 168, enough at D 64; D 128 needs ~250, so
// 6 consumers and the merger (2 per sub-partition).  Overridable at build time
// for tuning sweeps.
#ifndef MVB_SCHED64_NC
#define MVB_SCHED64_NC 11
#endif
#ifndef MVB_SCHED64_STAGES
#define MVB_SCHED64_STAGES 4
#endif
#ifndef MVB_SCHED128_NC
#define MVB_SCHED128_NC 6
#endif
#ifndef MVB_SCHED128_STAGES
#define MVB_SCHED128_STAGES 4
#endif
template <int D> struct SchedConfig;
template <> struct SchedConfig<64> {
  static constexpr int NC = MVB_SCHED64_NC, S = MVB_SCHED64_STAGES;
};
template <> struct SchedConfig<128> {
  static constexpr int NC = MVB_SCHED128_NC, S = MVB_SCHED128_STAGES;
};

// Shared memory: rings [NC][S] stages, NB merge buffers [NC][mg][D + 4] floats,
// barriers (NC * S tile-full, NB merge-full, NB merge-empty), per-stage bad-row
// flags, the abort flag (16 bytes), the merger's descriptor ring (4 x 32 bytes).
template <int D> struct SchedSmem {
  static constexpr int NC = SchedConfig<D>::NC, S = SchedConfig<D>::S;
  static_assert(NC * S <= kSchedRecRows, "the record carries every consumer's first rows");
  static_assert(NC * S % 4 == 0, "barriers and flags keep the descriptor ring 16-byte aligned");
  static constexpr int THREADS = (NC + 1) * 32;
  static constexpr int RING = NC * S * MmaGeom<D>::STAGE_BYTES;
  static __host__ __device__ constexpr int merge_bytes(int mg) { return NC * mg * (D + 4) * 4; }
  static __host__ __device__ constexpr int bytes(int mg, int nb) {
    return RING + nb * merge_bytes(mg) + (NC * S + 2 * nb) * 8 + NC * S * 4 + 16 + 128;
  }
};

// Bounded wait that also gives up when another warp has aborted the CTA.
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

// 16-byte global -> shared copy through L2 (cp.async), in the thread's current group.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One arrival for a whole warp: __syncwarp orders every lane's shared-memory
// accesses before lane 0's arrive (release).
__device__ __forceinline__ void warp_arrive(uint32_t bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// (M, L, O[cq .. cq + D/4)) of head row r from the consumer states of one
// merge buffer ([NC][mg][D + 4] floats: O, m, l): consumer cc holds tiles of the
// piece when some i < len has (first + i) % NC == cc; one without tiles, or
// whose tiles all had bad block ids (m = -inf, O = 0), weighs 0.  Branch-free,
// so that every consumer's loads are in flight together.  `row_ok`: r is a
// head row of the unit (else the result is zeros and nothing is read).
template <int D, int NC>
__device__ __forceinline__ void merge_row(const float* mb, int mg, int r, int cq, int first, int len, bool row_ok,
                                          float& M, float& L, float (&O)[D / 4]) {
  constexpr int CQ = D / 4, PR = D + 4;
  M = -INFINITY;
  L = 0.f;
#pragma unroll
  for (int i = 0; i < CQ; ++i) O[i] = 0.f;
  auto holds = [&](int cc) {
    int x = cc - first;
    x += x < 0 ? NC : 0;
    return row_ok && (len >= NC || x < len);
  };
#pragma unroll
  for (int cc = 0; cc < NC; ++cc)
    if (holds(cc)) M = fmaxf(M, mb[(cc * mg + r) * PR + D]);
  const float mref = M == -INFINITY ? 0.f : M;  // no readable token: zeros
#pragma unroll
  for (int cc = 0; cc < NC; ++cc) {
    const bool in = holds(cc);
    const float2 ml = in ? *reinterpret_cast<const float2*>(mb + (cc * mg + r) * PR + D) : make_float2(-INFINITY, 0.f);
    const float w = fast_exp2(ml.x - mref);  // 0 for m = -inf
    L = fmaf(ml.y, w, L);
    const float4* src = reinterpret_cast<const float4*>(mb + (cc * mg + r) * PR + cq);
#pragma unroll
    for (int i = 0; i < CQ / 4; ++i) {
      const float4 v = in ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      O[4 * i] = fmaf(v.x, w, O[4 * i]);
      O[4 * i + 1] = fmaf(v.y, w, O[4 * i + 1]);
      O[4 * i + 2] = fmaf(v.z, w, O[4 * i + 2]);
      O[4 * i + 3] = fmaf(v.w, w, O[4 * i + 3]);
    }
  }
}

// n = D / 4 normalised values of one output row, x[i] * inv, to p: two 16-byte
// stores when p is 16-byte aligned, else element by element.
template <typename T, int N>
__device__ __forceinline__ void store_row(T* p, const float (&x)[N], float inv) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
    for (int v = 0; v < N / 8; ++v) {
      uint4 w;
      w.x = Mma16816<T>::pack(x[8 * v] * inv, x[8 * v + 1] * inv);
      w.y = Mma16816<T>::pack(x[8 * v + 2] * inv, x[8 * v + 3] * inv);
      w.z = Mma16816<T>::pack(x[8 * v + 4] * inv, x[8 * v + 5] * inv);
      w.w = Mma16816<T>::pack(x[8 * v + 6] * inv, x[8 * v + 7] * inv);
      reinterpret_cast<uint4*>(p)[v] = w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = from_f32<T>(x[i] * inv);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(SchedSmem<D>::THREADS, 1)
decode_sched_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                    const DecodeArgs a, const SchedArgs sa) {
  using Geo = MmaGeom<D>;
  using L = SchedSmem<D>;
  constexpr int NC = L::NC, S = L::S, KC = D / 16, NO = D / 8, PR = D + 4;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NB = sa.nb, mg = sa.mg;
  uint8_t* ring = smem;
  float* merge = reinterpret_cast<float*>(smem + L::RING);  // [NB][NC][mg][PR]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::RING + NB * L::merge_bytes(mg));  // [NC][S]
  uint64_t* mfull = full + NC * S;  // [NB] consumer states written
  uint64_t* mempty = mfull + NB;    // [NB] states read by the merger
  volatile int* stage_bad = reinterpret_cast<volatile int*>(mempty + NB);  // [NC][S]
  volatile int* abort_flag = stage_bad + NC * S;
  int4* dring = reinterpret_cast<int4*>(const_cast<int*>(abort_flag) + 4);  // [4][2] merger's descriptor ring

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < NC * S; ++i) mbar_init(smem_u32(full + i), 1);
    for (int b = 0; b < NB; ++b) {
      mbar_init(smem_u32(mfull + b), NC);  // the consumer warps
      mbar_init(smem_u32(mempty + b), 1);  // the merger warp
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();  // the only CTA-wide barrier
  grid_launch_dependents();
  const int limit = a.wait_limit;
  // Without early_inputs the schedule or any input may come from the previous
  // kernel: wait for it first.  With it (the schedule is older than the
  // previous kernel, the KV write, which writes only the cache) everything but
  // the cache is read at once, and the first cache load waits.
  if (!a.early_inputs) grid_dependency_wait();
  const SchedRec* rc = sa.rec + blockIdx.x;
  const int4 h = __ldcg(&rc->h);
  // A consumer's first rows and the first two pieces share the header's round
  // trip (requested before anything waits for the header).
  int row0 = -1;
  int4 p00 = make_int4(0, 0, 0, 0), p01 = p00, p10 = p00, p11 = p00;
  if (warp < NC) {
    if (lane < S) row0 = __ldcg(&rc->rows0[warp * S + lane]);
    p00 = __ldcg(&rc->p[0][0]);
    p01 = __ldcg(&rc->p[0][1]);
    p10 = __ldcg(&rc->p[1][0]);
    p11 = __ldcg(&rc->p[1][1]);
  }
  const int pbase = h.x, np = h.y, r0 = h.z, n = h.w;
  auto piece = [&](int p, int4& d0, int4& d1) {
    if (p < 2) {
      d0 = __ldcg(&rc->p[p][0]);
      d1 = __ldcg(&rc->p[p][1]);
    } else {
      d0 = __ldcg(sa.desc + 2 * (pbase + p));
      d1 = __ldcg(sa.desc + 2 * (pbase + p) + 1);
    }
  };
  auto heads = [&](int uk, int& h0, int& nh) {
    const int kvh = uk / a.head_groups, hg = uk - kvh * a.head_groups;
    h0 = kvh * a.G + hg * 16;
    nh = min(16, a.G - hg * 16);
  };

  if (warp < NC) {
    // ================================ consumers ================================
    const int c = warp;
    const int g0 = lane >> 2, qd = lane & 3;
    const int nq = n > c ? (n - 1 - c) / NC + 1 : 0;  // this consumer's tiles: c + NC * q
    if (nq == 0 && np == 0) return;
    // pool rows: the first S from the record (row0), then batches of 32 (rb: rcur's batch)
    auto load_rows = [&](int batch) {
      const int q = batch * 32 + lane;
      return q < nq ? __ldcg(sa.rows + r0 + c + NC * q) : -1;
    };
    int rb = 0;
    int rcur = load_rows(0), rnext = load_rows(1);

    // current piece (cd), next (nd) with its query fragments (qn), the one after (fd)
    int4 cd0 = make_int4(0, 0, 0, 0), cd1 = cd0, nd0 = cd0, nd1 = cd0, fd0 = cd0, fd1 = cd0;
    uint32_t qa[KC][4], qn[KC][4];
    auto load_q = [&](const int4& d0, uint32_t(&dst)[KC][4]) {
      int h0, nh;
      heads(d0.y, h0, nh);
      load_q_frags<T, D>(a, d0.x, h0, nh, dst);
    };
    if (np > 0) {
      cd0 = p00;
      cd1 = p01;
      load_q(cd0, qa);
    }
    if (np > 1) {
      nd0 = p10;
      nd1 = p11;
      load_q(nd0, qn);
    }
    if (np > 2) piece(2, fd0, fd1);

    if (a.early_inputs) grid_dependency_wait();  // the cache is complete from here on
    if (c == 0 && lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
    }
    const uint64_t pol = l2_policy_evict_first();
    uint8_t* myring = ring + c * S * Geo::STAGE_BYTES;
    uint64_t* myfull = full + c * S;
    volatile int* mybad = stage_bad + c * S;
    const int W = (int)blockIdx.x * NC + c;
    // lane 0: start the loads of this consumer's tile q into its stage
    auto issue = [&](int q, int row) {
      const int st = q % S;
      mybad[st] = row < 0;
      if (W == a.hold_warp && q == a.hold_tile) return;  // test hook: the stage never completes
      const uint32_t bar = smem_u32(myfull + st);
      if (row < 0) {
        atomicOr(a.err, MVB_DEV_BLOCK_ID);
        mbar_arrive(bar);
        return;
      }
      mbar_arrive_expect_tx(bar, Geo::STAGE_BYTES);
      const uint32_t dk = smem_u32(myring + st * Geo::STAGE_BYTES);
#pragma unroll
      for (int p = 0; p < Geo::SUB; ++p) {
        tma_load_2d(dk + p * Geo::PANEL_BYTES, &tmk, p * 64, row, bar, pol);
        tma_load_2d(dk + Geo::TILE_BYTES + p * Geo::PANEL_BYTES, &tmv, p * 64, row, bar, pol);
      }
    };
    {
      const int n0 = nq < S ? nq : S;
      for (int q = 0; q < n0; ++q) {
        const int row = __shfl_sync(0xffffffffu, row0, q);
        if (lane == 0) issue(q, row);
      }
    }

    float o[NO][4];
#pragma unroll
    for (int nn = 0; nn < NO; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    // Hand this consumer's state for piece p to the merger (had: it holds tiles
    // of p); false when the CTA aborted.
    auto handoff = [&](int p, bool had) -> bool {
      const int b = NB == 1 ? 0 : (p & 1), use = NB == 1 ? p : (p >> 1);
      if (use > 0 &&
          !sched_wait_warp(smem_u32(mempty + b), (uint32_t)((use - 1) & 1), limit, abort_flag, a.err))
        return false;
      if (had) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
          lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
        }
        int h0, nh;
        heads(cd0.y, h0, nh);
        float* mo = merge + (int64_t)(b * NC + c) * mg * PR;
#pragma unroll
        for (int nn = 0; nn < NO; ++nn) {
          const int d = nn * 8 + 2 * qd;
          if (g0 < nh) *reinterpret_cast<float2*>(mo + g0 * PR + d) = make_float2(o[nn][0], o[nn][1]);
          if (g0 + 8 < nh) *reinterpret_cast<float2*>(mo + (g0 + 8) * PR + d) = make_float2(o[nn][2], o[nn][3]);
        }
        if (qd == 0) {
          if (g0 < nh) *reinterpret_cast<float2*>(mo + g0 * PR + D) = make_float2(mrow[0], lrow[0]);
          if (g0 + 8 < nh) *reinterpret_cast<float2*>(mo + (g0 + 8) * PR + D) = make_float2(mrow[1], lrow[1]);
        }
      }
      warp_arrive(smem_u32(mfull + b), lane);
#pragma unroll
      for (int nn = 0; nn < NO; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
      mrow[0] = mrow[1] = -INFINITY;
      lrow[0] = lrow[1] = 0.f;
      return true;
    };

    int p = 0;
    int vend = np > 0 ? cd1.x + cd0.w : 0;  // end of the current piece's positions
    bool had = false, failed = false;
    int q = 0;
    for (;; ++q) {
      const int j = q < nq ? c + NC * q : n;  // n, past the range: hand over every remaining piece
      while (p < np && j >= vend) {  // warp-uniform: the tile lies in a later piece
        if (!handoff(p, had)) {
          failed = true;
          break;
        }
        had = false;
        if (++p >= np) break;
        cd0 = nd0;
        cd1 = nd1;
#pragma unroll
        for (int kc = 0; kc < KC; ++kc)
#pragma unroll
          for (int e = 0; e < 4; ++e) qa[kc][e] = qn[kc][e];
        vend = cd1.x + cd0.w;
        nd0 = fd0;
        nd1 = fd1;
        if (p + 1 < np) load_q(nd0, qn);
        if (p + 2 < np) piece(p + 2, fd0, fd1);
      }
      if (failed || q >= nq) break;
      const int st = q % S;
      if (!sched_wait_warp(smem_u32(myfull + st), (uint32_t)((q / S) & 1), limit, abort_flag, a.err)) {
        failed = true;
        break;
      }
      if (!mybad[st]) {
        const int t = cd0.z + (j - cd1.x);  // tile of the unit
        const int valid = min(kTile, cd1.y - t * kTile);
        const uint32_t kb = smem_u32(myring + st * Geo::STAGE_BYTES);
        attend_tile<T, D>(kb, kb + Geo::TILE_BYTES, valid, a.scale_log2, qa, o, mrow, lrow);
      }
      had = true;
      __syncwarp();
      const int qi = q + S;
      if (qi < nq) {
        if ((qi >> 5) != rb) {
          rcur = rnext;
          ++rb;
          rnext = load_rows(rb + 1);
        }
        const int row = __shfl_sync(0xffffffffu, rcur, qi & 31);
        if (lane == 0) {
          fence_proxy_async_smem();  // V rows zeroed through the generic proxy before the next copy
          issue(qi, row);
        }
      }
    }
    if (!failed) return;
    // Aborted: wait (bounded, without the abort shortcut) for this consumer's
    // copies still in flight, so that none lands after the CTA has left.
    const int issued = nq < q + S ? nq : q + S;
    for (int jj = q; jj < issued; ++jj) {
      if (W == a.hold_warp && jj == a.hold_tile) continue;
      mbar_wait_bounded(smem_u32(myfull + jj % S), (uint32_t)((jj / S) & 1), limit);
    }
    return;
  }

  // ================================== merger ==================================
  // Lane l takes head row l / 4 (+ 8 for more than 8 heads) and column quarter
  // l % 4 (CQ = D / 4 columns).
  {
    constexpr int CQ = D / 4;
    const int rq = lane >> 2, cq = (lane & 3) * CQ;
    T* const outp = static_cast<T*>(a.out);
    grid_dependency_wait();  // the previous decode's counters, outputs and partial states
    const int n_bad = __ldcg(&sa.hdr->n_bad);
    if (blockIdx.x == 0 && lane == 0) {
      const int bb = __ldcg(&sa.hdr->bad_bits);
      if (bb) atomicOr(a.err, bb);
    }
    for (int i = blockIdx.x; i < n_bad; i += gridDim.x) {  // rows of the sequences left out: zeros
      T* o = outp + (int64_t)__ldcg(sa.bad + i) * a.o_s0;
      for (int e = lane; e < a.num_heads * D; e += 32) o[(int64_t)(e / D) * a.o_s1 + e % D] = from_f32<T>(0.f);
    }
    // Slot of CTA `cta`'s partial state of the cut unit of descriptor d1.
    auto cut_slot = [&](const int4& d1, int cta) {
      const int c0 = d1.z;
      return cta == c0 ? 2 * c0 + ((d1.w & 1) ? 0 : 1) : 2 * cta;
    };
    // Cut pieces (at most two, the CTA's first two) whose partial states are
    // stored: count them in on their units' counters, both in flight at once,
    // and merge the units they arrive last at, in CTA order (deterministic).
    // Each step is an L2 round trip (~2 us under a full DRAM stream): it runs
    // behind the first whole piece's merge, so the buffers keep draining.
    int npend = 0;
    int4 pa0 = make_int4(0, 0, 0, 0), pa1 = pa0, pb0 = pa0, pb1 = pa0;
    auto finish_cuts = [&]() {
      if (npend == 0) return;
      fence_acq_rel_gpu();  // this lane's partial stores are visible GPU-wide before the arrivals
      __syncwarp();
      int arr = 0;
      if (lane == 0) arr = atomicAdd(sa.ucnt + pa1.z, 1);
      if (lane == 1 && npend > 1) arr = atomicAdd(sa.ucnt + pb1.z, 1);
      const int arr_a = __shfl_sync(0xffffffffu, arr, 0), arr_b = __shfl_sync(0xffffffffu, arr, 1);
      const bool last_a = arr_a == (pa1.w >> 1) - 1, last_b = npend > 1 && arr_b == (pb1.w >> 1) - 1;
      npend = 0;
      if (!last_a && !last_b) return;
      fence_acq_rel_gpu();  // acquire side: the other CTAs' partials
#pragma unroll 1
      for (int k = 0; k < 2; ++k) {
        if (!(k == 0 ? last_a : last_b)) continue;
        const int4 d0 = k == 0 ? pa0 : pb0, d1 = k == 0 ? pa1 : pb1;
        const int seq = d0.x, c0 = d1.z, ncon = d1.w >> 1;
        int h0, nh;
        heads(d0.y, h0, nh);
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          const int r = rq + 8 * pass;
          if (r >= nh) continue;  // lane-divergent: no warp collectives below
          float M = -INFINITY, Lsum = 0.f, acc[CQ];
#pragma unroll
          for (int i = 0; i < CQ; ++i) acc[i] = 0.f;
          for (int i0 = 0; i0 < ncon; i0 += 4) {
            float2 ml[4];
            float4 ov[4][CQ / 4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const int i = i0 + t < ncon ? i0 + t : ncon - 1;
              const float* pp = sa.part + ((int64_t)cut_slot(d1, c0 + i) * mg + r) * PR;
              ml[t] = __ldcg(reinterpret_cast<const float2*>(pp + D));
#pragma unroll
              for (int v = 0; v < CQ / 4; ++v) ov[t][v] = __ldcg(reinterpret_cast<const float4*>(pp + cq) + v);
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              if (i0 + t >= ncon || ml[t].x == -INFINITY) continue;
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
          store_row(outp + (int64_t)seq * a.o_s0 + (int64_t)(h0 + r) * a.o_s1 + cq, acc,
                    Lsum > 0.f ? 1.f / Lsum : 0.f);
        }
        __syncwarp();
        if (lane == 0) sa.ucnt[c0] = 0;  // zero at rest for the next decode of this schedule
      }
    };
    // Piece descriptors reach the merger through a 4-slot shared-memory ring,
    // copied 4 pieces ahead with cp.async (lanes 0 and 1, one group per piece):
    // a load into registers would stall the warp at its first use (~1-2 us from
    // L2 under a full DRAM stream), and one call site of the merge keeps the
    // merger's code small (it runs a few times per kernel, from a cold
    // instruction cache).
    auto fetch = [&](int p) {
      if (p < np && lane < 2) {
        const int4* src = p < 2 ? &rc->p[p][lane] : sa.desc + 2 * (pbase + p) + lane;
        cp_async_16(smem_u32(dring + 2 * (p & 3) + lane), src);
      }
      cp_async_commit();
    };
#pragma unroll 1
    for (int p = 0; p < 4; ++p) fetch(p);
#pragma unroll 1
    for (int p = 0; p < np; ++p) {
      cp_async_wait_group<3>();  // piece p's group has landed
      __syncwarp();
      const int4 d0 = dring[2 * (p & 3)], d1 = dring[2 * (p & 3) + 1];
      __syncwarp();  // every lane has read the slot before it is refilled
      fetch(p + 4);
      const int b = NB == 1 ? 0 : (p & 1), use = NB == 1 ? p : (p >> 1);
      if (!sched_wait_warp(smem_u32(mfull + b), (uint32_t)(use & 1), limit, abort_flag, a.err)) return;
      int h0, nh;
      heads(d0.y, h0, nh);
      const float* mb = merge + (int64_t)b * NC * mg * PR;
      const int first = d1.x % NC;
      float M0, L0, O0[CQ], M1 = 0.f, L1 = 0.f, O1[CQ];
      merge_row<D, NC>(mb, mg, rq, cq, first, d0.w, rq < nh, M0, L0, O0);
      if (nh > 8) merge_row<D, NC>(mb, mg, rq + 8, cq, first, d0.w, rq + 8 < nh, M1, L1, O1);
      warp_arrive(smem_u32(mempty + b), lane);  // the states are in registers: the buffer is free
      if (d1.z < 0) {  // the whole unit
        T* po = outp + (int64_t)d0.x * a.o_s0 + (int64_t)h0 * a.o_s1 + cq;
        if (rq < nh) store_row(po + (int64_t)rq * a.o_s1, O0, L0 > 0.f ? 1.f / L0 : 0.f);
        if (rq + 8 < nh) store_row(po + (int64_t)(rq + 8) * a.o_s1, O1, L1 > 0.f ? 1.f / L1 : 0.f);
      } else {
        // a piece of a cut unit: store its partial state now; the arrival
        // waits for finish_cuts
        const int self = cut_slot(d1, (int)blockIdx.x);
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          const int r = rq + 8 * pass;
          if (r >= nh) continue;
          float* pp = sa.part + ((int64_t)self * mg + r) * PR;
          const float* src = pass == 0 ? O0 : O1;
          float4* dst = reinterpret_cast<float4*>(pp + cq);
#pragma unroll
          for (int i = 0; i < CQ / 4; ++i)
            dst[i] = make_float4(src[4 * i], src[4 * i + 1], src[4 * i + 2], src[4 * i + 3]);
          if ((lane & 3) == 0)
            *reinterpret_cast<float2*>(pp + D) = pass == 0 ? make_float2(M0, L0) : make_float2(M1, L1);
        }
        if (npend == 0) {
          pa0 = d0;
          pa1 = d1;
        } else {
          pb0 = d0;
          pb1 = d1;
        }
        ++npend;
      }
      if (p == 2) finish_cuts();  // behind the first whole piece
    }
    cp_async_wait_group<0>();
    finish_cuts();  // fewer than three pieces
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int sched_max_smem_per_block() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 232448;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0)
      v = 232448;
    cache[dev] = v;
  }
  return cache[dev];
}

static int sched_smem_for(int head_dim, int mg, int nb) {
  return 1024 + (head_dim == 64 ? SchedSmem<64>::bytes(mg, nb) : SchedSmem<128>::bytes(mg, nb));
}

SchedLayout sched_layout(int num_seqs, int num_kv_heads, int head_groups, int G, int max_blocks,
                         int block_size, int head_dim, int ctas) {
  SchedLayout l = {};
  const int64_t units = (int64_t)num_seqs * num_kv_heads * head_groups;
  const int64_t unit_tiles = ((int64_t)max_blocks * block_size + kTile - 1) / kTile;
  l.ctas = ctas;
  l.mg = G < 16 ? G : 16;
  l.max_tiles = units * unit_tiles;
  l.max_pieces = units + ctas;
  const int cap = sched_max_smem_per_block();
  l.nb = sched_smem_for(head_dim, l.mg, 2) <= cap ? 2 : sched_smem_for(head_dim, l.mg, 1) <= cap ? 1 : 0;
  l.ok = l.nb > 0 && num_seqs <= kSchedMaxSeqs && ctas >= 1 && ctas <= kSchedMaxCtas &&
         l.max_tiles < ((int64_t)1 << 31) - 1;
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  l.off_rec = 256;
  l.off_desc = l.off_rec + up((int64_t)ctas * 256);
  l.off_rows = l.off_desc + up(l.max_pieces * 32);
  l.off_bad = l.off_rows + up(l.max_tiles * 4);
  l.off_ucnt = l.off_bad + up((int64_t)num_seqs * 4);
  l.off_part = l.off_ucnt + up((int64_t)ctas * 4);
  l.bytes = l.off_part + up((int64_t)2 * ctas * l.mg * (head_dim + 4) * 4);
  return l;
}

int sched_smem_bytes(int head_dim, int mg, int nb) { return sched_smem_for(head_dim, mg, nb); }

cudaError_t launch_decode_schedule(const DecodeArgs& a, int head_dim, const SchedLayout& l, void* ws,
                                   bool wait_at_end, cudaStream_t stream) {
  char* w = static_cast<char*>(ws);
  auto kern = decode_schedule_kernel;
  const int smem = 2 * (a.num_seqs + 1) * 4;
  cudaError_t e = ensure_kernel_attrs(kern, smem);
  if (e != cudaSuccess) return e;
  const int nc = head_dim == 64 ? SchedConfig<64>::NC : SchedConfig<128>::NC;
  const int st = head_dim == 64 ? SchedConfig<64>::S : SchedConfig<128>::S;
  return launch_pdl(kern, dim3(l.ctas), dim3(kSchedBuildThreads), smem, stream, a.kv_len, a.bt, a.bt_s0,
                    a.num_seqs, a.num_kv_heads, a.head_groups, a.block_size, a.max_blocks, a.num_blocks, nc, st,
                    reinterpret_cast<SchedHeader*>(w), reinterpret_cast<SchedRec*>(w + l.off_rec),
                    reinterpret_cast<int4*>(w + l.off_desc), reinterpret_cast<int*>(w + l.off_rows),
                    reinterpret_cast<int*>(w + l.off_bad), reinterpret_cast<int*>(w + l.off_ucnt), a.err,
                    wait_at_end ? 1 : 0);
}

template <typename T, int D>
cudaError_t launch_sched_t(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                           const SchedLayout& l, void* ws, cudaStream_t stream) {
  auto kern = decode_sched_kernel<T, D>;
  const int smem = sched_smem_for(D, l.mg, l.nb);
  cudaError_t e = ensure_kernel_attrs(kern, smem);
  if (e != cudaSuccess) return e;
  char* w = static_cast<char*>(ws);
  SchedArgs sa;
  sa.hdr = reinterpret_cast<const SchedHeader*>(w);
  sa.rec = reinterpret_cast<const SchedRec*>(w + l.off_rec);
  sa.desc = reinterpret_cast<const int4*>(w + l.off_desc);
  sa.rows = reinterpret_cast<const int*>(w + l.off_rows);
  sa.bad = reinterpret_cast<const int*>(w + l.off_bad);
  sa.ucnt = reinterpret_cast<int*>(w + l.off_ucnt);
  sa.part = reinterpret_cast<float*>(w + l.off_part);
  sa.mg = l.mg;
  sa.nb = l.nb;
  return launch_pdl(kern, dim3(l.ctas), dim3(SchedSmem<D>::THREADS), smem, stream, tmk, tmv, a, sa);
}

cudaError_t launch_decode_sched(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a, int dtype,
                                int head_dim, const SchedLayout& l, void* ws, cudaStream_t stream) {
  if (dtype == MVB_DTYPE_BF16)
    return head_dim == 64 ? launch_sched_t<__nv_bfloat16, 64>(tmk, tmv, a, l, ws, stream)
                          : launch_sched_t<__nv_bfloat16, 128>(tmk, tmv, a, l, ws, stream);
  return head_dim == 64 ? launch_sched_t<__half, 64>(tmk, tmv, a, l, ws, stream)
                        : launch_sched_t<__half, 128>(tmk, tmv, a, l, ws, stream);
}

}  // namespace mvb
