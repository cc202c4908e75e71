// mvb_paged_gather: logical -> physical gather of cached K/V into contiguous
// [total_tokens, KH, D] tensors (the prefill path's prefix read).
//
// Replaces the reference's Triton _gather_prefix_kv_kernel and its wrapper
// gather_prefix_kv (mini_vllm/attention/paged_attention_gpu.py:329-433), whose
// index maps were built by a Python loop over every prefix token, and restates
// gather_paged_kv (mini_vllm/cache/cache_read.py:19-84) for a batch of
// sequences: out[off_i + p] = cache[block_table[row_i][p / BS], :, p % BS, :]
// for p < n_i, where n_i = out_offsets[i + 1] - out_offsets[i].
//
// It is an HBM copy (2 x read + 2 x write of T * KH * D elements) in two forms:
//  * the tile form (paged_gather_tma_kernel) for 2- or 4-byte elements, rows of
//    at most 512 bytes and block sizes that are multiples of 16: a 16-token
//    tile of one KV head is one contiguous run of the pool, so each warp moves
//    (sequence, tile, KV head) items through a ring of shared-memory stages --
//    two bulk copies in (K and V), two 3-D tensor-map stores out into the
//    head's strided rows -- with several items in flight per warp.  A
//    sequence's last, partial tile is stored by the warp's lanes so that it
//    never touches the next sequence's rows;
//  * the vector form (paged_gather_kernel) for every other layout: 16-byte
//    vectors, four per lane in flight, over a grid-stride loop.
// A token whose logical block lies past the table (IndexError in
// gather_paged_kv) or whose block id is outside [0, num_blocks) (-1 padding,
// where the Triton kernel left the output unwritten) gets zero rows and an
// error bit; so does a token that offsets which are not a prefix sum from 0
// to total_tokens leave without a sequence (the tile form checks the offsets
// first and runs the vector form's loop when they are not).
#include <cudaTypedefs.h>

#include "mvb_common.cuh"

namespace mvb {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

namespace {

struct GatherArgs {
  const uint4* kc;
  const uint4* vc;
  const int64_t* bt;
  int64_t bt_s0;
  int64_t bt_rows;
  int max_blocks;
  const int64_t* rows;     // [num_seqs] block-table row of each sequence
  const int64_t* offsets;  // [num_seqs + 1] exclusive prefix of the token counts
  uint4* ko;
  uint4* vo;
  int num_seqs;
  int64_t total_chunks;    // total_tokens * KH * CH
  int kh;
  int ch;                  // 16-byte chunks per (token, KV head) row
  int block_size;
  int num_blocks;
  int* err;
};

// Chunk c of the output is (token t, KV head, 16-byte chunk) with
// c = (t * KH + kvh) * CH + chunk.  A warp moves U * 32 consecutive chunks per
// step: it finds the sequence of its first token once (32-ary ballot search
// over the offsets), each lane steps forward only across sequence boundaries,
// and all U loads of K and V are in flight before the stores.  POW2: KH, CH and
// the block size are powers of two, so the index math is shifts and masks.
constexpr int kGatherUnroll = 4;

__device__ __forceinline__ int gather_find_sequence(const GatherArgs& a, int64_t t, int lane) {
  int lo = 0, hi = a.num_seqs;  // the last i with offsets[i] <= t (offsets[0] <= t assumed; checked later)
  while (hi - lo > 1) {
    const int step = (hi - lo + 31) >> 5;
    const int probe = lo + lane * step;
    const bool le = probe < hi && __ldg(a.offsets + probe) <= t;
    const unsigned m = __ballot_sync(0xffffffffu, le) | 1u;
    lo += (31 - __clz(m)) * step;
    hi = min(hi, lo + step);
  }
  return lo;
}

constexpr int kGatherCtasPerSm = 4;  // 256 threads x <= 64 registers

// The vector form's grid-stride loop over output chunks (any grid and block
// shape whose block size is a multiple of 32).
template <bool POW2>
__device__ __forceinline__ void gather_vector_loop(const GatherArgs& a) {
  constexpr int U = kGatherUnroll;
  const int lane = threadIdx.x & 31;
  const int per_token = a.kh * a.ch;
  const int sh_tok = POW2 ? __ffs(per_token) - 1 : 0, sh_ch = POW2 ? __ffs(a.ch) - 1 : 0;
  const int sh_bs = POW2 ? __ffs(a.block_size) - 1 : 0;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t step = (((int64_t)gridDim.x * blockDim.x) >> 5) * (U * 32);
  int bad = 0;
  // Source chunk of each of this lane's U output chunks in the step at `base`
  // (-1: a zero row).  Warp-uniform `base`: the search is warp-collective.
  auto resolve = [&](int64_t base, int64_t (&src)[U]) {
    const int64_t t0 = POW2 ? (base >> sh_tok) : base / per_token;
    const int s0 = gather_find_sequence(a, t0, lane);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      src[u] = -1;
      const int64_t c = base + u * 32 + lane;
      if (c >= a.total_chunks) continue;
      const int r = (int)(c - t0 * per_token);  // < U * 32 + per_token
      const int dt = POW2 ? (r >> sh_tok) : r / per_token;
      const int rem = r - dt * per_token;
      const int kvh = POW2 ? (rem >> sh_ch) : rem / a.ch;
      const int chunk = rem - kvh * a.ch;
      const int64_t t = t0 + dt;
      int s = s0;
      while (s + 1 < a.num_seqs && t >= __ldg(a.offsets + s + 1)) ++s;
      const int64_t o0 = __ldg(a.offsets + s);
      const int64_t row = __ldg(a.rows + s);
      if (t < o0 || t >= __ldg(a.offsets + s + 1)) {
        bad |= MVB_DEV_KV_LEN;  // offsets are not an increasing prefix starting at 0
        continue;
      }
      if (row < 0 || row >= a.bt_rows) {
        bad |= MVB_DEV_BLOCK_ID;
        continue;
      }
      const int p = (int)(t - o0);  // a position inside one sequence
      const int blk = POW2 ? (p >> sh_bs) : p / a.block_size;
      if (blk >= a.max_blocks) {
        bad |= MVB_DEV_TABLE_SHORT;
        continue;
      }
      const int64_t bid = __ldg(a.bt + row * a.bt_s0 + blk);
      if (bid < 0 || bid >= a.num_blocks) {
        bad |= MVB_DEV_BLOCK_ID;
        continue;
      }
      src[u] = ((bid * a.kh + kvh) * a.block_size + (p - blk * a.block_size)) * a.ch + chunk;
    }
  };
  // Software pipeline: the next step's addresses are resolved (its metadata
  // loads in flight) while this step's K/V loads are in flight.
  int64_t base = warp0 * (U * 32);
  int64_t cur[U];
  if (base < a.total_chunks) resolve(base, cur);
  for (; base < a.total_chunks; base += step) {
    uint4 kv[U], vv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      kv[u] = make_uint4(0, 0, 0, 0);
      vv[u] = make_uint4(0, 0, 0, 0);
      if (cur[u] >= 0) {  // read once: streaming (evict-first) loads
        kv[u] = __ldcs(a.kc + cur[u]);
        vv[u] = __ldcs(a.vc + cur[u]);
      }
    }
    const int64_t next = base + step;
    if (next < a.total_chunks) resolve(next, cur);  // cur is free once the loads are issued
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = base + u * 32 + lane;
      if (c < a.total_chunks) {  // streaming stores: the outputs are consumed by the next kernel
        __stcs(a.ko + c, kv[u]);
        __stcs(a.vo + c, vv[u]);
      }
    }
  }
  if (bad) atomicOr(a.err, bad);
}

template <bool POW2>
__global__ void __launch_bounds__(256, kGatherCtasPerSm) paged_gather_kernel(const GatherArgs a) {
  grid_dependency_wait();  // the cache may have been written by the previous kernel
  grid_launch_dependents();
  gather_vector_loop<POW2>(a);
}

// ---- tile form ---------------------------------------------------------------
// Items: (sequence s, 16-token tile j, group of KHB KV heads).  Sequence s owns
// the virtual tile indices [vstart(s), vstart(s) + ceil(n_s / 16)) with
// vstart(s) = floor(off_s / 16) + s, an increasing map whose ranges never
// overlap (floor((off_s + n_s) / 16) + 1 >= floor(off_s / 16) + ceil(n_s / 16)),
// so there are V = floor(T / 16) + S virtual tiles, at most S of them empty,
// and V * (KH / KHB) items, head group fastest.  Each warp owns one contiguous
// range of items; it resolves 32 of them at a time (one per lane) and feeds
// them through its ring of stages in order.  A stage holds the item's K and V
// tiles as [KHB][16][D]: one 4-D tensor load per tile from the pool (dims D,
// BS, KH, NB) and one 3-D tensor store per tile into the output viewed with
// dims (D, T, KH), whose box {D, 16, KHB} has the same shared-memory layout.
//
// The MVB_GATHER_* macros are build-time tuning knobs; their defaults are the
// best of the measured settings (ring depth and size, static share, ticket
// size) on the config-2 contexts.
#ifndef MVB_GATHER_TMA_STAGES
#define MVB_GATHER_TMA_STAGES 4
#endif
#ifndef MVB_GATHER_TMA_RING_BYTES
#define MVB_GATHER_TMA_RING_BYTES (64 * 1024)
#endif
#ifndef MVB_GATHER_TMA_STAGE_MAX
#define MVB_GATHER_TMA_STAGE_MAX (16 * 1024)
#endif
#ifndef MVB_GATHER_STATIC_PCT
#define MVB_GATHER_STATIC_PCT 50
#endif
#ifndef MVB_GATHER_CHUNK
#define MVB_GATHER_CHUNK 2
#endif
constexpr int kStaticPct = MVB_GATHER_STATIC_PCT;  // share of the items split statically when balancing
constexpr int kDynChunk = MVB_GATHER_CHUNK;        // items per counter ticket
constexpr int kTmaStages = MVB_GATHER_TMA_STAGES;         // per warp; kTmaStages - 1 items in flight
constexpr int kTmaRingBytes = MVB_GATHER_TMA_RING_BYTES;  // stage bytes of one CTA (all its warps)
constexpr int kTmaStageMax = MVB_GATHER_TMA_STAGE_MAX;    // K + V bytes of one item, at most
constexpr int kTmaTile = 16;                              // tokens per tile
constexpr int kTmaMaxWarps = 4;
constexpr int kItemFull = 1, kItemPartial = 2, kItemBad = 3;

struct GatherTmaArgs {
  GatherArgs g;
  int64_t total_tokens;
  int64_t total_items;    // V * groups
  int64_t items_per_warp; // static items of each warp
  int64_t dyn_start;      // first item handed out by the counter (total_items: no counter)
  uint32_t* counter;      // [next ticket, finished warps], zero on entry and on exit; or nullptr
  int row_bytes;          // R = head_dim * element size
  int khb;                // KV heads per item
  int groups;             // KH / khb
  int warps;              // warps per CTA
  int stage_off;          // byte offset of the first stage in dynamic shared memory
};

// Per-stage record, written by lane 0 when it issues the stage's loads.
struct StageMeta {
  int64_t z;   // first output token
  int hg;      // head group
  int code;    // tokens | kind << 8
  int group;   // lane 0's bulk-group count after this stage's stores (0: none)
  int pad;
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int x, int y, int z, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's bulk groups still read shared memory.
template <int N> __device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kTmaMaxWarps * 32)
    paged_gather_tma_kernel(const __grid_constant__ CUtensorMap kpool, const __grid_constant__ CUtensorMap vpool,
                            const __grid_constant__ CUtensorMap kout, const __grid_constant__ CUtensorMap vout,
                            const GatherTmaArgs t) {
  grid_dependency_wait();  // the cache (and the offsets) may come from the previous kernel
  grid_launch_dependents();
  const GatherArgs& a = t.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The item map needs offsets that rise from 0 to total_tokens; other offsets
  // take the vector form's per-token loop (zero rows and MVB_DEV_KV_LEN for
  // tokens without a sequence).  Every warp checks all offsets itself, 256 per
  // round of independent loads, so all warps of the grid take the same path.
  {
    bool bad_offsets = false;
    int64_t carry = 0;  // offsets[base - 1]
    for (int base = 0; base <= a.num_seqs; base += 256) {
      int64_t o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = base + k * 32 + lane;
        o[k] = i <= a.num_seqs ? __ldg(a.offsets + i) : 0;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = base + k * 32 + lane;
        const int64_t up = __shfl_up_sync(0xffffffffu, o[k], 1);
        const int64_t prev = lane > 0 ? up : carry;
        carry = __shfl_sync(0xffffffffu, o[k], 31);
        if (i <= a.num_seqs && (i == 0 ? o[k] != 0 : o[k] < prev)) bad_offsets = true;
        if (i == a.num_seqs && o[k] != t.total_tokens) bad_offsets = true;
      }
    }
    if (__any_sync(0xffffffffu, bad_offsets)) {
      gather_vector_loop<false>(a);
      return;
    }
  }
  extern __shared__ __align__(128) unsigned char smem[];
  auto vstart = [&](int i) -> int64_t { return (__ldg(a.offsets + i) >> 4) + i; };
  constexpr int S = kTmaStages;
  const int R = t.row_bytes, khb = t.khb;
  const uint32_t tile_bytes = (uint32_t)kTmaTile * R * khb, stage_bytes = 2 * tile_bytes;  // K tile, V tile
  const uint32_t bar0 = smem_u32(smem) + warp * S * 8;
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + t.warps * S * 8) + warp * S;
  const uint32_t ring = smem_u32(smem + t.stage_off) + (uint32_t)warp * S * stage_bytes;
  if (lane == 0) {
    for (int i = 0; i < S; ++i) mbar_init(bar0 + 8 * i, 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int64_t gw = (int64_t)blockIdx.x * t.warps + warp;
  const int64_t i0 = gw * t.items_per_warp;
  const int64_t i1 = min(i0 + t.items_per_warp, min(t.dyn_start, t.total_items));
  const uint64_t policy = l2_policy_evict_first();
  const int ch = R >> 4;  // 16-byte chunks per row
  int issued = 0, consumed = 0, groups = 0, bad = 0;
  bool ok = true;

  // Store the oldest item out of its stage (all lanes).
  auto consume = [&]() {
    const int st = consumed % S;
    const bool landed = mbar_wait_bounded(bar0 + 8 * st, (uint32_t)(consumed / S) & 1u);
    if (!__all_sync(0xffffffffu, landed)) {
      ok = false;
      return;
    }
    const StageMeta m = meta[st];
    const int kind = (m.code >> 8) & 3, n_tok = m.code & 0xff;
    const uint32_t ks = ring + st * stage_bytes, vs = ks + tile_bytes;
    if (kind == kItemFull) {
      if (lane == 0) {
        // coordinates (x, token, first head) of the (D, T, KH) view, or
        // (x, head, token) of the natural view that one-head items use
        const int y = khb == 1 ? m.hg : (int)m.z, zc = khb == 1 ? (int)m.z : m.hg * khb;
        tma_store_3d(&kout, 0, y, zc, ks);
        tma_store_3d(&vout, 0, y, zc, vs);
        bulk_commit();
        meta[st].group = ++groups;
      }
    } else {  // a partial tile (rows < n_tok from shared memory) or a bad one (zero rows)
      for (int c = lane; c < khb * n_tok * ch; c += 32) {
        const int hr = c / ch, k = c - hr * ch;
        const int h = hr / n_tok, r = hr - h * n_tok;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (kind == kItemPartial) {
          const uint32_t off = (uint32_t)((h * kTmaTile + r) * R + k * 16);
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(kv.x), "=r"(kv.y), "=r"(kv.z), "=r"(kv.w)
                       : "r"(ks + off));
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(vv.x), "=r"(vv.y), "=r"(vv.z), "=r"(vv.w)
                       : "r"(vs + off));
        }
        const int64_t o = ((m.z + r) * a.kh + m.hg * khb + h) * ch + k;
        a.ko[o] = kv;
        a.vo[o] = vv;
      }
      if (lane == 0) meta[st].group = 0;
    }
    __syncwarp();
    ++consumed;
  };

  // Load one item into the next stage (lane 0 issues).
  auto issue = [&](int bid, int r0, int64_t z, int hg, int code) {
    const int st = issued % S;
    if (lane == 0) {
      if (issued >= S) {
        // The stage's previous stores must have finished reading it; the
        // fence orders the lanes' earlier reads of it before the new copies.
        const int g = meta[st].group;
        if (g != 0) {
          if (groups - g >= 1)
            bulk_wait_read<1>();
          else
            bulk_wait_read<0>();
        }
        fence_proxy_async_smem();
      }
      meta[st].z = z;
      meta[st].hg = hg;
      meta[st].code = code;
      const uint32_t bar = bar0 + 8 * st, ks = ring + st * stage_bytes;
      if (((code >> 8) & 3) == kItemBad) {
        mbar_arrive(bar);
      } else {
        mbar_arrive_expect_tx(bar, stage_bytes);
        tma_load_4d(ks, &kpool, 0, r0, hg * khb, bid, bar, policy);
        tma_load_4d(ks + tile_bytes, &vpool, 0, r0, hg * khb, bid, bar, policy);
      }
    }
    __syncwarp();
    ++issued;
  };

  // Batches: the warp's static range, 32 items at a time, then (with a
  // counter) kDynChunk items per ticket until the tickets run past the items,
  // so SMs that get more bandwidth take more of the tail.  Lane 0 asks for
  // the next ticket one batch ahead.
  uint32_t ticket = 0;
  auto grab = [&]() {
    if (lane == 0) ticket = atomicAdd(t.counter, 1u);
  };
  int64_t cursor = i0;
  if (t.counter != nullptr && cursor >= i1) grab();
  while (ok) {
    int64_t base, end;
    if (cursor < i1) {
      base = cursor;
      end = min(cursor + 32, i1);
      cursor = end;
      if (t.counter != nullptr && cursor >= i1) grab();
    } else if (t.counter != nullptr) {
      base = t.dyn_start + (int64_t)__shfl_sync(0xffffffffu, ticket, 0) * kDynChunk;
      if (base >= t.total_items) break;
      end = min(base + kDynChunk, t.total_items);
      grab();
    } else {
      break;
    }
    // Resolve item base + lane.  s0: the sequence of the batch's first tile
    // (32-ary ballot search over vstart); lane L's tile lies at most 31
    // sequences further, counted against vstart(s0 + 1 .. s0 + 32).
    const int64_t w = base + lane;
    const bool in = w < end;
    const int64_t vfirst = base / t.groups;
    int lo = 0, hi = a.num_seqs;
    while (hi - lo > 1) {
      const int step = (hi - lo + 31) >> 5;
      const int probe = lo + lane * step;
      const bool le = probe < hi && vstart(probe) <= vfirst;
      const unsigned msk = __ballot_sync(0xffffffffu, le) | 1u;
      lo += (31 - __clz(msk)) * step;
      hi = min(hi, lo + step);
    }
    const int64_t v = (in ? w : base) / t.groups;
    const int hg = (int)((in ? w : base) - v * t.groups);
    const int sn = lo + 1 + lane;
    const int64_t next_start = sn < a.num_seqs ? vstart(sn) : INT64_MAX;
    int s = lo;
#pragma unroll
    for (int i = 0; i < 32; ++i) s += __shfl_sync(0xffffffffu, next_start, i) <= v ? 1 : 0;
    int64_t z = 0;
    int bid = 0, r0 = 0, code = 0;
    if (in) {
      const int64_t o = __ldg(a.offsets + s), n = __ldg(a.offsets + s + 1) - o;
      const int64_t p0 = (v - ((o >> 4) + s)) * kTmaTile;
      if (p0 < n) {
        const int n_tok = (int)min((int64_t)kTmaTile, n - p0);
        z = o + p0;
        int err = 0;
        const int64_t row = __ldg(a.rows + s);
        const int64_t blk = p0 / a.block_size;
        if (row < 0 || row >= a.bt_rows) {
          err = MVB_DEV_BLOCK_ID;
        } else if (blk >= a.max_blocks) {
          err = MVB_DEV_TABLE_SHORT;
        } else {
          const int64_t b = __ldg(a.bt + row * a.bt_s0 + blk);
          if (b < 0 || b >= a.num_blocks) {
            err = MVB_DEV_BLOCK_ID;
          } else {
            bid = (int)b;
            r0 = (int)(p0 - blk * a.block_size);
          }
        }
        bad |= err;
        code = n_tok | ((err ? kItemBad : n_tok == kTmaTile ? kItemFull : kItemPartial) << 8);
      }
    }
    unsigned todo = __ballot_sync(0xffffffffu, code != 0);
    while (todo != 0 && ok) {
      const int from = __ffs(todo) - 1;
      todo &= todo - 1;
      const int ibid = __shfl_sync(0xffffffffu, bid, from);
      const int ir0 = __shfl_sync(0xffffffffu, r0, from);
      const int64_t iz = __shfl_sync(0xffffffffu, z, from);
      const int ihg = __shfl_sync(0xffffffffu, hg, from);
      const int icode = __shfl_sync(0xffffffffu, code, from);
      while (ok && consumed < issued - S + 2) consume();
      if (ok) issue(ibid, ir0, iz, ihg, icode);
    }
  }
  while (ok && consumed < issued) consume();
  if (!ok) {
    // A copy never completed: report it and wait (bounded) for the copies
    // still in flight into this warp's stages before the CTA exits.
    if (lane == 0) atomicOr(a.err, MVB_DEV_TIMEOUT);
    for (int c = consumed; c < issued; ++c) mbar_wait_bounded(bar0 + 8 * (c % S), (uint32_t)(c / S) & 1u);
  }
  if (lane == 0) bulk_wait_read<0>();
  if (bad) atomicOr(a.err, bad);
  if (t.counter != nullptr && lane == 0) {
    // The last warp to finish puts both words back to zero for the next call;
    // every warp's last ticket request is ordered before its count.
    __threadfence();
    const uint32_t done = atomicAdd(t.counter + 1, 1u);
    if (done == (uint32_t)gridDim.x * t.warps - 1) {
      atomicExch(t.counter, 0u);
      atomicExch(t.counter + 1, 0u);
    }
  }
}

int64_t round_up_128(int64_t v) { return (v + 127) / 128 * 128; }

// Tensor map of one pool [NB, KH, BS, D] (innermost first: D, BS, KH, NB)
// whose box {D, 16, khb, 1} is one item's K or V tile: [khb][16][D] in shared
// memory.  Elements are moved as raw 2- or 4-byte words.
bool gather_pool_map(const void* base, int nb, int kh, int bs, int head_dim, int es, int khb, CUtensorMap* out) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)bs, (cuuint64_t)kh, (cuuint64_t)nb};
  const cuuint64_t strides[3] = {(cuuint64_t)head_dim * es, (cuuint64_t)bs * head_dim * es,
                                 (cuuint64_t)kh * bs * head_dim * es};
  const cuuint32_t box[4] = {(cuuint32_t)head_dim, (cuuint32_t)kTmaTile, (cuuint32_t)khb, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(out, es == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 4,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of one gather output [T, KH, D] viewed with dims (D, T, KH)
// (strides KH * D and D elements), whose box {D, 16, khb} has the layout of a
// stage's tile, [khb][16][D]; with khb = 1 the dims are the natural (D, KH, T)
// and the box {D, 1, 16}, the same layout.
bool gather_out_map(void* base, int64_t tokens, int kh, int head_dim, int es, int khb, CUtensorMap* out) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t row = (cuuint64_t)head_dim * es;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  if (khb == 1) {
    dims[0] = head_dim, dims[1] = kh, dims[2] = tokens;
    strides[0] = row, strides[1] = row * kh;
    box[0] = head_dim, box[1] = 1, box[2] = kTmaTile;
  } else {
    dims[0] = head_dim, dims[1] = tokens, dims[2] = kh;
    strides[0] = row * kh, strides[1] = row;
    box[0] = head_dim, box[1] = kTmaTile, box[2] = khb;
  }
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(out, es == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, base, dims,
            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Resident CTAs per SM of the tile form at one launch shape (cached per device).
int tma_ctas_per_sm(int dev, int warps, int smem) {
  static std::mutex mu;
  static int cache_dev[16], cache_warps[16], cache_smem[16], cache_n[16], count = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < count; ++i)
    if (cache_dev[i] == dev && cache_warps[i] == warps && cache_smem[i] == smem) return cache_n[i];
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, paged_gather_tma_kernel, warps * 32, smem) != cudaSuccess)
    return 0;
  if (count < 16) {
    cache_dev[count] = dev;
    cache_warps[count] = warps;
    cache_smem[count] = smem;
    cache_n[count] = n;
    ++count;
  }
  return n;
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int mvb_paged_gather(const void* key_cache, const void* value_cache, const int64_t* block_table,
                                int64_t block_table_rows, int64_t block_table_stride, int32_t max_blocks_per_seq,
                                const int64_t* seq_rows,
                                const int64_t* out_offsets, void* key_out, void* value_out, int32_t num_seqs,
                                int64_t total_tokens, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                int32_t num_blocks, int32_t dtype, uint32_t* work_counter, int32_t* error_flags,
                                void* stream) {
  mvb::NvtxRange nvtx_range("mvb_paged_gather");
  if (dtype != MVB_DTYPE_F32 && dtype != MVB_DTYPE_F16 && dtype != MVB_DTYPE_BF16) return MVB_ERR_DTYPE;
  if (head_dim <= 0) return MVB_ERR_HEAD_DIM;
  if (block_size <= 0) return MVB_ERR_BLOCK_SIZE;
  if (num_seqs < 0 || total_tokens < 0 || num_kv_heads <= 0 || num_blocks <= 0 || max_blocks_per_seq < 0 ||
      block_table_rows < 0)
    return MVB_ERR_INVALID_ARG;
  if (total_tokens == 0 || num_seqs == 0) return MVB_OK;
  if (!key_cache || !value_cache || !block_table || !seq_rows || !out_offsets || !key_out || !value_out ||
      !error_flags)
    return MVB_ERR_INVALID_ARG;
  if (max_blocks_per_seq > 0 && block_table_stride < max_blocks_per_seq) return MVB_ERR_INVALID_ARG;
  const int64_t row_bytes = (int64_t)head_dim * (dtype == MVB_DTYPE_F32 ? 4 : 2);
  if (row_bytes % 16 != 0) return MVB_ERR_HEAD_DIM;  // rows move as 16-byte vectors
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!aligned(key_cache) || !aligned(value_cache) || !aligned(key_out) || !aligned(value_out) ||
      (reinterpret_cast<uintptr_t>(work_counter) & 3) != 0)
    return MVB_ERR_ALIGNMENT;

  GatherArgs a;
  a.kc = static_cast<const uint4*>(key_cache);
  a.vc = static_cast<const uint4*>(value_cache);
  a.bt = block_table;
  a.bt_s0 = block_table_stride;
  a.bt_rows = block_table_rows;
  a.max_blocks = max_blocks_per_seq;
  a.rows = seq_rows;
  a.offsets = out_offsets;
  a.ko = static_cast<uint4*>(key_out);
  a.vo = static_cast<uint4*>(value_out);
  a.num_seqs = num_seqs;
  a.kh = num_kv_heads;
  a.ch = (int)(row_bytes / 16);
  a.total_chunks = total_tokens * num_kv_heads * a.ch;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.err = error_flags;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);

  const int es = dtype == MVB_DTYPE_F32 ? 4 : 2;
  if (row_bytes <= 512 && block_size % kTmaTile == 0 && total_tokens < ((int64_t)1 << 31)) {
    // Heads per item: the most that divide KH and keep one item's K + V
    // within kTmaStageMax bytes; one head when the grouped maps do not encode.
    int khb = num_kv_heads;
    while (khb > 1 && (num_kv_heads % khb != 0 || 2 * kTmaTile * row_bytes * khb > kTmaStageMax)) --khb;
    CUtensorMap maps[4];
    auto encode = [&](int h) {
      return gather_pool_map(key_cache, num_blocks, num_kv_heads, block_size, head_dim, es, h, &maps[0]) &&
             gather_pool_map(value_cache, num_blocks, num_kv_heads, block_size, head_dim, es, h, &maps[1]) &&
             gather_out_map(key_out, total_tokens, num_kv_heads, head_dim, es, h, &maps[2]) &&
             gather_out_map(value_out, total_tokens, num_kv_heads, head_dim, es, h, &maps[3]);
    };
    bool have = encode(khb);
    if (!have && khb > 1) have = encode(khb = 1);
    if (have) {
      GatherTmaArgs t;
      t.g = a;
      t.total_tokens = total_tokens;
      t.row_bytes = (int)row_bytes;
      t.khb = khb;
      t.groups = num_kv_heads / t.khb;
      const int stage_bytes = 2 * kTmaTile * (int)row_bytes * t.khb;
      int warps = kTmaRingBytes / (kTmaStages * stage_bytes);
      warps = warps < 1 ? 1 : warps > kTmaMaxWarps ? kTmaMaxWarps : warps;
      t.warps = warps;
      t.stage_off = (int)round_up_128(warps * kTmaStages * (8 + (int)sizeof(StageMeta)));
      const int smem = t.stage_off + warps * kTmaStages * stage_bytes;
      if (ensure_kernel_attrs(paged_gather_tma_kernel, smem) != cudaSuccess) return MVB_ERR_CUDA;
      const int per_sm = tma_ctas_per_sm(dev, warps, smem);
      if (per_sm <= 0) return MVB_ERR_CUDA;
      t.total_items = (total_tokens / kTmaTile + num_seqs) * (int64_t)t.groups;
      const int64_t want = (t.total_items + warps - 1) / warps, cap = (int64_t)sms * per_sm;
      const int64_t grid = want < cap ? want : cap;
      const int64_t all_warps = grid * warps;
      t.counter = work_counter;
      if (work_counter != nullptr) {  // a static share, then tickets
        t.items_per_warp = t.total_items * kStaticPct / 100 / all_warps;
        t.dyn_start = t.items_per_warp * all_warps;
      } else {
        t.items_per_warp = (t.total_items + all_warps - 1) / all_warps;
        t.dyn_start = t.total_items;
      }
      const cudaError_t e = launch_pdl(paged_gather_tma_kernel, dim3((unsigned)grid), dim3(warps * 32), smem, st,
                                       maps[0], maps[1], maps[2], maps[3], t);
      return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
    }
  }

  auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
  const bool p2 = pow2(a.kh) && pow2(a.ch) && pow2(a.block_size);
  auto kern = p2 ? paged_gather_kernel<true> : paged_gather_kernel<false>;
  cudaError_t e = ensure_kernel_attrs(kern, 0);
  if (e != cudaSuccess) return MVB_ERR_CUDA;
  const int64_t per_cta = 256 * kGatherUnroll;
  const int64_t want = (a.total_chunks + per_cta - 1) / per_cta;
  const int64_t cap = (int64_t)sms * kGatherCtasPerSm;  // one wave of resident CTAs
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  e = launch_pdl(kern, dim3(grid), dim3(256), 0, st, a);
  return e == cudaSuccess ? MVB_OK : MVB_ERR_CUDA;
}
