// Tensor-core math of one 16-token KV tile, shared by the paged-decode kernels
// that stage K/V with TMA (decode_mma.cu, decode_stream.cu).
#pragma once

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

// Query fragments (A operand of S = Q K^T): rows = the (up to 16) query heads
// of one head group, zero padded past `nh`.
template <typename T, int D>
__device__ __forceinline__ void load_q_frags(const DecodeArgs& a, int seq, int h0, int nh,
                                             uint32_t (&qa)[D / 16][4]) {
  const int lane = threadIdx.x & 31;
  const int g0 = lane >> 2, qd = lane & 3;
  const T* qp = static_cast<const T*>(a.q) + seq * a.q_s0 + (int64_t)h0 * a.q_s1;
  const bool r0 = g0 < nh, r1 = g0 + 8 < nh;
#pragma unroll
  for (int kc = 0; kc < D / 16; ++kc) {
    const int d = kc * 16 + 2 * qd;
    qa[kc][0] = r0 ? ld_u32(qp + g0 * a.q_s1 + d) : 0u;
    qa[kc][1] = r1 ? ld_u32(qp + (g0 + 8) * a.q_s1 + d) : 0u;
    qa[kc][2] = r0 ? ld_u32(qp + g0 * a.q_s1 + d + 8) : 0u;
    qa[kc][3] = r1 ? ld_u32(qp + (g0 + 8) * a.q_s1 + d + 8) : 0u;
  }
}

// One 16-token tile of online-softmax attention for one warp.  `kb` / `vb` are
// the shared-memory addresses of the tile's swizzled K and V (16 x D each);
// `valid` (1..16) tokens are real.  Updates the warp's running state:
// o (16 x D accumulator fragments), mrow / lrow (running max and thread-partial
// sums of rows g0 and g0 + 8, in the exp2 domain).
template <typename T, int D>
__device__ __forceinline__ void attend_tile(uint32_t kb, uint32_t vb, int valid, float scale_log2,
                                            const uint32_t (&qa)[D / 16][4], float (&o)[D / 8][4],
                                            float (&mrow)[2], float (&lrow)[2]) {
  using MMA = Mma16816<T>;
  constexpr int KC = D / 16, NO = D / 8, PANEL = kTile * 128;
  const int lane = threadIdx.x & 31;
  const int qd = lane & 3;
  if (valid < kTile) {
    // rows past the context may hold any bits (torch.empty): zero the V rows so
    // 0 * NaN cannot reach the sum
    const int nchunk = (kTile - valid) * (D / 8);
    for (int e = lane; e < nchunk; e += 32) {
      const int r = valid + e / (D / 8), ch = e % (D / 8);
      st_shared_zero16(vb + (ch >> 3) * PANEL + r * 128 + (ch & 7) * 16);
    }
    __syncwarp();
  }
  // S = Q K^T : s0 holds tokens 0-7, s1 tokens 8-15 of the tile.
  float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kc = 0; kc < KC; ++kc) {
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
      x[r][k] = tk < valid ? x[r][k] * scale_log2 : -INFINITY;
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
    for (int n = 0; n < NO; ++n) {
      o[n][2 * r] *= al;
      o[n][2 * r + 1] *= al;
    }
  }
  // P enters the tensor core as a bf16/f16 pair: hi = round(p) and
  // lo = round(p - hi), so P V = hi V + lo V carries ~16 significant bits of P
  // instead of 8 (bf16); the two MMAs share the V fragments.
  uint32_t pa_hi[4], pa_lo[4];
  {
    float hi[2][4], lo[2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        hi[r][k] = MMA::round(p[r][k]);
        lo[r][k] = p[r][k] - hi[r][k];
      }
    pa_hi[0] = MMA::pack(hi[0][0], hi[0][1]);
    pa_hi[1] = MMA::pack(hi[1][0], hi[1][1]);
    pa_hi[2] = MMA::pack(hi[0][2], hi[0][3]);
    pa_hi[3] = MMA::pack(hi[1][2], hi[1][3]);
    pa_lo[0] = MMA::pack(lo[0][0], lo[0][1]);
    pa_lo[1] = MMA::pack(lo[1][0], lo[1][1]);
    pa_lo[2] = MMA::pack(lo[0][2], lo[0][3]);
    pa_lo[3] = MMA::pack(lo[1][2], lo[1][3]);
  }
  // O += P V
#pragma unroll
  for (int n = 0; n < NO; n += 2) {
    const int mi = lane >> 3;
    const int r = (lane & 7) + ((mi & 1) << 3);
    const int ch = n + (mi >> 1);
    uint32_t b0, b1, b2, b3;
    ldsm_x4_trans(vb + swz(r, ch), b0, b1, b2, b3);
    MMA::run(o[n], pa_hi, b0, b1);
    MMA::run(o[n + 1], pa_hi, b2, b3);
    MMA::run(o[n], pa_lo, b0, b1);
    MMA::run(o[n + 1], pa_lo, b2, b3);
  }
}

// attend_tile for rows with their own limits (causal prefill): row g0 of the
// tile (this thread's c0 / c1 values) sees tokens t < valid0, row g0 + 8 tokens
// t < valid1 (limits may be <= 0 or > 16).  The V rows are not zeroed: every
// row the producer did not fill is zero-filled by its copies, and a real row a
// limit masks gets weight 0.  Each row must see at least one token in the
// first tile it is given (its running max is then finite).
template <typename T, int D>
__device__ __forceinline__ void attend_tile_rows(uint32_t kb, uint32_t vb, int valid0, int valid1,
                                                 float scale_log2, const uint32_t (&qa)[D / 16][4],
                                                 float (&o)[D / 8][4], float (&mrow)[2], float (&lrow)[2]) {
  using MMA = Mma16816<T>;
  constexpr int KC = D / 16, NO = D / 8;
  const int lane = threadIdx.x & 31;
  const int qd = lane & 3;
  float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kc = 0; kc < KC; ++kc) {
    const int mi = lane >> 3;
    const int r = (lane & 7) + ((mi >> 1) << 3);
    const int ch = 2 * kc + (mi & 1);
    uint32_t b0, b1, b2, b3;
    ldsm_x4(kb + swz(r, ch), b0, b1, b2, b3);
    MMA::run(s0, qa[kc], b0, b1);
    MMA::run(s1, qa[kc], b2, b3);
  }
  float x[2][4] = {{s0[0], s0[1], s1[0], s1[1]}, {s0[2], s0[3], s1[2], s1[3]}};
  const int tk0 = 2 * qd;
  float p[2][4];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int lim = r == 0 ? valid0 : valid1;
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int tk = tk0 + (k & 1) + ((k >> 1) << 3);
      x[r][k] = tk < lim ? x[r][k] * scale_log2 : -INFINITY;
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
    for (int n = 0; n < NO; ++n) {
      o[n][2 * r] *= al;
      o[n][2 * r + 1] *= al;
    }
  }
  uint32_t pa_hi[4], pa_lo[4];
  {
    float hi[2][4], lo[2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        hi[r][k] = MMA::round(p[r][k]);
        lo[r][k] = p[r][k] - hi[r][k];
      }
    pa_hi[0] = MMA::pack(hi[0][0], hi[0][1]);
    pa_hi[1] = MMA::pack(hi[1][0], hi[1][1]);
    pa_hi[2] = MMA::pack(hi[0][2], hi[0][3]);
    pa_hi[3] = MMA::pack(hi[1][2], hi[1][3]);
    pa_lo[0] = MMA::pack(lo[0][0], lo[0][1]);
    pa_lo[1] = MMA::pack(lo[1][0], lo[1][1]);
    pa_lo[2] = MMA::pack(lo[0][2], lo[0][3]);
    pa_lo[3] = MMA::pack(lo[1][2], lo[1][3]);
  }
#pragma unroll
  for (int n = 0; n < NO; n += 2) {
    const int mi = lane >> 3;
    const int r = (lane & 7) + ((mi & 1) << 3);
    const int ch = n + (mi >> 1);
    uint32_t b0, b1, b2, b3;
    ldsm_x4_trans(vb + swz(r, ch), b0, b1, b2, b3);
    MMA::run(o[n], pa_hi, b0, b1);
    MMA::run(o[n + 1], pa_hi, b2, b3);
    MMA::run(o[n], pa_lo, b0, b1);
    MMA::run(o[n + 1], pa_lo, b2, b3);
  }
}

}  // namespace mvb
