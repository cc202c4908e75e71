/*
 * CPU oracle for mini-vLLM's paged KV write, paged KV gather and paged decode
 * attention — TEST INFRASTRUCTURE ONLY.
 *
 * This is a restatement, in plain C with OpenMP, of the reference's torch CPU
 * path.  It is the checker the parity tests compare the CUDA kernels against
 * and the CPU baseline bench.py times; the product (libmvb200.so and the
 * mini_vllm_b200 package) never links, loads or calls it.
 *
 *   oracle_cache_write  <- write_to_paged_cache   (mini_vllm/cache/cache_write.py:25-74)
 *   oracle_gather       <- gather_paged_kv        (mini_vllm/cache/cache_read.py:19-84)
 *   oracle_decode       <- AttentionBackendRef.decode_attention
 *                          (mini_vllm/attention/paged_attention_ref.py:102-161), whose
 *                          math is torch.nn.functional.scaled_dot_product_attention
 *                          (torch 2.11, math path: softmax(q k^T * scale) v).
 *
 * Storage types: 0 = float32, 1 = float16 (IEEE binary16), 2 = bfloat16; all
 * arithmetic of the decode runs in double on the upcast values, so the result
 * is at least as accurate as an fp32-accumulated reference.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_F32 0
#define ORACLE_F16 1
#define ORACLE_BF16 2

/* decode status codes */
#define ORACLE_OK 0
#define ORACLE_KV_LEN 1      /* kv_len < 1 (the GPU path raises ValueError)       */
#define ORACLE_TABLE_SHORT 2 /* table (after dropping -1) too short: IndexError   */
#define ORACLE_BLOCK_ID 3    /* block id < -1 or >= num_blocks: IndexError        */

static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1f;
  const uint32_t man = h & 0x3ff;
  float v;
  if (exp == 0) {
    v = ldexpf((float)man, -24); /* subnormal or zero */
  } else if (exp == 31) {
    v = man ? NAN : INFINITY;
  } else {
    v = ldexpf((float)(man | 0x400), (int)exp - 25);
  }
  uint32_t bits;
  memcpy(&bits, &v, 4);
  bits |= sign;
  memcpy(&v, &bits, 4);
  return v;
}

static float bf16_to_f32(uint16_t b) {
  const uint32_t bits = (uint32_t)b << 16;
  float v;
  memcpy(&v, &bits, 4);
  return v;
}

static double load(const void* base, int64_t i, int dtype) {
  if (dtype == ORACLE_F32) return ((const float*)base)[i];
  if (dtype == ORACLE_F16) return f16_to_f32(((const uint16_t*)base)[i]);
  return bf16_to_f32(((const uint16_t*)base)[i]);
}

static int elem_size(int dtype) { return dtype == ORACLE_F32 ? 4 : 2; }

/*
 * Sequential scatter, last writer wins (cache_write.py:55-74).  key/value are
 * contiguous [T][KH][D]; caches [NB][KH][BS][D].  Returns 0, or -(t+1) for the
 * first token t whose slot is neither -1 nor in [0, NB*BS) — tokens before it
 * have been written, as in the reference loop that raises IndexError there.
 */
int oracle_cache_write(const void* key, const void* value, void* kc, void* vc,
                       const int64_t* slots, int64_t T, int KH, int D, int BS, int64_t NB,
                       int dtype) {
  const int es = elem_size(dtype);
  const int64_t row = (int64_t)D * es;
  const int64_t total = NB * BS;
  for (int64_t t = 0; t < T; ++t) {
    const int64_t slot = slots[t];
    if (slot == -1) continue;
    if (slot < -1 || slot >= total) return (int)-(t + 1);
    const int64_t blk = slot / BS, off = slot % BS;
    for (int h = 0; h < KH; ++h) {
      const int64_t src = (t * KH + h) * row;
      const int64_t dst = ((blk * KH + h) * BS + off) * row;
      memcpy((char*)kc + dst, (const char*)key + src, (size_t)row);
      memcpy((char*)vc + dst, (const char*)value + src, (size_t)row);
    }
  }
  return 0;
}

/*
 * Logical-to-physical gather (cache_read.py:40-84): tokens 0..num_tokens-1 come
 * from table[0], table[1], ... block_size at a time.  out_k/out_v are
 * [num_tokens][KH][D] in the storage type.  Returns 0, or ORACLE_TABLE_SHORT
 * when the table does not cover num_tokens.
 */
int oracle_gather(const void* kc, const void* vc, const int64_t* table, int64_t table_len,
                  int64_t num_tokens, int KH, int D, int BS, int dtype, void* out_k,
                  void* out_v) {
  const int es = elem_size(dtype);
  const int64_t row = (int64_t)D * es;
  if ((num_tokens + BS - 1) / BS > table_len) return ORACLE_TABLE_SHORT;
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t blk = table[t / BS], off = t % BS;
    for (int h = 0; h < KH; ++h) {
      const int64_t src = ((blk * KH + h) * BS + off) * row;
      const int64_t dst = (t * KH + h) * row;
      memcpy((char*)out_k + dst, (const char*)kc + src, (size_t)row);
      memcpy((char*)out_v + dst, (const char*)vc + src, (size_t)row);
    }
  }
  return 0;
}

/*
 * Paged decode attention, one query per sequence (paged_attention_ref.py:102-161):
 * for sequence s, the -1 entries of its table row are dropped (:137-138), the
 * first kv_len[s] tokens are gathered in logical order, query head h attends
 * KV head h / (H / KH) (repeat_interleave, :146-147), and
 *     out[s][h] = sum_t softmax_t(scale * q[s][h] . k_t) v_t      (:155-157).
 * query is [Nd][H][D] (contiguous), table [Nd][max_blocks], out float32
 * [Nd][H][D].  status[s] receives ORACLE_OK or an error code for sequence s.
 * Sequences run in parallel over `threads` OpenMP threads (<= 0: all).
 */
int oracle_decode(const void* query, const void* kc, const void* vc, const int64_t* table,
                  int64_t max_blocks, const int32_t* kv_len, int64_t Nd, int H, int KH, int D,
                  int BS, int64_t NB, double scale, int dtype, int threads, float* out,
                  int32_t* status) {
  const int G = H / KH;
  int nerr = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : omp_get_max_threads()) reduction(+ : nerr)
  for (int64_t s = 0; s < Nd; ++s) {
    const int64_t n = kv_len[s];
    status[s] = ORACLE_OK;
    if (n < 1) {
      status[s] = ORACLE_KV_LEN;
      ++nerr;
      continue;
    }
    /* compact the row: drop -1 padding, keep order */
    int64_t* ids = (int64_t*)malloc(sizeof(int64_t) * (size_t)(max_blocks > 0 ? max_blocks : 1));
    int64_t nids = 0;
    int bad = 0;
    for (int64_t b = 0; b < max_blocks; ++b) {
      const int64_t id = table[s * max_blocks + b];
      if (id == -1) continue;
      if (id < -1 || id >= NB) bad = 1;
      ids[nids++] = id;
    }
    const int64_t need = (n + BS - 1) / BS;
    if (need > nids) {
      status[s] = ORACLE_TABLE_SHORT;
    } else {
      for (int64_t b = 0; b < need; ++b)
        if (ids[b] < 0 || ids[b] >= NB) bad = 1;
      if (bad) status[s] = ORACLE_BLOCK_ID;
    }
    if (status[s] != ORACLE_OK) {
      free(ids);
      ++nerr;
      continue;
    }
    double* logit = (double*)malloc(sizeof(double) * (size_t)n * (size_t)G);
    double* acc = (double*)malloc(sizeof(double) * (size_t)D);
    double* q = (double*)malloc(sizeof(double) * (size_t)D * (size_t)G);
    for (int kvh = 0; kvh < KH; ++kvh) {
      for (int g = 0; g < G; ++g)
        for (int d = 0; d < D; ++d)
          q[g * D + d] = load(query, (s * H + (int64_t)kvh * G + g) * D + d, dtype);
      /* logits for the G heads that share this KV head */
      for (int64_t t = 0; t < n; ++t) {
        const int64_t base = ((ids[t / BS] * KH + kvh) * BS + t % BS) * D;
        for (int g = 0; g < G; ++g) {
          double dot = 0.0;
          for (int d = 0; d < D; ++d) dot += q[g * D + d] * load(kc, base + d, dtype);
          logit[t * G + g] = dot * scale;
        }
      }
      for (int g = 0; g < G; ++g) {
        double mx = -INFINITY;
        for (int64_t t = 0; t < n; ++t) mx = logit[t * G + g] > mx ? logit[t * G + g] : mx;
        double sum = 0.0;
        for (int d = 0; d < D; ++d) acc[d] = 0.0;
        for (int64_t t = 0; t < n; ++t) {
          const double p = exp(logit[t * G + g] - mx);
          sum += p;
          const int64_t base = ((ids[t / BS] * KH + kvh) * BS + t % BS) * D;
          for (int d = 0; d < D; ++d) acc[d] += p * load(vc, base + d, dtype);
        }
        float* o = out + (s * H + (int64_t)kvh * G + g) * D;
        for (int d = 0; d < D; ++d) o[d] = (float)(acc[d] / sum);
      }
    }
    free(q);
    free(acc);
    free(logit);
    free(ids);
  }
  return nerr;
}

int oracle_max_threads(void) { return omp_get_max_threads(); }
