/*
 * CPU restatement of the paged decode attention — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm load
 * this library, as the checker or as the timed CPU baseline; the product
 * (nvattn) never does.
 *
 * It restates what the reference computes at nanovllm/layers/attention.py:72-74,
 * flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache, cache_seqlens,
 * block_table, softmax_scale, causal=True) for one query per sequence:
 * out[b, h] = softmax(scale * q[b, h] . K_b^T) V_b over the cache_seqlens[b]
 * cached keys of sequence b, key j at row j % block_size of block
 * block_table[b, j / block_size], query head h reading KV head
 * h / (H / KVH); a sequence with no keys gives 0. The arithmetic is fp32
 * from bf16 inputs, in two passes per (sequence, KV head): scores of the
 * whole GQA group, then the max-shifted exponentials and the weighted sum of
 * V, so every K and V row is read once. The same function as
 * oracle/reference_math.py:decode_attention, in C with OpenMP over
 * (sequence, KV head) pairs, so the CPU baseline uses every host core.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { kD = 128 }; /* head_dim: the path's only size */

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof(f));
  return f;
}

/* One (sequence, KV head) pair; scores holds G * n floats. */
__attribute__((target_clones("avx2", "default")))
static void decode_pair(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                        const int32_t* table, int64_t n, int64_t kvh, int64_t G, int64_t KVH,
                        int64_t D, int64_t bs, float scale, float* scores, float* out) {
  float qf[16 * kD];
  float row[kD];
  for (int64_t g = 0; g < G; ++g)
    for (int64_t d = 0; d < D; ++d) qf[g * D + d] = bf16_to_f32(q[(kvh * G + g) * D + d]);
  for (int64_t t = 0; t < n; ++t) {
    const int64_t slot = (int64_t)table[t / bs] * bs + t % bs;
    const uint16_t* k = k_cache + (slot * KVH + kvh) * D;
    for (int64_t d = 0; d < D; ++d) row[d] = bf16_to_f32(k[d]);
    for (int64_t g = 0; g < G; ++g) {
      /* 16 independent partial sums (vectorisable), then their total */
      const float* qg = qf + g * kD;
      float part[16] = {0.f};
      for (int d0 = 0; d0 < kD; d0 += 16)
        for (int j = 0; j < 16; ++j) part[j] += qg[d0 + j] * row[d0 + j];
      float acc = 0.f;
      for (int j = 0; j < 16; ++j) acc += part[j];
      scores[g * n + t] = acc * scale;
    }
  }
  float denom[16];
  for (int64_t g = 0; g < G; ++g) {
    float m = -INFINITY;
    for (int64_t t = 0; t < n; ++t) m = fmaxf(m, scores[g * n + t]);
    float s = 0.f;
    for (int64_t t = 0; t < n; ++t) {
      const float p = expf(scores[g * n + t] - m);
      scores[g * n + t] = p;
      s += p;
    }
    denom[g] = s;
  }
  float acc[16 * 128];
  memset(acc, 0, sizeof(float) * (size_t)(G * D));
  for (int64_t t = 0; t < n; ++t) {
    const int64_t slot = (int64_t)table[t / bs] * bs + t % bs;
    const uint16_t* v = v_cache + (slot * KVH + kvh) * D;
    for (int64_t d = 0; d < D; ++d) row[d] = bf16_to_f32(v[d]);
    for (int64_t g = 0; g < G; ++g) {
      const float p = scores[g * n + t];
      for (int64_t d = 0; d < D; ++d) acc[g * D + d] += p * row[d];
    }
  }
  for (int64_t g = 0; g < G; ++g)
    for (int64_t d = 0; d < D; ++d) out[(kvh * G + g) * D + d] = acc[g * D + d] / denom[g];
}

/*
 * q: (B, H, D) bf16; k_cache, v_cache: (num_blocks, bs, KVH, D) bf16;
 * cache_seqlens: (B,); block_table: (B, W); out: (B, H, D) fp32.
 * Returns 0, or -1 for unsupported sizes (D != 128, H / KVH > 16), a length
 * beyond its block table (W * bs keys), or a block id that a sequence's keys
 * use outside [0, num_blocks) (checked before any cache read).
 */
int oracle_decode_attention(const uint16_t* q, const uint16_t* k_cache,
                            const uint16_t* v_cache, const int32_t* cache_seqlens,
                            const int32_t* block_table, int64_t B, int64_t H, int64_t KVH,
                            int64_t D, int64_t bs, int64_t W, int64_t num_blocks, float scale,
                            float* out, int threads) {
  if (B < 0 || KVH <= 0 || H % KVH != 0 || H / KVH > 16 || D != kD || bs <= 0) return -1;
  const int64_t G = H / KVH;
  for (int64_t b = 0; b < B; ++b) {
    /* every key must lie inside the sequence's block table, in a real block */
    if (cache_seqlens[b] > W * bs) return -1;
    const int64_t used = cache_seqlens[b] > 0 ? (cache_seqlens[b] + bs - 1) / bs : 0;
    for (int64_t i = 0; i < used; ++i) {
      const int32_t id = block_table[b * W + i];
      if (id < 0 || id >= num_blocks) return -1;
    }
  }
  int failed = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
  for (int64_t job = 0; job < B * KVH; ++job) {
    const int64_t b = job / KVH, kvh = job % KVH;
    const int64_t n = cache_seqlens[b];
    float* o = out + b * H * D;
    if (n <= 0) {
      for (int64_t i = kvh * G * D; i < (kvh + 1) * G * D; ++i) o[i] = 0.f;
      continue;
    }
    float* scores = (float*)malloc(sizeof(float) * (size_t)(G * n));
    if (!scores) {
#pragma omp atomic write
      failed = 1;
      continue;
    }
    decode_pair(q + b * H * D, k_cache, v_cache, block_table + b * W, n, kvh, G, KVH, D, bs,
                scale, scores, o);
    free(scores);
  }
  return failed ? -1 : 0;
}
