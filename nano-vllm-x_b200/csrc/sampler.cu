// Token sampling from bf16 logits in one pass (replaces Sampler.forward,
// nanovllm/layers/sampler.py:5-12, and the greedy argmax of the same logits).
//
// The reference computes probs = softmax(logits / T) and picks
// argmax(probs / E) with E ~ Exp(1) per element (the exponential race). The
// softmax normaliser is common to a row, so the pick equals
// argmax(logits / T - log E) = argmax(logits / T + G), G = -log(-log U) a
// Gumbel variable: one pass over the row, no probability tensor. T <= 0
// selects greedy decoding: argmax(logits), first index on ties (the rule of
// torch.argmax).
//
// U comes from Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011): counter (column/4, row,
// offset_lo, offset_hi), key (seed_lo, seed_hi); the four 32-bit outputs
// serve columns 4c..4c+3, each mapped to (0, 1) as ((x >> 9) + 0.5) * 2^-23.
//
// Work split: one CTA per (row, column chunk), 16-byte loads of 8 logits
// where the row allows it. Each CTA folds its best (score, column) into the
// row's 64-bit key with atomicMax; a merge kernel turns keys into columns.
// The same keys, computed per vocabulary shard on tensor-parallel ranks
// (columns numbered globally), merge across ranks to exactly the pick over
// the whole row, so the LM head's logits never have to be gathered
// (embed_head.py:56-66 gathers them to rank 0 before sampling).
#include "common.cuh"

namespace nvattn {

constexpr int kSampleThreads = 256;

__device__ __forceinline__ void philox_round(uint32_t c[4], const uint32_t k[2]) {
  const uint32_t m0 = 0xD2511F53u, m1 = 0xCD9E8D57u;  // multipliers of Philox4x32
  const uint32_t hi0 = __umulhi(m0, c[0]), lo0 = m0 * c[0];
  const uint32_t hi1 = __umulhi(m1, c[2]), lo1 = m1 * c[2];
  const uint32_t n0 = hi1 ^ c[1] ^ k[0], n2 = hi0 ^ c[3] ^ k[1];
  c[0] = n0;
  c[1] = lo1;
  c[2] = n2;
  c[3] = lo0;
}

// Philox4x32-10 of one counter: ten rounds, the key bumped by the Weyl
// constants between rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                               uint32_t k0, uint32_t k1) {
  uint32_t c[4] = {c0, c1, c2, c3};
  uint32_t k[2] = {k0, k1};
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k[0] += 0x9E3779B9u;
      k[1] += 0xBB67AE85u;
    }
    philox_round(c, k);
  }
  return make_uint4(c[0], c[1], c[2], c[3]);
}

// Gumbel variable from a 32-bit word: a 23-bit uniform u = (k + 0.5) * 2^-23,
// k = x >> 9. k + 0.5 < 2^23 needs 24 significant bits, so u is exact in
// fp32 and lies in [2^-24, 1 - 2^-24]: -log u > 0 and the noise is finite
// (with 24 bits, k + 0.5 would round to 2^24 for the largest k, u to 1 and
// the noise to +inf). Then -log(-log u).
//
// The inner -log u needs relative accuracy where it is small (u near 1: the
// largest noise values, the ones that win). t = 1 - u is exact in fp32 (u is
// an odd multiple of 2^-24: for u >= 1/2 by Sterbenz's lemma, below that 1 - u
// lies in [1/2, 1), where the spacing is 2^-24), and -log u = -log1p(-t) =
// t + t^2/2 + t^3/3 + ...:
// for t < 1/32 five terms leave a relative error below t^5/6 < 6e-9. For
// t >= 1/32, -log u >= 0.031 and the MUFU log (absolute error ~2^-22 in
// log2) is within 6e-6 relative, so the noise moves by less than 6e-6: far
// below the bf16 spacing of the logits it is added to, and every path and
// shard computes it the same way.
__device__ __forceinline__ float gumbel(uint32_t x) {
  const float u = (static_cast<float>(x >> 9) + 0.5f) * 1.1920928955078125e-07f;  // 2^-23
  const float t = 1.0f - u;
  float p = fmaf(t, 0.2f, 0.25f);
  p = fmaf(t, p, 0.333333343f);
  p = fmaf(t, p, 0.5f);
  p = fmaf(t, p, 1.0f);
  const float e = t < 0.03125f ? t * p : -__logf(u);
  return -__logf(e);
}

// No gumbel() value exceeds this: the largest u = 1 - 2^-24 gives
// -log(-log u) = 16.64, and the margin covers the approximate outer log.
constexpr float kGumbelBound = 17.0f;

// Largest of the 8 bf16 logits of a 16-byte vector (NaN ignored, as by
// __hmax2: an all-NaN vector gives NaN).
__device__ __forceinline__ float vec_max8(const int4 raw) {
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
  const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&raw.z);
  const __nv_bfloat162 d = *reinterpret_cast<const __nv_bfloat162*>(&raw.w);
  const __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
  return fmaxf(__low2float(m), __high2float(m));
}

// A (score, column) pair as one 64-bit key whose unsigned order is the pick
// order: the high word is the score's bits made monotone (sign bit set for
// x >= 0, all bits flipped for x < 0; -0 is folded into +0 first so that
// equal scores compare equal), the low word is 0xFFFFFFFF - column, so on
// equal scores the lower column wins. 0 means "no column": a key is only
// made from a score > -inf, whose high word is above 0x007FFFFF.
__device__ __forceinline__ unsigned long long pick_key(float s, uint32_t col) {
  uint32_t b = __float_as_uint(s == 0.f ? 0.f : s);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - col);
}

// Per-thread running pick: columns arrive in increasing order, so the strict
// > keeps the first of equal scores; NaN and -inf never replace the start
// value (-inf, "none").
__device__ __forceinline__ void take(float s, uint32_t col, float& best, uint32_t& bcol) {
  if (s > best) {
    best = s;
    bcol = col;
  }
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

// One CTA scans `chunk` columns of one row (chunks are multiples of 8
// columns) and folds its best key into keys[row] with a 64-bit atomicMax.
// Columns are numbered globally: col0 + local column, so vocabulary shards
// of one row on different ranks draw the same noise per column and their
// keys merge to the pick over the whole row. VEC requires 16-byte aligned
// rows and col0 % 4 == 0 (8 columns = two whole Philox counters).
template <bool VEC>
__global__ void __launch_bounds__(kSampleThreads, 8)
    sample_chunk_kernel(const __nv_bfloat16* __restrict__ logits, int64_t row_stride,
                        int64_t vocab, int64_t chunk, int64_t num_chunks, uint64_t col0,
                        const float* __restrict__ temperatures, uint64_t seed, uint64_t offset,
                        unsigned long long* __restrict__ keys) {
  // the host keeps num_rows * num_chunks below 2^31: 32-bit division
  const uint32_t nch = static_cast<uint32_t>(num_chunks);
  const uint32_t row32 = blockIdx.x / nch;
  const int64_t row = row32;
  const int64_t c_begin = static_cast<int64_t>(blockIdx.x - row32 * nch) * chunk;
  const int64_t c_end = min(vocab, c_begin + chunk);
  const __nv_bfloat16* x = logits + row * row_stride;
  const float t = temperatures ? temperatures[row] : 0.f;
  const bool greedy = !(t > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / t;
  const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  const uint32_t o0 = static_cast<uint32_t>(offset), o1 = static_cast<uint32_t>(offset >> 32);
  const uint32_t r32 = row32;
  float best = -INFINITY;
  uint32_t bcol = 0;

  // score of one column: the logit (greedy) or logit / T + Gumbel noise, as
  // one rounded fma so that every path and every shard computes the same bits
  auto score = [&](float l, uint32_t word) {
    return greedy ? l : __fmaf_rn(l, inv_t, gumbel(word));
  };
  int64_t scalar_from = c_begin;
  if (VEC) {
    const int64_t v_end = c_end / 8;  // whole vectors of this chunk
    const int4* xv = reinterpret_cast<const int4*>(x);
    // 8 columns of one vector, in column order
    auto take8 = [&](const int4 raw, int64_t vi, const uint32_t rr[8]) {
      const uint32_t w[4] = {static_cast<uint32_t>(raw.x), static_cast<uint32_t>(raw.y),
                             static_cast<uint32_t>(raw.z), static_cast<uint32_t>(raw.w)};
      const uint64_t g = col0 + static_cast<uint64_t>(vi) * 8;  // global column of element 0
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t bits = (e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16);
        take(score(__uint_as_float(bits), rr[e]), static_cast<uint32_t>(g + e), best, bcol);
      }
    };
    if (greedy) {
      // memory-bound: four 16-byte loads in flight per thread. A vector's
      // columns are scanned only when its largest logit beats the thread's
      // best; the scan then takes its first column holding that value (the
      // order-preserving equivalent of scanning every column with a strict >).
      for (int64_t base = c_begin / 8 + threadIdx.x; base < v_end; base += 4 * kSampleThreads) {
        int4 raw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t vi = base + u * kSampleThreads;
          raw[u] = vi < v_end ? __ldg(xv + vi) : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t vi = base + u * kSampleThreads;
          if (vi >= v_end) break;
          const float m = vec_max8(raw[u]);
          if (m > best) {
            const uint32_t w[4] = {static_cast<uint32_t>(raw[u].x), static_cast<uint32_t>(raw[u].y),
                                   static_cast<uint32_t>(raw[u].z), static_cast<uint32_t>(raw[u].w)};
            int first = 7;
#pragma unroll
            for (int e = 7; e >= 0; --e) {
              const uint32_t bits = (e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16);
              if (__uint_as_float(bits) == m) first = e;
            }
            best = m;
            bcol = static_cast<uint32_t>(col0 + static_cast<uint64_t>(vi) * 8 + first);
          }
        }
      }
    } else {
      // bound by the noise arithmetic: one vector and two Philox counters per
      // step. A vector none of whose columns can beat the thread's best
      // (largest logit / T + the noise bound below it, with the same rounded
      // fma, hence an upper bound of every score in the vector) skips the
      // noise: its columns would never be picked.
      for (int64_t vi = c_begin / 8 + threadIdx.x; vi < v_end; vi += kSampleThreads) {
        const int4 raw = __ldg(xv + vi);
        if (__fmaf_rn(vec_max8(raw), inv_t, kGumbelBound) < best) continue;
        const uint32_t c = static_cast<uint32_t>((col0 + static_cast<uint64_t>(vi) * 8) >> 2);
        const uint4 r0 = philox4x32_10(c, r32, o0, o1, k0, k1);
        const uint4 r1 = philox4x32_10(c + 1, r32, o0, o1, k0, k1);
        const uint32_t rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
        take8(raw, vi, rr);
      }
    }
    scalar_from = v_end * 8 > c_begin ? v_end * 8 : c_begin;  // the row's tail (< 8 columns)
  }
  for (int64_t i = scalar_from + threadIdx.x; i < c_end; i += kSampleThreads) {
    const uint64_t g = col0 + static_cast<uint64_t>(i);
    uint32_t word = 0;
    if (!greedy) {
      const uint4 r = philox4x32_10(static_cast<uint32_t>(g >> 2), r32, o0, o1, k0, k1);
      const uint32_t q = static_cast<uint32_t>(g & 3);
      word = q == 0 ? r.x : (q == 1 ? r.y : (q == 2 ? r.z : r.w));
    }
    take(score(__bfloat162float(x[i]), word), static_cast<uint32_t>(g), best, bcol);
  }

  unsigned long long key = best > -INFINITY ? pick_key(best, bcol) : 0ull;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) key = umax64(key, __shfl_xor_sync(0xffffffffu, key, off));
  __shared__ unsigned long long sbest[kSampleThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sbest[warp] = key;
  __syncthreads();
  if (warp == 0) {
    key = lane < kSampleThreads / 32 ? sbest[lane] : 0ull;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) key = umax64(key, __shfl_xor_sync(0xffffffffu, key, off));
    if (lane == 0 && key != 0ull) atomicMax(keys + row, key);
  }
}

// tokens[r] = the column of max over shards of keys[s * num_rows + r]; a row
// with no candidate (all NaN / -inf) takes column 0. In place is allowed
// (keys == tokens with one shard): each thread reads its row before writing it.
__global__ void sample_merge_kernel(const unsigned long long* keys, int64_t num_shards,
                                    int64_t num_rows, int64_t* tokens) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= num_rows) return;
  unsigned long long k = 0ull;
  for (int64_t s = 0; s < num_shards; ++s) k = umax64(k, keys[s * num_rows + r]);
  tokens[r] = k ? static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(k)) : 0;
}

static int device_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Zero the keys, then one CTA per (row, chunk). Chunks: enough per row that
// all rows together fill about 4 CTAs per SM-slot (8 slots of 256 threads
// per SM), never under 2048 columns (one 8-column vector per thread), a
// multiple of 8. The split depends on host sizes only, so a captured graph
// keeps its grid.
static int launch_keys(const void* logits, int64_t row_stride, int64_t num_rows, int64_t vocab,
                       uint64_t col0, const float* temperatures, uint64_t seed, uint64_t offset,
                       unsigned long long* keys, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(keys, 0, static_cast<size_t>(num_rows) * 8, s);
  if (e != cudaSuccess) return cuda_fail(e, "sample: memset");
  const int64_t target = 4LL * 8 * device_sms();
  const int64_t max_chunks = (vocab + 2047) / 2048;
  int64_t nch = (target + num_rows - 1) / num_rows;
  nch = nch < 1 ? 1 : (nch > max_chunks ? max_chunks : nch);
  int64_t chunk = (vocab + nch - 1) / nch;
  chunk = (chunk + 7) / 8 * 8;
  nch = (vocab + chunk - 1) / chunk;
  if (num_rows * nch > 0x7fffffffLL) return fail(NVATTN_ERR_INVALID, "sample: grid too large");
  const bool vec = reinterpret_cast<uintptr_t>(logits) % 16 == 0 && (row_stride * 2) % 16 == 0 &&
                   col0 % 4 == 0;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(logits);
  const unsigned grid = static_cast<unsigned>(num_rows * nch);
  if (vec)
    sample_chunk_kernel<true><<<grid, kSampleThreads, 0, s>>>(
        x, row_stride, vocab, chunk, nch, col0, temperatures, seed, offset, keys);
  else
    sample_chunk_kernel<false><<<grid, kSampleThreads, 0, s>>>(
        x, row_stride, vocab, chunk, nch, col0, temperatures, seed, offset, keys);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "sample_chunk_kernel");
  return NVATTN_OK;
}

static int launch_merge(const unsigned long long* keys, int64_t num_shards, int64_t num_rows,
                        int64_t* tokens, cudaStream_t s) {
  const unsigned grid = static_cast<unsigned>((num_rows + 255) / 256);
  sample_merge_kernel<<<grid, 256, 0, s>>>(keys, num_shards, num_rows, tokens);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "sample_merge_kernel");
  return NVATTN_OK;
}

}  // namespace nvattn

using namespace nvattn;

static int check_rows(const char* fn, const void* logits, int64_t row_stride, int64_t num_rows,
                      int64_t vocab, uint64_t col0, const void* out) {
  if (num_rows < 0 || vocab <= 0 || row_stride < vocab)
    return fail(NVATTN_ERR_INVALID, std::string(fn) + ": bad size or row stride");
  if (num_rows > 0x7fffffffLL || col0 + static_cast<uint64_t>(vocab) > 0xFFFFFFFFull)
    return fail(NVATTN_ERR_INVALID, std::string(fn) + ": too many rows or columns");
  if (num_rows > 0 && (!logits || !out))
    return fail(NVATTN_ERR_INVALID, std::string(fn) + ": NULL pointer");
  return NVATTN_OK;
}

extern "C" NVATTN_API int nvattn_sample(const void* logits, int64_t row_stride, int64_t num_rows,
                                        int64_t vocab, const float* temperatures, uint64_t seed,
                                        uint64_t offset, int64_t* out_tokens, void* stream) {
  clear_error();
  int rc = check_rows("sample", logits, row_stride, num_rows, vocab, 0, out_tokens);
  if (rc != NVATTN_OK || num_rows == 0) return rc;
  if (reinterpret_cast<uintptr_t>(out_tokens) % 8 != 0)
    return fail(NVATTN_ERR_INVALID, "sample: out_tokens must be 8-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // out_tokens holds the row keys until the merge turns them into columns
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(out_tokens);
  rc = launch_keys(logits, row_stride, num_rows, vocab, 0, temperatures, seed, offset, keys, s);
  if (rc != NVATTN_OK) return rc;
  return launch_merge(keys, 1, num_rows, out_tokens, s);
}

extern "C" NVATTN_API int nvattn_sample_shard(const void* logits, int64_t row_stride,
                                              int64_t num_rows, int64_t vocab_shard,
                                              int64_t vocab_offset, const float* temperatures,
                                              uint64_t seed, uint64_t offset, uint64_t* out_keys,
                                              void* stream) {
  clear_error();
  if (vocab_offset < 0) return fail(NVATTN_ERR_INVALID, "sample_shard: negative vocab_offset");
  int rc = check_rows("sample_shard", logits, row_stride, num_rows, vocab_shard,
                      static_cast<uint64_t>(vocab_offset), out_keys);
  if (rc != NVATTN_OK || num_rows == 0) return rc;
  if (reinterpret_cast<uintptr_t>(out_keys) % 8 != 0)
    return fail(NVATTN_ERR_INVALID, "sample_shard: out_keys must be 8-byte aligned");
  return launch_keys(logits, row_stride, num_rows, vocab_shard, static_cast<uint64_t>(vocab_offset),
                     temperatures, seed, offset, reinterpret_cast<unsigned long long*>(out_keys),
                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" NVATTN_API int nvattn_sample_merge(const uint64_t* keys, int64_t num_shards,
                                              int64_t num_rows, int64_t* out_tokens,
                                              void* stream) {
  clear_error();
  if (num_shards <= 0 || num_rows < 0)
    return fail(NVATTN_ERR_INVALID, "sample_merge: bad number of shards or rows");
  if (num_rows == 0) return NVATTN_OK;
  if (!keys || !out_tokens) return fail(NVATTN_ERR_INVALID, "sample_merge: NULL pointer");
  if (num_rows > 0x7fffffffLL - 255)
    return fail(NVATTN_ERR_INVALID, "sample_merge: too many rows");
  if (num_shards > 1 && reinterpret_cast<const void*>(keys) == reinterpret_cast<void*>(out_tokens))
    return fail(NVATTN_ERR_INVALID, "sample_merge: in place needs one shard");
  return launch_merge(reinterpret_cast<const unsigned long long*>(keys), num_shards, num_rows,
                      out_tokens, reinterpret_cast<cudaStream_t>(stream));
}
