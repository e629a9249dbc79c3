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
// serve columns 4c..4c+3, each mapped to (0, 1) as ((x >> 8) + 0.5) * 2^-24.
//
// One CTA per row, 16-byte loads of 8 logits where the row allows it; each
// thread keeps its best (score, index), then a warp-shuffle and a
// shared-memory reduction pick the row's winner (lowest index on equal
// scores).
#include "common.cuh"

namespace nvattn {

constexpr int kSampleThreads = 512;

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

// Gumbel variable from a 32-bit word: a 24-bit uniform (exact in fp32,
// strictly inside (0, 1), so the noise is finite), then -log(-log u). The
// inner log uses the accurate logf: near u = 1, -log u is ~1e-7 and an
// approximate log's absolute error would swamp it.
__device__ __forceinline__ float gumbel(uint32_t x) {
  const float u = (static_cast<float>(x >> 8) + 0.5f) * 5.9604644775390625e-08f;  // 2^-24
  return -__logf(-logf(u));
}

__device__ __forceinline__ void take(float s, int64_t i, float& best, int64_t& bi) {
  // columns arrive in increasing order per thread: strict > keeps the first
  if (s > best) {
    best = s;
    bi = i;
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kSampleThreads)
    sample_kernel(const __nv_bfloat16* __restrict__ logits, int64_t row_stride, int64_t vocab,
                  const float* __restrict__ temperatures, uint64_t seed, uint64_t offset,
                  int64_t* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * row_stride;
  const float t = temperatures ? temperatures[row] : 0.f;
  const bool greedy = !(t > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / t;
  const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  const uint32_t o0 = static_cast<uint32_t>(offset), o1 = static_cast<uint32_t>(offset >> 32);
  float best = -INFINITY;
  int64_t bi = vocab;  // "none yet": loses to any real column

  auto score = [&](float l, float g) { return greedy ? l : l * inv_t + g; };
  if (VEC) {
    const int64_t nvec = vocab / 8;
    for (int64_t vi = threadIdx.x; vi < nvec; vi += kSampleThreads) {
      const int4 raw = __ldg(reinterpret_cast<const int4*>(x) + vi);
      const uint32_t w[4] = {static_cast<uint32_t>(raw.x), static_cast<uint32_t>(raw.y),
                             static_cast<uint32_t>(raw.z), static_cast<uint32_t>(raw.w)};
      uint4 r0 = make_uint4(0, 0, 0, 0), r1 = r0;
      if (!greedy) {
        const uint64_t c = static_cast<uint64_t>(vi) * 2;  // 8 columns = two Philox counters
        r0 = philox4x32_10(static_cast<uint32_t>(c), static_cast<uint32_t>(row), o0, o1, k0, k1);
        r1 = philox4x32_10(static_cast<uint32_t>(c + 1), static_cast<uint32_t>(row), o0, o1, k0,
                           k1);
      }
      const uint32_t rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t bits = (e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16);
        take(score(__uint_as_float(bits), greedy ? 0.f : gumbel(rr[e])), vi * 8 + e, best, bi);
      }
    }
    // the tail (< 8 columns) goes to the scalar loop below
  }
  const int64_t start = VEC ? (vocab / 8) * 8 : 0;
  for (int64_t i = start + threadIdx.x; i < vocab; i += kSampleThreads) {
    float g = 0.f;
    if (!greedy) {
      const uint4 r = philox4x32_10(static_cast<uint32_t>(i >> 2), static_cast<uint32_t>(row), o0,
                                    o1, k0, k1);
      const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
      g = gumbel(rr[i & 3]);
    }
    take(score(__bfloat162float(x[i]), g), i, best, bi);
  }

  // Row reduction: larger score wins, the lower index on ties.
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  __shared__ float sb[kSampleThreads / 32];
  __shared__ int64_t si[kSampleThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < kSampleThreads / 32 ? sb[lane] : -INFINITY;
    bi = lane < kSampleThreads / 32 ? si[lane] : vocab;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    // a row of NaN/-inf only: fall back to column 0 like argmax of equal values
    if (lane == 0) out[row] = bi < vocab ? bi : 0;
  }
}

}  // namespace nvattn

using namespace nvattn;

extern "C" NVATTN_API int nvattn_sample(const void* logits, int64_t row_stride, int64_t num_rows,
                                        int64_t vocab, const float* temperatures, uint64_t seed,
                                        uint64_t offset, int64_t* out_tokens, void* stream) {
  clear_error();
  if (num_rows < 0 || vocab <= 0 || row_stride < vocab)
    return fail(NVATTN_ERR_INVALID, "sample: bad size or row stride");
  if (num_rows == 0) return NVATTN_OK;
  if (!logits || !out_tokens) return fail(NVATTN_ERR_INVALID, "sample: NULL pointer");
  if (num_rows > 0x7fffffff || vocab > 0x7fffffffLL * 4)
    return fail(NVATTN_ERR_INVALID, "sample: too many rows or columns");
  const bool vec = reinterpret_cast<uintptr_t>(logits) % 16 == 0 && (row_stride * 2) % 16 == 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(logits);
  if (vec)
    sample_kernel<true><<<static_cast<unsigned>(num_rows), kSampleThreads, 0, s>>>(
        x, row_stride, vocab, temperatures, seed, offset, out_tokens);
  else
    sample_kernel<false><<<static_cast<unsigned>(num_rows), kSampleThreads, 0, s>>>(
        x, row_stride, vocab, temperatures, seed, offset, out_tokens);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NVATTN_ERR_CUDA, cudaGetErrorString(e));
  return NVATTN_OK;
}
