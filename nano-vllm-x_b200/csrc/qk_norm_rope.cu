// Fused per-head q/k RMSNorm + rotary embedding + KV-cache scatter.
//
// Replaces the four steps of Qwen3Attention.forward between the QKV
// projection and attention (nanovllm/models/qwen3.py:82-86):
//   q = q_norm(q); k = k_norm(k)         RMSNorm over head_dim
//                                        (nanovllm/layers/layernorm.py:16-26)
//   q, k = rotary_emb(positions, q, k)   neox-style rotation with the
//                                        module's fp32 cos/sin cache
//                                        (nanovllm/layers/rotary_embedding.py:6-14,37-48)
//   store_kvcache(k, v, ...)             inside Attention.forward
//                                        (nanovllm/layers/attention.py:10-40,62-63)
// One launch reads each q/k/v row once and writes q, k and the cache rows.
//
// Work unit: a warp takes one token's group of 4 consecutive head rows of
// its (q heads, then KV heads) list, 128 elements each, as two pairs: each
// half-warp owns one row of a pair, lane i of the half holding dims
// 8i..8i+7 (16-byte accesses, 256 contiguous bytes per row). All loads of
// the group are issued before any arithmetic so enough bytes are in flight
// to cover HBM latency, and the token's position, cos/sin and slot are
// loaded once. KV-head rows also copy the token's V row into the cache.
// Rotation partners (dim j and j+64) sit in lanes i and i+8 of a half.
//
// Arithmetic is fp32 in a fixed order, every step correctly rounded and
// never contracted into an FMA, so the result is a pure function of the
// inputs (the oracle restates the same order):
//   lane sum  s_i = ((((((x0*x0 + x1*x1) + x2*x2) + x3*x3) + x4*x4) + x5*x5) + x6*x6) + x7*x7
//   row sum   butterfly over lane distances 8, 4, 2, 1 (within the half-warp)
//   r = 1 / sqrt(sum/128 + eps)                 (sqrt and divide rounded)
//   n_j = bf16(bf16(x_j * r) * w_j)             (reference: x.to(bf16) * weight)
//   j < 64 : o_j = bf16(n_j*cos_j - n_{j+64}*sin_j)
//   j >= 64: o_j = bf16(n_j*cos_{j-64} + n_{j-64}*sin_{j-64})
#include "common.cuh"

namespace nvattn {

constexpr int kNormWarps = 8;
constexpr int kRowsPerWarp = 4;  // rows in flight per warp (latency hiding for HBM)

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__global__ void __launch_bounds__(kNormWarps * 32, 4)
    qk_norm_rope_store_kernel(const char* __restrict__ q, int64_t q_stride_b,
                              const char* __restrict__ k, int64_t k_stride_b,
                              const char* __restrict__ v, int64_t v_stride_b,
                              const __nv_bfloat16* __restrict__ q_weight,
                              const __nv_bfloat16* __restrict__ k_weight,
                              const float* __restrict__ cos_sin, int64_t max_position,
                              const int64_t* __restrict__ positions,
                              const int32_t* __restrict__ slot_mapping,
                              __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out,
                              char* __restrict__ k_cache, char* __restrict__ v_cache,
                              int64_t num_slots, int64_t num_groups, int num_heads,
                              int num_kv_heads, float eps, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;  // row of the pair
  const int li = lane & 15;    // dims 8li..8li+7
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
  if (gw >= num_groups) return;
  const int per_tok = num_heads + num_kv_heads;
  const int groups_per_tok = (per_tok + kRowsPerWarp - 1) / kRowsPerWarp;
  const int64_t tok = gw / groups_per_tok;
  const int hi0 = static_cast<int>(gw % groups_per_tok) * kRowsPerWarp;
  constexpr int kPairs = kRowsPerWarp / 2;

  // Issue every load of the warp's rows (one token) before any arithmetic.
  // V rows are loaded whether or not the token has a slot, so no load waits
  // on the slot lookup (only padding tokens, slot -1, read V for nothing).
  uint4 raw[kPairs], vraw[kPairs];
  const char* qrow = q + tok * q_stride_b;
  const char* krow = k + tok * k_stride_b;
  const char* vrow = v + tok * v_stride_b;
#pragma unroll
  for (int i = 0; i < kPairs; ++i) {
    const int hi = hi0 + 2 * i + half;
    raw[i] = make_uint4(0u, 0u, 0u, 0u);
    vraw[i] = make_uint4(0u, 0u, 0u, 0u);
    if (hi >= per_tok) continue;
    if (hi < num_heads) {
      raw[i] = __ldg(reinterpret_cast<const uint4*>(qrow + hi * 256) + li);
    } else {
      raw[i] = __ldg(reinterpret_cast<const uint4*>(krow + (hi - num_heads) * 256) + li);
      if (slot_mapping)
        vraw[i] = __ldg(reinterpret_cast<const uint4*>(vrow + (hi - num_heads) * 256) + li);
    }
  }
  const int64_t slot = slot_mapping ? static_cast<int64_t>(slot_mapping[tok]) : -1;
  const bool store = slot != -1;
  int64_t pos = positions[tok];
  if (pos < 0 || pos >= max_position) {
    if (lane == 0 && hi0 == 0) set_status(status, NVATTN_STATUS_BAD_POSITION);
    pos = pos < 0 ? 0 : max_position - 1;
  }
  const int c = (li & 7) * 8;  // cos/sin index of dims 8li..8li+7 (mod 64)
  const float4* cs4 = reinterpret_cast<const float4*>(cos_sin + pos * 128 + c);
  const float4* sn4 = reinterpret_cast<const float4*>(cos_sin + pos * 128 + 64 + c);
  const float4 ca = __ldg(cs4), cb = __ldg(cs4 + 1), sa = __ldg(sn4), sb = __ldg(sn4 + 1);
  const float cv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
  const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
  const uint4 qw = __ldg(reinterpret_cast<const uint4*>(q_weight) + li);
  const uint4 kw = __ldg(reinterpret_cast<const uint4*>(k_weight) + li);
  const bool first = li < 8;
  const bool slot_ok = slot >= 0 && slot < num_slots;
  if (store && !slot_ok && lane == 0 && hi0 == 0) set_status(status, NVATTN_STATUS_BAD_SLOT);

#pragma unroll
  for (int i = 0; i < kPairs; ++i) {
    const int hi = hi0 + 2 * i + half;
    if (hi0 + 2 * i >= per_tok) break;  // warp-uniform: no row of this pair exists
    const bool live = hi < per_tok;
    const bool is_q = hi < num_heads;
    const uint32_t rw[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
    float x[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      x[2 * e] = bf16_lo(rw[e]);
      x[2 * e + 1] = bf16_hi(rw[e]);
    }
    // RMSNorm (layernorm.py:20-24): fp32 sum of squares, mean, 1/sqrt.
    float s = __fmul_rn(x[0], x[0]);
#pragma unroll
    for (int e = 1; e < 8; ++e) s = __fadd_rn(s, __fmul_rn(x[e], x[e]));
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    const float var = __fmul_rn(s, 1.0f / 128.0f);  // exact: a power-of-two scale
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    const uint4 wr = is_q ? qw : kw;
    const uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
    float n[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      n[2 * e] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[2 * e], r)), bf16_lo(ww[e])));
      n[2 * e + 1] =
          round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[2 * e + 1], r)), bf16_hi(ww[e])));
    }
    // Rotary embedding (rotary_embedding.py:6-14) with the position's cos/sin.
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, n[e], 8);
      o[e] = first ? __fsub_rn(__fmul_rn(n[e], cv[e]), __fmul_rn(other, sv[e]))
                   : __fadd_rn(__fmul_rn(n[e], cv[e]), __fmul_rn(other, sv[e]));
    }
    uint4 packed;
    packed.x = pack_bf16x2(o[0], o[1]);
    packed.y = pack_bf16x2(o[2], o[3]);
    packed.z = pack_bf16x2(o[4], o[5]);
    packed.w = pack_bf16x2(o[6], o[7]);
    if (!live) continue;
    if (is_q) {
      reinterpret_cast<uint4*>(q_out + (tok * num_heads + hi) * 128)[li] = packed;
      continue;
    }
    const int kh = hi - num_heads;
    if (k_out) reinterpret_cast<uint4*>(k_out + (tok * num_kv_heads + kh) * 128)[li] = packed;
    if (!store || !slot_ok) continue;  // slot -1: attention.py:23
    const int64_t dst = (slot * num_kv_heads + kh) * 256;
    reinterpret_cast<uint4*>(k_cache + dst)[li] = packed;
    reinterpret_cast<uint4*>(v_cache + dst)[li] = vraw[i];
  }
}

}  // namespace nvattn

using namespace nvattn;

extern "C" NVATTN_API int nvattn_qk_norm_rope_store(
    const void* q, int64_t q_stride_tok, const void* k, int64_t k_stride_tok, const void* v,
    int64_t v_stride_tok, const void* q_weight, const void* k_weight, const float* cos_sin,
    int64_t max_position, const int64_t* positions, const int32_t* slot_mapping, void* q_out,
    void* k_out, void* k_cache, void* v_cache, int64_t num_slots, int64_t num_tokens,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float eps, int32_t* status,
    void* stream) {
  clear_error();
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_position <= 0 || num_slots < 0)
    return fail(NVATTN_ERR_INVALID, "qk_norm_rope_store: bad size");
  if (head_dim != 128) return fail(NVATTN_ERR_UNSUPPORTED, "qk_norm_rope_store: head_dim must be 128");
  if (num_tokens == 0) return NVATTN_OK;
  if (!q || !k || !v || !q_weight || !k_weight || !cos_sin || !positions || !q_out)
    return fail(NVATTN_ERR_INVALID, "qk_norm_rope_store: NULL pointer");
  if (slot_mapping && (!k_cache || !v_cache))
    return fail(NVATTN_ERR_INVALID, "qk_norm_rope_store: slot_mapping without caches");
  if (q_stride_tok < int64_t(num_heads) * 128 || k_stride_tok < int64_t(num_kv_heads) * 128 ||
      v_stride_tok < int64_t(num_kv_heads) * 128)
    return fail(NVATTN_ERR_INVALID, "qk_norm_rope_store: token stride smaller than the heads");
  auto al = [](const void* ptr, int a) { return reinterpret_cast<uintptr_t>(ptr) % a == 0; };
  if (!al(q, 16) || !al(k, 16) || !al(v, 16) || (q_stride_tok * 2) % 16 ||
      (k_stride_tok * 2) % 16 || (v_stride_tok * 2) % 16 || !al(q_weight, 16) ||
      !al(k_weight, 16) || !al(cos_sin, 16) || !al(q_out, 16) || (k_out && !al(k_out, 16)) ||
      (k_cache && !al(k_cache, 16)) || (v_cache && !al(v_cache, 16)))
    return fail(NVATTN_ERR_UNSUPPORTED, "qk_norm_rope_store: rows must be 16-byte aligned");
  const int64_t groups =
      num_tokens * ((num_heads + num_kv_heads + kRowsPerWarp - 1) / kRowsPerWarp);
  const int64_t blocks = (groups + kNormWarps - 1) / kNormWarps;
  if (blocks > 0x7fffffff) return fail(NVATTN_ERR_INVALID, "qk_norm_rope_store: too many tokens");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  qk_norm_rope_store_kernel<<<static_cast<unsigned>(blocks), kNormWarps * 32, 0, s>>>(
      static_cast<const char*>(q), q_stride_tok * 2, static_cast<const char*>(k), k_stride_tok * 2,
      static_cast<const char*>(v), v_stride_tok * 2,
      static_cast<const __nv_bfloat16*>(q_weight), static_cast<const __nv_bfloat16*>(k_weight),
      cos_sin, max_position, positions, slot_mapping, static_cast<__nv_bfloat16*>(q_out),
      static_cast<__nv_bfloat16*>(k_out), static_cast<char*>(k_cache), static_cast<char*>(v_cache),
      num_slots, groups, num_heads, num_kv_heads, eps, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NVATTN_ERR_CUDA, cudaGetErrorString(e));
  return NVATTN_OK;
}
