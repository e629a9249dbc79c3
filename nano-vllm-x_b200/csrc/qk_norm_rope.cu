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
// its (q heads, then KV heads) list, 128 elements each; lane i holds dims
// 4i..4i+3 (8-byte accesses, 256 contiguous bytes per row). All loads of the
// group are issued before any arithmetic so enough bytes are in flight to
// cover HBM latency, and the token's position, cos/sin and slot are loaded
// once. KV-head rows also copy the token's V row into the cache. Rotation
// partners (dim j and j+64) sit in lanes i and i+16.
//
// Arithmetic is fp32 in a fixed order, every step correctly rounded and
// never contracted into an FMA, so the result is a pure function of the
// inputs (the oracle restates the same order):
//   lane sum  s_i = ((x0*x0 + x1*x1) + x2*x2) + x3*x3
//   warp sum  butterfly over lane distances 16, 8, 4, 2, 1
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

__global__ void __launch_bounds__(kNormWarps * 32, 5)
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
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
  if (gw >= num_groups) return;
  const int per_tok = num_heads + num_kv_heads;
  const int groups_per_tok = (per_tok + kRowsPerWarp - 1) / kRowsPerWarp;
  const int64_t tok = gw / groups_per_tok;
  const int hi0 = static_cast<int>(gw % groups_per_tok) * kRowsPerWarp;

  // Issue every load of the warp's rows (one token) before any arithmetic.
  uint2 raw[kRowsPerWarp], vraw[kRowsPerWarp];
  const char* qrow = q + tok * q_stride_b;
  const char* krow = k + tok * k_stride_b;
  const char* vrow = v + tok * v_stride_b;
  // V rows are loaded whether or not the token has a slot, so no load waits
  // on the slot lookup (only padding tokens, slot -1, read V for nothing).
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int hi = hi0 + i;
    raw[i] = make_uint2(0u, 0u);
    vraw[i] = make_uint2(0u, 0u);
    if (hi >= per_tok) continue;
    if (hi < num_heads) {
      raw[i] = __ldg(reinterpret_cast<const uint2*>(qrow + hi * 256) + lane);
    } else {
      raw[i] = __ldg(reinterpret_cast<const uint2*>(krow + (hi - num_heads) * 256) + lane);
      if (slot_mapping)
        vraw[i] = __ldg(reinterpret_cast<const uint2*>(vrow + (hi - num_heads) * 256) + lane);
    }
  }
  const int64_t slot = slot_mapping ? static_cast<int64_t>(slot_mapping[tok]) : -1;
  const bool store = slot != -1;
  int64_t pos = positions[tok];
  if (pos < 0 || pos >= max_position) {
    if (lane == 0 && hi0 == 0) set_status(status, NVATTN_STATUS_BAD_POSITION);
    pos = pos < 0 ? 0 : max_position - 1;
  }
  const int c = (lane & 15) * 4;
  const float4 cs = __ldg(reinterpret_cast<const float4*>(cos_sin + pos * 128 + c));
  const float4 sn = __ldg(reinterpret_cast<const float4*>(cos_sin + pos * 128 + 64 + c));
  const uint2 qw = __ldg(reinterpret_cast<const uint2*>(q_weight) + lane);
  const uint2 kw = __ldg(reinterpret_cast<const uint2*>(k_weight) + lane);
  const bool first = lane < 16;
  const bool slot_ok = slot >= 0 && slot < num_slots;
  if (store && !slot_ok && lane == 0 && hi0 == 0) set_status(status, NVATTN_STATUS_BAD_SLOT);

#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int hi = hi0 + i;
    if (hi >= per_tok) break;
    const bool is_q = hi < num_heads;
    const float x[4] = {bf16_lo(raw[i].x), bf16_hi(raw[i].x), bf16_lo(raw[i].y),
                        bf16_hi(raw[i].y)};
    // RMSNorm (layernorm.py:20-24): fp32 sum of squares, mean, 1/sqrt.
    float s = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1])),
                                  __fmul_rn(x[2], x[2])),
                        __fmul_rn(x[3], x[3]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    const float var = __fmul_rn(s, 1.0f / 128.0f);  // exact: a power-of-two scale
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    const uint2 wr = is_q ? qw : kw;
    const float w[4] = {bf16_lo(wr.x), bf16_hi(wr.x), bf16_lo(wr.y), bf16_hi(wr.y)};
    float n[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      n[e] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[e], r)), w[e]));
    // Rotary embedding (rotary_embedding.py:6-14) with the position's cos/sin.
    const float cv[4] = {cs.x, cs.y, cs.z, cs.w};
    const float sv[4] = {sn.x, sn.y, sn.z, sn.w};
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, n[e], 16);
      o[e] = first ? __fsub_rn(__fmul_rn(n[e], cv[e]), __fmul_rn(other, sv[e]))
                   : __fadd_rn(__fmul_rn(n[e], cv[e]), __fmul_rn(other, sv[e]));
    }
    uint2 packed;
    packed.x = pack_bf16x2(o[0], o[1]);
    packed.y = pack_bf16x2(o[2], o[3]);
    if (is_q) {
      reinterpret_cast<uint2*>(q_out + (tok * num_heads + hi) * 128)[lane] = packed;
      continue;
    }
    const int kh = hi - num_heads;
    if (k_out) reinterpret_cast<uint2*>(k_out + (tok * num_kv_heads + kh) * 128)[lane] = packed;
    if (!store || !slot_ok) continue;  // slot -1: attention.py:23
    const int64_t dst = (slot * num_kv_heads + kh) * 256;
    reinterpret_cast<uint2*>(k_cache + dst)[lane] = packed;
    reinterpret_cast<uint2*>(v_cache + dst)[lane] = vraw[i];
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
  if (!al(q, 8) || !al(k, 8) || !al(v, 8) || (q_stride_tok * 2) % 8 || (k_stride_tok * 2) % 8 ||
      (v_stride_tok * 2) % 8 || !al(q_weight, 8) || !al(k_weight, 8) || !al(cos_sin, 16) ||
      !al(q_out, 8) || (k_out && !al(k_out, 8)) || (k_cache && !al(k_cache, 8)) ||
      (v_cache && !al(v_cache, 8)))
    return fail(NVATTN_ERR_UNSUPPORTED,
                "qk_norm_rope_store: rows must be 8-byte aligned (cos_sin 16-byte aligned)");
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
