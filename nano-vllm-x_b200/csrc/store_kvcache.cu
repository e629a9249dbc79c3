// KV-cache scatter (replaces store_kvcache / store_kvcache_kernel,
// nanovllm/layers/attention.py:10-40) and grouped in-cache slot moves.
//
// The reference runs one Triton program per token that loads D elements of K
// and V and stores them at slot*D. Here two layouts of the same copy, both in
// VEC-byte vectors (16 bytes when every pointer, stride and D allow it), so
// each warp instruction touches 512 contiguous bytes on the load and on the
// store side:
//   * few tokens (a decode batch): each thread moves one vector of one
//     token's K row and the same vector of its V row; a CTA of 128 threads
//     covers 128/vpr whole tokens (vpr = vectors per row: 128 at 8 KV heads
//     x 128 dims), so a batch of a few hundred tokens spreads over every SM;
//   * many tokens (a prefill chunk): one warp per token, each lane with
//     eight vectors in flight (four of K, four of V) before its stores.
// Pure copy: bit-exact.
#include "common.cuh"

namespace nvattn {

template <int VEC>
struct VecType;
template <>
struct VecType<16> {
  using T = int4;
};
template <>
struct VecType<8> {
  using T = int2;
};
template <>
struct VecType<4> {
  using T = int;
};
template <>
struct VecType<2> {
  using T = short;
};

constexpr int kVecThreads = 128;   // per CTA, vector-per-thread layout
constexpr int kRowWarps = 8;       // per CTA, warp-per-token layout
// Up to this many tokens x vectors per row (1024 tokens at 8 KV heads x 128
// dims), the vector-per-thread layout; beyond, the warp-per-token one (both
// measured on B200 from 64 to 16,384 tokens).
constexpr int64_t kVecLayoutMaxVectors = 131072;

// The rows are read once and the cache rows written once, so neither goes
// through L1 (no_allocate) and the stores are streaming (evict first in L2).
template <typename V>
__device__ __forceinline__ V ld_stream(const V* p) {
  return __ldg(p);
}
template <>
__device__ __forceinline__ int4 ld_stream<int4>(const int4* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
template <typename V>
__device__ __forceinline__ void st_stream(V* p, const V& v) {
  *p = v;
}
template <>
__device__ __forceinline__ void st_stream<int4>(int4* p, const int4& v) {
  asm volatile("st.global.cs.v4.s32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

template <int VEC>
__global__ void __launch_bounds__(kVecThreads)
    store_kvcache_vec_kernel(const char* __restrict__ key, int64_t key_stride_b,
                             const char* __restrict__ value, int64_t value_stride_b,
                             char* __restrict__ k_cache, char* __restrict__ v_cache,
                             const int32_t* __restrict__ slot_mapping, int64_t n_tokens,
                             int64_t row_bytes, int64_t num_slots, int vpr, int tokens_per_cta,
                             int32_t* status) {
  using V = typename VecType<VEC>::T;
  const int t_in = static_cast<int>(threadIdx.x) / vpr;  // 0 when a row has >= 128 vectors
  if (t_in >= tokens_per_cta) return;
  const int64_t tok = static_cast<int64_t>(blockIdx.x) * tokens_per_cta + t_in;
  if (tok >= n_tokens) return;
  const int first = static_cast<int>(threadIdx.x) - t_in * vpr;
  const V* ksrc = reinterpret_cast<const V*>(key + tok * key_stride_b);
  const V* vsrc = reinterpret_cast<const V*>(value + tok * value_stride_b);
  // The rows' loads do not depend on the slot: issue them with the slot load,
  // so the two latencies overlap (a skipped token's loads are simply unused).
  const int32_t slot32 = __ldg(slot_mapping + tok);
  V k = ld_stream(ksrc + first), v = ld_stream(vsrc + first);
  const int64_t slot = slot32;
  if (slot == -1) return;  // attention.py:23
  if (slot < 0 || slot >= num_slots) {
    if (first == 0) set_status(status, NVATTN_STATUS_BAD_SLOT);
    return;
  }
  V* kdst = reinterpret_cast<V*>(k_cache + slot * row_bytes);
  V* vdst = reinterpret_cast<V*>(v_cache + slot * row_bytes);
  for (int i = first;;) {
    st_stream(kdst + i, k);
    st_stream(vdst + i, v);
    i += kVecThreads;
    if (i >= vpr) break;
    k = ld_stream(ksrc + i);
    v = ld_stream(vsrc + i);
  }
}

template <int VEC>
__global__ void __launch_bounds__(kRowWarps * 32)
    store_kvcache_rows_kernel(const char* __restrict__ key, int64_t key_stride_b,
                              const char* __restrict__ value, int64_t value_stride_b,
                              char* __restrict__ k_cache, char* __restrict__ v_cache,
                              const int32_t* __restrict__ slot_mapping, int64_t n_tokens,
                              int64_t row_bytes, int64_t num_slots, int32_t* status) {
  using V = typename VecType<VEC>::T;
  const int lane = threadIdx.x & 31;
  const int64_t tok = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  if (tok >= n_tokens) return;
  const int64_t nvec = row_bytes / VEC;
  const V* ksrc = reinterpret_cast<const V*>(key + tok * key_stride_b);
  const V* vsrc = reinterpret_cast<const V*>(value + tok * value_stride_b);
  const int32_t slot32 = __ldg(slot_mapping + tok);
  // All loads of this lane (and the slot's) before its stores, so both rows'
  // reads and the slot overlap in flight.
  for (int64_t i = lane; i < nvec; i += 128) {
    V k[4], v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i + 32 * u < nvec) {
        k[u] = ld_stream(ksrc + i + 32 * u);
        v[u] = ld_stream(vsrc + i + 32 * u);
      }
    }
    const int64_t slot = slot32;
    if (slot == -1) return;  // attention.py:23
    if (slot < 0 || slot >= num_slots) {
      if (lane == 0 && i == lane) set_status(status, NVATTN_STATUS_BAD_SLOT);
      return;
    }
    V* kdst = reinterpret_cast<V*>(k_cache + slot * row_bytes);
    V* vdst = reinterpret_cast<V*>(v_cache + slot * row_bytes);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i + 32 * u < nvec) {
        st_stream(kdst + i + 32 * u, k[u]);
        st_stream(vdst + i + 32 * u, v[u]);
      }
    }
  }
}

// Group g: read every source row of the group into shared memory, then write
// all destinations, so a group may shift rows onto its own sources. Rows are
// processed in column chunks of kMoveChunk bytes; chunks of different columns
// never overlap, so read-all-then-write per chunk keeps the guarantee.
constexpr int kMoveMax = 64;
constexpr int kMoveChunk = 128;  // 2 x 64 x 128 B = 16 KB of static shared memory

__global__ void __launch_bounds__(256)
    kv_move_kernel(char* __restrict__ k_cache, char* __restrict__ v_cache,
                   const int32_t* __restrict__ src, const int32_t* __restrict__ dst,
                   const int32_t* __restrict__ cu_moves, int32_t num_moves, int64_t row_bytes,
                   int64_t num_slots, int32_t* status) {
  __shared__ int4 kbuf[kMoveMax * kMoveChunk / 16];
  __shared__ int4 vbuf[kMoveMax * kMoveChunk / 16];
  const int g = blockIdx.x;
  const int begin = cu_moves[g];
  int end = cu_moves[g + 1];
  if (begin < 0 || end > num_moves) {
    if (threadIdx.x == 0) set_status(status, NVATTN_STATUS_BAD_SLOT);
    end = min(end, num_moves);
  }
  int count = end - begin;
  if (begin < 0 || count <= 0) return;
  if (count > kMoveMax) {
    if (threadIdx.x == 0) set_status(status, NVATTN_STATUS_BAD_SLOT);
    count = kMoveMax;
  }
  for (int64_t col = 0; col < row_bytes; col += kMoveChunk) {
    const int64_t width = (row_bytes - col < kMoveChunk) ? row_bytes - col : kMoveChunk;
    const int nvec = static_cast<int>(width / 16);
    for (int e = threadIdx.x; e < count * nvec; e += blockDim.x) {
      const int m = e / nvec, i = e % nvec;
      const int64_t s = src[begin + m];
      int4 kv = make_int4(0, 0, 0, 0), vv = make_int4(0, 0, 0, 0);
      if (s >= 0 && s < num_slots) {
        kv = reinterpret_cast<const int4*>(k_cache + s * row_bytes + col)[i];
        vv = reinterpret_cast<const int4*>(v_cache + s * row_bytes + col)[i];
      }
      kbuf[m * nvec + i] = kv;
      vbuf[m * nvec + i] = vv;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < count * nvec; e += blockDim.x) {
      const int m = e / nvec, i = e % nvec;
      const int64_t s = src[begin + m];
      const int64_t d = dst[begin + m];
      if (s < 0 || s >= num_slots || d < 0 || d >= num_slots) {
        if (i == 0 && col == 0) set_status(status, NVATTN_STATUS_BAD_SLOT);
        continue;
      }
      reinterpret_cast<int4*>(k_cache + d * row_bytes + col)[i] = kbuf[m * nvec + i];
      reinterpret_cast<int4*>(v_cache + d * row_bytes + col)[i] = vbuf[m * nvec + i];
    }
    __syncthreads();
  }
}

}  // namespace nvattn

using namespace nvattn;

extern "C" int nvattn_store_kvcache(const void* key, int64_t key_stride, const void* value,
                                    int64_t value_stride, void* k_cache, void* v_cache,
                                    const int32_t* slot_mapping, int64_t num_tokens, int64_t D,
                                    int64_t num_slots, int32_t* status, void* stream) {
  clear_error();
  if (num_tokens < 0 || D <= 0 || num_slots < 0)
    return fail(NVATTN_ERR_INVALID, "store_kvcache: negative size");
  if (num_tokens == 0) return NVATTN_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping)
    return fail(NVATTN_ERR_INVALID, "store_kvcache: NULL pointer");
  if (key_stride < D || value_stride < D)
    return fail(NVATTN_ERR_INVALID, "store_kvcache: token stride smaller than D (rows overlap)");
  const int64_t row_bytes = D * 2;
  // Widest vector that every address and stride allows.
  auto fits = [&](int v) {
    return (row_bytes % v == 0) && ((key_stride * 2) % v == 0) && ((value_stride * 2) % v == 0) &&
           (reinterpret_cast<uintptr_t>(key) % v == 0) &&
           (reinterpret_cast<uintptr_t>(value) % v == 0) &&
           (reinterpret_cast<uintptr_t>(k_cache) % v == 0) &&
           (reinterpret_cast<uintptr_t>(v_cache) % v == 0);
  };
  if (row_bytes > (static_cast<int64_t>(1) << 30))
    return fail(NVATTN_ERR_UNSUPPORTED, "store_kvcache: rows over 1 GiB");
  const int vec = fits(16) ? 16 : fits(8) ? 8 : fits(4) ? 4 : 2;
  const int vpr = static_cast<int>(row_bytes / vec);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const char* kp = static_cast<const char*>(key);
  const char* vp = static_cast<const char*>(value);
  char* kc = static_cast<char*>(k_cache);
  char* vc = static_cast<char*>(v_cache);
  const int64_t ks = key_stride * 2, vs = value_stride * 2;
  if (num_tokens * vpr <= kVecLayoutMaxVectors) {
    const int tpc = vpr >= kVecThreads ? 1 : kVecThreads / vpr;
    const dim3 grid(static_cast<unsigned>((num_tokens + tpc - 1) / tpc)), block(kVecThreads);
#define NVATTN_STORE_VEC(V_)                                                                   \
  store_kvcache_vec_kernel<V_><<<grid, block, 0, s>>>(kp, ks, vp, vs, kc, vc, slot_mapping,    \
                                                      num_tokens, row_bytes, num_slots, vpr, tpc, \
                                                      status)
    if (vec == 16) NVATTN_STORE_VEC(16);
    else if (vec == 8) NVATTN_STORE_VEC(8);
    else if (vec == 4) NVATTN_STORE_VEC(4);
    else NVATTN_STORE_VEC(2);
#undef NVATTN_STORE_VEC
  } else {
    const int64_t blocks = (num_tokens + kRowWarps - 1) / kRowWarps;
    if (blocks > 0x7fffffff) return fail(NVATTN_ERR_INVALID, "store_kvcache: too many tokens");
    const dim3 grid(static_cast<unsigned>(blocks)), block(kRowWarps * 32);
#define NVATTN_STORE_ROWS(V_)                                                               \
  store_kvcache_rows_kernel<V_><<<grid, block, 0, s>>>(kp, ks, vp, vs, kc, vc, slot_mapping, \
                                                       num_tokens, row_bytes, num_slots, status)
    if (vec == 16) NVATTN_STORE_ROWS(16);
    else if (vec == 8) NVATTN_STORE_ROWS(8);
    else if (vec == 4) NVATTN_STORE_ROWS(4);
    else NVATTN_STORE_ROWS(2);
#undef NVATTN_STORE_ROWS
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "store_kvcache launch");
  return NVATTN_OK;
}

extern "C" int nvattn_kv_move(void* k_cache, void* v_cache, const int32_t* src_slots,
                              const int32_t* dst_slots, const int32_t* cu_moves,
                              int32_t num_groups, int32_t num_moves, int64_t D,
                              int64_t num_slots, int32_t* status, void* stream) {
  clear_error();
  if (num_groups < 0 || num_moves < 0 || D <= 0)
    return fail(NVATTN_ERR_INVALID, "kv_move: bad sizes");
  if (num_groups == 0) return NVATTN_OK;
  if (!k_cache || !v_cache || !src_slots || !dst_slots || !cu_moves)
    return fail(NVATTN_ERR_INVALID, "kv_move: NULL pointer");
  const int64_t row_bytes = D * 2;
  if (row_bytes % 16 || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(NVATTN_ERR_UNSUPPORTED, "kv_move: rows must be 16-byte multiples and aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  kv_move_kernel<<<num_groups, 256, 0, s>>>(static_cast<char*>(k_cache),
                                               static_cast<char*>(v_cache), src_slots, dst_slots,
                                               cu_moves, num_moves, row_bytes, num_slots, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kv_move launch");
  return NVATTN_OK;
}
