// Varlen causal prefill (dense and paged) and tree-verification attention on
// a warp-level MMA tile loop. Replaces flash_attn_varlen_func as called at
// nanovllm/layers/attention.py:64-70; the tree mode has no counterpart in the
// reference.
//
// Rows are GQA-packed: CTA (row tile m, KV head g, sequence b) owns 64 rows of
// the sequence's (query token, head-in-group) space, row R = token*group + hh,
// so one K/V tile in shared memory serves every query head of the group.
// A producer warp streams 64-key K/V tiles with TMA (3-D map over the dense
// K/V projections, or 4-D map over the paged cache; 128-byte swizzle; no
// multicast) into a 3-stage mbarrier ring; four consumer warps own 16 rows
// each and run S = Q K^T, the masked online softmax (fp32, exp2 domain) and
// O += P V with mma.m16n8k16 (bf16 in, fp32 accumulate).
//
// Masks (query token i of the sequence, key j):
//   dense/paged causal: j <= seqlen_k - seqlen_q + i  (bottom-right aligned)
//   tree:               j <  context_len, or bit (j - context_len) of the
//                       row's tree_mask word is set
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace nvattn {

namespace mma_attn {

constexpr int kTile = 64;
constexpr int kStages = 3;
constexpr int kHalfBytes = kTile * 128;
constexpr int kStageBytes = 4 * kHalfBytes;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kRows = kConsumerWarps * 16;

enum Mode { kDense = 0, kPaged = 1, kTree = 2 };

struct Params {
  const __nv_bfloat16* q;
  int64_t q_stride_tok, q_stride_head;
  __nv_bfloat16* out;
  int64_t o_stride_tok, o_stride_head;
  const int32_t* cu_q;
  const int32_t* cu_k;       // dense/paged
  const int32_t* ctx_lens;   // tree
  const uint64_t* tree_mask; // tree
  const int32_t* block_table;
  int64_t bt_stride;
  int32_t num_blocks, block_size, num_heads, num_kv_heads, group;
  int32_t max_blocks;  // block-table width (paged/tree)
  int64_t total_q;     // rows of q/out: sequences never reach past it
  int32_t causal;
  float scale_log2;
  int32_t* status;
};

template <int MODE>
__global__ void __launch_bounds__(kThreads, 2)
    attn_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap, const Params p) {
  const int b = blockIdx.z;
  const int g = blockIdx.y;
  const int m = gridDim.x - 1 - blockIdx.x;  // heaviest (latest) row tiles first
  const int q_begin = p.cu_q[b];
  int Lq = p.cu_q[b + 1] - q_begin;
  if (q_begin < 0 || q_begin > p.total_q) return;
  if (q_begin + static_cast<int64_t>(Lq) > p.total_q) Lq = static_cast<int>(p.total_q - q_begin);
  if (Lq <= 0) return;
  int Lk, k_begin = 0, ctx = 0;
  if (MODE == kTree) {
    ctx = p.ctx_lens[b];
    Lk = ctx + Lq;
  } else {
    k_begin = p.cu_k[b];
    Lk = p.cu_k[b + 1] - k_begin;
  }
  if (MODE != kDense && Lk > p.max_blocks * p.block_size) {
    // keys past the block table cannot be located: keep the visible prefix
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(p.status, NVATTN_STATUS_BAD_BLOCK);
    const int cut = Lk - p.max_blocks * p.block_size;
    Lk -= cut;
    if (MODE == kTree) ctx = max(0, ctx - cut);
  }
  const int group = p.group;
  const int rows = Lq * group;
  const int row0 = m * kRows;
  if (row0 >= rows) return;
  const int tok_hi = min(Lq - 1, (row0 + kRows - 1) / group);
  const int diag = Lk - Lq;  // causal: token i sees keys j <= diag + i
  int kend;
  if (MODE == kTree)
    kend = Lk;
  else
    kend = p.causal ? min(Lk, diag + tok_hi + 1) : Lk;
  const int ntiles = kend > 0 ? (kend + kTile - 1) / kTile : 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      prefetch_tensor_map(&kmap);
      prefetch_tensor_map(&vmap);
      const int32_t* bt =
          (MODE == kDense) ? nullptr : p.block_table + static_cast<int64_t>(b) * p.bt_stride;
      for (int it = 0; it < ntiles; ++it) {
        const int stage = it % kStages;
        const uint32_t phase = (it / kStages) & 1;
        if (!mbar_wait(&empty[stage], phase ^ 1)) {
          set_status(p.status, NVATTN_STATUS_TIMEOUT);
          break;
        }
        const int j0 = it * kTile;
        uint8_t* st = smem + stage * kStageBytes;
        mbar_arrive_expect_tx(&full[stage], kStageBytes);
        if (MODE == kDense) {
          const int row = k_begin + j0;
          tma_load_3d(st, &kmap, &full[stage], 0, g, row);
          tma_load_3d(st + kHalfBytes, &kmap, &full[stage], 64, g, row);
          tma_load_3d(st + 2 * kHalfBytes, &vmap, &full[stage], 0, g, row);
          tma_load_3d(st + 3 * kHalfBytes, &vmap, &full[stage], 64, g, row);
        } else {
          int blk = bt[j0 / p.block_size];
          if (blk < 0 || blk >= p.num_blocks) {
            set_status(p.status, NVATTN_STATUS_BAD_BLOCK);
            blk = 0;
          }
          const int tin = j0 % p.block_size;
          tma_load_4d(st, &kmap, &full[stage], 0, g, tin, blk);
          tma_load_4d(st + kHalfBytes, &kmap, &full[stage], 64, g, tin, blk);
          tma_load_4d(st + 2 * kHalfBytes, &vmap, &full[stage], 0, g, tin, blk);
          tma_load_4d(st + 3 * kHalfBytes, &vmap, &full[stage], 64, g, tin, blk);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int quad = lane & 3;
  const int r_a = row0 + warp * 16 + (lane >> 2);  // packed rows of this thread
  const int r_b = r_a + 8;
  const bool va = r_a < rows, vb = r_b < rows;
  const int ia = r_a / group, ha = r_a % group;
  const int ib = r_b / group, hb = r_b % group;
  const int warp_row_hi = min(rows - 1, row0 + warp * 16 + 15);
  const bool warp_live = row0 + warp * 16 < rows;
  const int warp_tok_hi = warp_row_hi / group;
  const int warp_tok_lo = (row0 + warp * 16) / group;
  int warp_kend;  // keys this warp can see
  if (MODE == kTree)
    warp_kend = Lk;
  else
    warp_kend = p.causal ? min(Lk, diag + warp_tok_hi + 1) : Lk;
  // First key at which some row of this warp is masked.
  int mask_from;
  if (MODE == kTree)
    mask_from = ctx;
  else
    mask_from = p.causal ? min(Lk, diag + warp_tok_lo + 1) : Lk;

  uint64_t mw_a = 0, mw_b = 0;
  if (MODE == kTree) {
    if (va) mw_a = p.tree_mask[q_begin + ia];
    if (vb) mw_b = p.tree_mask[q_begin + ib];
  }
  // key limits for the causal modes (inclusive); invalid rows see nothing
  const int lim_a = va ? ((MODE != kTree && p.causal) ? min(Lk - 1, diag + ia) : Lk - 1) : -1;
  const int lim_b = vb ? ((MODE != kTree && p.causal) ? min(Lk - 1, diag + ib) : Lk - 1) : -1;

  uint32_t qa[8][4];
  {
    const int hq_a = g * group + ha, hq_b = g * group + hb;
    const uint32_t* qra = reinterpret_cast<const uint32_t*>(
        p.q + static_cast<int64_t>(q_begin + (va ? ia : 0)) * p.q_stride_tok +
        static_cast<int64_t>(hq_a) * p.q_stride_head);
    const uint32_t* qrb = reinterpret_cast<const uint32_t*>(
        p.q + static_cast<int64_t>(q_begin + (vb ? ib : 0)) * p.q_stride_tok +
        static_cast<int64_t>(hq_b) * p.q_stride_head);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 8 + quad;
      qa[kk][0] = va ? qra[c] : 0u;
      qa[kk][1] = vb ? qrb[c] : 0u;
      qa[kk][2] = va ? qra[c + 4] : 0u;
      qa[kk][3] = vb ? qrb[c + 4] : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

  bool timed_out = false;
  for (int it = 0; it < ntiles; ++it) {
    const int stage = it % kStages;
    const uint32_t phase = (it / kStages) & 1;
    if (!mbar_wait(&full[stage], phase)) {
      timed_out = true;
      break;
    }
    const int j0 = it * kTile;
    if (warp_live && j0 < warp_kend) {
      const uint32_t kbase = smem_u32(smem + stage * kStageBytes);
      const uint32_t vbase = kbase + 2 * kHalfBytes;
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
      {
        const int mi = lane >> 3;
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of n8 tiles (16 keys)
          const int row = np * 16 + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t half = (kk >> 2) * kHalfBytes;
            const int chunk = ((kk & 3) << 1) + (mi & 1);
            uint32_t b00, b01, b10, b11;
            ldmatrix_x4(kbase + half + swz128(row, chunk), b00, b01, b10, b11);
            mma_bf16_16816(s[2 * np], qa[kk], b00, b01);
            mma_bf16_16816(s[2 * np + 1], qa[kk], b10, b11);
          }
        }
      }
      const bool need_mask = (j0 + kTile > mask_from) || !va || !vb;
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = j0 + n * 8 + quad * 2 + e;
          bool oka = true, okb = true;
          if (need_mask) {
            if (MODE == kTree) {
              const int t = j - ctx;
              oka = va && (t < 0 || (t < Lq && ((mw_a >> t) & 1ull)));
              okb = vb && (t < 0 || (t < Lq && ((mw_b >> t) & 1ull)));
            } else {
              oka = j <= lim_a;
              okb = j <= lim_b;
            }
          }
          s[n][e] = oka ? s[n][e] * p.scale_log2 : -INFINITY;
          s[n][2 + e] = okb ? s[n][2 + e] * p.scale_log2 : -INFINITY;
          mx_a = fmaxf(mx_a, s[n][e]);
          mx_b = fmaxf(mx_b, s[n][2 + e]);
        }
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      // A row with no visible key yet keeps max -inf: use 0 as the base so
      // exp2 sees -inf (-> 0) rather than NaN.
      const float base_a = (mn_a == -INFINITY) ? 0.f : mn_a;
      const float base_b = (mn_b == -INFINITY) ? 0.f : mn_b;
      const float al_a = fast_exp2(m_a - base_a), al_b = fast_exp2(m_b - base_b);
      m_a = mn_a;
      m_b = mn_b;
      float ps_a = 0.f, ps_b = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[n][e] = fast_exp2(s[n][e] - base_a);
          s[n][2 + e] = fast_exp2(s[n][2 + e] - base_b);
          ps_a += s[n][e];
          ps_b += s[n][2 + e];
        }
      }
      l_a = l_a * al_a + ps_a;
      l_b = l_b * al_b + ps_b;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= al_a;
        o[j][1] *= al_a;
        o[j][2] *= al_b;
        o[j][3] *= al_b;
      }
      // Keys at or past kend may be stale cache bytes (maybe NaN): zero their
      // V elements; all other masked keys hold finite data and get P = 0.
      const int vlim = kend - j0;  // keys [0, vlim) of this tile are real
      {
        const int mi = lane >> 3;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
          uint32_t pa[4];
          pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
          pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
          pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
          pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
          const int t_lo = kk * 16 + quad * 2;
          const uint32_t mlo = (t_lo + 16 <= vlim)
                                   ? 0xffffffffu
                                   : ((t_lo < vlim ? 0x0000ffffu : 0u) |
                                      (t_lo + 1 < vlim ? 0xffff0000u : 0u));
          const uint32_t mhi = (t_lo + 16 <= vlim)
                                   ? 0xffffffffu
                                   : ((t_lo + 8 < vlim ? 0x0000ffffu : 0u) |
                                      (t_lo + 9 < vlim ? 0xffff0000u : 0u));
          const int row = kk * 16 + ((mi & 1) << 3) + (lane & 7);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const uint32_t half = (jj >> 2) * kHalfBytes;
            const int chunk = ((jj & 3) << 1) + (mi >> 1);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(vbase + half + swz128(row, chunk), b0, b1, b2, b3);
            mma_bf16_16816(o[2 * jj], pa, b0 & mlo, b1 & mhi);
            mma_bf16_16816(o[2 * jj + 1], pa, b2 & mlo, b3 & mhi);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
  if (timed_out && lane == 0) set_status(p.status, NVATTN_STATUS_TIMEOUT);

  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  __nv_bfloat16* oa = p.out + static_cast<int64_t>(q_begin + ia) * p.o_stride_tok +
                      static_cast<int64_t>(g * group + ha) * p.o_stride_head;
  __nv_bfloat16* ob = p.out + static_cast<int64_t>(q_begin + ib) * p.o_stride_tok +
                      static_cast<int64_t>(g * group + hb) * p.o_stride_head;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = j * 8 + quad * 2;
    if (va)
      *reinterpret_cast<uint32_t*>(oa + d) = pack_bf16x2(o[j][0] * inv_a, o[j][1] * inv_a);
    if (vb)
      *reinterpret_cast<uint32_t*>(ob + d) = pack_bf16x2(o[j][2] * inv_b, o[j][3] * inv_b);
  }
}

int make_dense_map(CUtensorMap* map, const void* base, int64_t total, int num_kv_heads,
                   int64_t stride_tok, int64_t stride_head) {
  const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(num_kv_heads),
                            static_cast<uint64_t>(total)};
  const uint64_t strides[2] = {static_cast<uint64_t>(stride_head) * 2,
                               static_cast<uint64_t>(stride_tok) * 2};
  const uint32_t box[3] = {64, 1, static_cast<uint32_t>(kTile)};
  return make_tensor_map(map, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace mma_attn

int make_cache_map(CUtensorMap* map, const void* cache, int num_blocks, int block_size,
                   int num_kv_heads);

static int set_smem_attr_once(const void* fn, int bytes, int slot) {
  static int done[8][64] = {{0}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && done[slot][dev] >= bytes) return NVATTN_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  if (dev < 64) done[slot][dev] = bytes;
  return NVATTN_OK;
}

template <int MODE>
static int launch_mma(const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const mma_attn::Params& p, int num_seqs, int max_rows,
                      cudaStream_t stream) {
  using namespace mma_attn;
  const int smem = kStages * kStageBytes + 1024 + 2 * kStages * 8;
  int rc = set_smem_attr_once(reinterpret_cast<const void*>(attn_mma_kernel<MODE>), smem, MODE);
  if (rc) return rc;
  const int mtiles = (max_rows + kRows - 1) / kRows;
  if (mtiles <= 0) return NVATTN_OK;
  if (num_seqs > 65535) return fail(NVATTN_ERR_UNSUPPORTED, "more than 65535 sequences");
  dim3 grid(mtiles, p.num_kv_heads, num_seqs);
  attn_mma_kernel<MODE><<<grid, kThreads, smem, stream>>>(kmap, vmap, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention kernel launch");
  return NVATTN_OK;
}

static int check_common(const void* q, int64_t q_stride_tok, int64_t q_stride_head, void* out,
                        int64_t o_stride_tok, int64_t o_stride_head, int num_heads,
                        int num_kv_heads, int head_dim, const char* who) {
  if (!q || !out) return fail(NVATTN_ERR_INVALID, std::string(who) + ": NULL q/out");
  if (head_dim != kHeadDim)
    return fail(NVATTN_ERR_UNSUPPORTED, std::string(who) + ": head_dim must be 128");
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads)
    return fail(NVATTN_ERR_INVALID,
                std::string(who) + ": num_heads must be a multiple of num_kv_heads");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(out) & 3) ||
      (q_stride_tok & 1) || (q_stride_head & 1) || (o_stride_tok & 1) || (o_stride_head & 1))
    return fail(NVATTN_ERR_UNSUPPORTED, std::string(who) + ": q/out rows must be 4-byte aligned");
  return NVATTN_OK;
}

}  // namespace nvattn

using namespace nvattn;

extern "C" int nvattn_varlen_prefill(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* k,
    int64_t k_stride_tok, int64_t k_stride_head, const void* v, int64_t v_stride_tok,
    int64_t v_stride_head, void* out, int64_t o_stride_tok, int64_t o_stride_head,
    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t num_seqs,
    int32_t max_seqlen_q, int32_t max_seqlen_k, int64_t total_q, int64_t total_k,
    const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks_per_seq,
    int32_t num_blocks, int32_t block_size, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, float softmax_scale, int32_t causal, int32_t* status, void* stream) {
  using namespace mma_attn;
  clear_error();
  if (num_seqs < 0 || total_q < 0 || total_k < 0 || max_seqlen_q < 0 || max_seqlen_k < 0)
    return fail(NVATTN_ERR_INVALID, "varlen_prefill: negative size");
  if (num_seqs == 0 || total_q == 0 || max_seqlen_q == 0) return NVATTN_OK;
  int rc = check_common(q, q_stride_tok, q_stride_head, out, o_stride_tok, o_stride_head,
                        num_heads, num_kv_heads, head_dim, "varlen_prefill");
  if (rc) return rc;
  if (!k || !v || !cu_seqlens_q || !cu_seqlens_k)
    return fail(NVATTN_ERR_INVALID, "varlen_prefill: NULL k/v/cu_seqlens");
  const int group = num_heads / num_kv_heads;
  if (group > 16)
    return fail(NVATTN_ERR_UNSUPPORTED, "varlen_prefill: more than 16 query heads per KV head");
  CUtensorMap kmap, vmap;
  if (block_table) {
    if (block_size <= 0 || block_size % kTile)
      return fail(NVATTN_ERR_UNSUPPORTED, "varlen_prefill: block_size must be a multiple of 64");
    if (num_blocks <= 0 || max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
      return fail(NVATTN_ERR_INVALID, "varlen_prefill: bad block table geometry");
    if (!aligned16(k) || !aligned16(v))
      return fail(NVATTN_ERR_INVALID, "varlen_prefill: caches must be 16-byte aligned");
    rc = make_cache_map(&kmap, k, num_blocks, block_size, num_kv_heads);
    if (rc) return rc;
    rc = make_cache_map(&vmap, v, num_blocks, block_size, num_kv_heads);
    if (rc) return rc;
  } else {
    if (total_k <= 0) return fail(NVATTN_ERR_INVALID, "varlen_prefill: total_k must be > 0");
    if (!aligned16(k) || !aligned16(v) || (k_stride_tok * 2) % 16 || (k_stride_head * 2) % 16 ||
        (v_stride_tok * 2) % 16 || (v_stride_head * 2) % 16)
      return fail(NVATTN_ERR_UNSUPPORTED,
                  "varlen_prefill: k/v base and strides must be 16-byte multiples (TMA)");
    rc = make_dense_map(&kmap, k, total_k, num_kv_heads, k_stride_tok, k_stride_head);
    if (rc) return rc;
    rc = make_dense_map(&vmap, v, total_k, num_kv_heads, v_stride_tok, v_stride_head);
    if (rc) return rc;
  }
  Params p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride_tok = q_stride_tok;
  p.q_stride_head = q_stride_head;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_stride_tok = o_stride_tok;
  p.o_stride_head = o_stride_head;
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.max_blocks = block_table ? max_blocks_per_seq : 0;
  p.total_q = total_q;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = group;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = softmax_scale * kLog2e;
  p.status = status;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int max_rows = max_seqlen_q * group;
  return block_table ? launch_mma<kPaged>(kmap, vmap, p, num_seqs, max_rows, s)
                     : launch_mma<kDense>(kmap, vmap, p, num_seqs, max_rows, s);
}

extern "C" int nvattn_tree_verify(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                  const void* k_cache, const void* v_cache, void* out,
                                  int64_t o_stride_tok, int64_t o_stride_head,
                                  const int32_t* cu_seqlens_q, const int32_t* context_lens,
                                  const uint64_t* tree_mask, const int32_t* block_table,
                                  int64_t block_table_stride, int32_t max_blocks_per_seq,
                                  int32_t num_blocks, int32_t block_size, int32_t num_seqs,
                                  int32_t max_nodes, int64_t total_q, int32_t num_heads,
                                  int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                                  int32_t* status, void* stream) {
  using namespace mma_attn;
  clear_error();
  if (num_seqs < 0 || total_q < 0 || max_nodes < 0)
    return fail(NVATTN_ERR_INVALID, "tree_verify: negative size");
  if (num_seqs == 0 || total_q == 0 || max_nodes == 0) return NVATTN_OK;
  if (max_nodes > 64) return fail(NVATTN_ERR_UNSUPPORTED, "tree_verify: at most 64 tree nodes");
  int rc = check_common(q, q_stride_tok, q_stride_head, out, o_stride_tok, o_stride_head,
                        num_heads, num_kv_heads, head_dim, "tree_verify");
  if (rc) return rc;
  if (!k_cache || !v_cache || !cu_seqlens_q || !context_lens || !tree_mask || !block_table)
    return fail(NVATTN_ERR_INVALID, "tree_verify: NULL pointer");
  const int group = num_heads / num_kv_heads;
  if (group > 16)
    return fail(NVATTN_ERR_UNSUPPORTED, "tree_verify: more than 16 query heads per KV head");
  if (block_size <= 0 || block_size % kTile)
    return fail(NVATTN_ERR_UNSUPPORTED, "tree_verify: block_size must be a multiple of 64");
  if (num_blocks <= 0 || max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
    return fail(NVATTN_ERR_INVALID, "tree_verify: bad block table geometry");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(NVATTN_ERR_INVALID, "tree_verify: caches must be 16-byte aligned");
  CUtensorMap kmap, vmap;
  rc = make_cache_map(&kmap, k_cache, num_blocks, block_size, num_kv_heads);
  if (rc) return rc;
  rc = make_cache_map(&vmap, v_cache, num_blocks, block_size, num_kv_heads);
  if (rc) return rc;
  Params p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride_tok = q_stride_tok;
  p.q_stride_head = q_stride_head;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_stride_tok = o_stride_tok;
  p.o_stride_head = o_stride_head;
  p.cu_q = cu_seqlens_q;
  p.ctx_lens = context_lens;
  p.tree_mask = tree_mask;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.max_blocks = max_blocks_per_seq;
  p.total_q = total_q;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = group;
  p.causal = 1;
  p.scale_log2 = softmax_scale * kLog2e;
  p.status = status;
  return launch_mma<kTree>(kmap, vmap, p, num_seqs, max_nodes * group,
                           reinterpret_cast<cudaStream_t>(stream));
}
