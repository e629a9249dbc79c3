// Varlen causal prefill (dense and paged / prefix-cache) and tree-verification
// attention on the 5th-generation tensor cores. Replaces flash_attn_varlen_func
// as called at nanovllm/layers/attention.py:64-70; the tree mode (EAGLE-style
// speculative verification) has no counterpart in the reference.
//
// CTA = (row block m, KV head g, sequence b). Rows are GQA-packed: row
// (token t, head-in-group hh) of the sequence is t*group + hh, so one K/V tile
// serves every query head of the group. A CTA owns two 128-row Q tiles.
//
// Warp roles (10 warps):
//   warp 0      TMA producer: both Q tiles once, then 128-key K and V tiles
//               through a 2-stage mbarrier ring (3-D map over the dense K/V
//               projections or 4-D map over the paged cache; 128-byte
//               swizzle; no multicast).
//   warp 1      owns the TMEM allocation (512 columns) and issues every
//               tcgen05.mma from one thread:
//                 S_i = Q_i K^T   (M=128, N=128 keys, K=128 dims; A and B from
//                                  shared memory, K-major)
//                 O_i += P_i V    (M=128, N=128 dims, K=128 keys; A = P from
//                                  TMEM, B = V from shared memory, MN-major)
//               ordered S0, S1, then per key tile: PV0_j, S0_{j+1}, PV1_j,
//               S1_{j+1}, so one warpgroup's softmax overlaps the other's MMAs.
//   warps 2-5   softmax warpgroup for Q tile 0, warps 6-9 for Q tile 1. A
//               thread owns one row: it reads its 128 scores from TMEM, masks
//               and scales them, keeps the row max and sum in registers, and
//               writes P (bf16 pairs) back over S in TMEM. The output is
//               rescaled only when the running max grows by more than 2^8
//               (P then stays <= 256; the final O/l is unchanged), so the
//               O read-modify-write in TMEM is rare. In tree mode a
//               warpgroup hands P over in two 64-key halves, so the P V of
//               the first half overlaps the softmax of the second.
// TMEM columns: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512).
//
// Masks (query token i of the sequence, key j):
//   causal (dense/paged): j <= seqlen_k - seqlen_q + i   (bottom-right aligned)
//   tree: j < context_len, or bit (j - context_len) of the row's mask word.
// Keys past the sequence's end in the last tile of the paged cache are stale
// bytes (maybe NaN): their scores are masked and their V rows zeroed in
// shared memory before the P V product.
// Query rows past the sequence (the last row block, short drafts) are never
// written: a warp with no valid row skips its softmax entirely, and inside a
// live warp such rows take the unmasked path (rows are independent in both
// MMAs, so their values cannot reach a valid row).
#include <algorithm>
#include <cmath>
#include <mutex>

#include "sm100.cuh"

namespace nvattn {
namespace tc {

constexpr int kBM = 128;                 // rows per Q tile
constexpr int kBN = 128;                 // keys per K/V tile
constexpr int kHalf = 128 * 128;         // 128 rows x 128 B (64 bf16) = 16 KB
constexpr int kOperand = 2 * kHalf;      // one 128 x 128 bf16 operand = 32 KB
constexpr int kStages = 2;
constexpr int kQBytes = 2 * kOperand;                       // Q0, Q1
constexpr int kRingBytes = kStages * 2 * kOperand;          // K and V per stage
constexpr int kSmemData = kQBytes + kRingBytes;             // 192 KB
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
// TMEM column of S_i (later P_i) and O_i
__device__ __forceinline__ uint32_t col_s(int i) { return static_cast<uint32_t>(i) * 128u; }
__device__ __forceinline__ uint32_t col_o(int i) { return 256u + static_cast<uint32_t>(i) * 128u; }
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale when max grows by > 2^8
// Lean tiles take 1 exp2 pair in this many from the FMA-pipe polynomial instead
// of MUFU (measured: prefill 785/875/896/890/895 TFLOP/s and tree 724/760/763/
// 779/781 for 1 in 2/3/4/6/8; the tree's two passes leave the FMA pipe busier).
constexpr int kPolyEveryPrefill = 4;
constexpr int kPolyEveryTree = 8;
#ifndef NVATTN_L2_PREFETCH_TILES
#define NVATTN_L2_PREFETCH_TILES 3
#endif
constexpr int kPrefetch = NVATTN_L2_PREFETCH_TILES;  // key tiles of L2 prefetch ahead of the ring

enum Mode { kDense = 0, kPaged = 1, kTree = 2 };


struct Params {
  __nv_bfloat16* out;
  int64_t o_stride_tok, o_stride_head;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* ctx_lens;
  const uint64_t* tree_mask;
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t total_q;
  int32_t max_blocks, num_blocks, block_size, num_kv_heads, group;
  int32_t tpt;  // query tokens per Q tile (floor(128 / group))
  int32_t rpt;  // rows per Q tile (group * tpt <= 128)
  int32_t causal;
  int32_t out_vec16;  // output rows 16-byte aligned
  float scale_log2;
  int32_t* status;
  // Split of the key range over CTAs (tree mode): split s covers key tiles
  // [s*split_tiles, (s+1)*split_tiles); with nsplit > 1 every CTA writes an
  // fp32 partial (unnormalised O, reference max, sum) per row to ws_o/ws_ml
  // and tree_combine_kernel merges them.
  int32_t nsplit, split_tiles, num_heads;
  float* ws_o;    // [total_q][num_heads][nsplit][128]
  float2* ws_ml;  // [total_q][num_heads][nsplit]
  // Tree mode: sequences in decreasing key count (written by
  // tree_order_kernel), so CTAs are dispatched longest first; null = in order.
  const int32_t* order;
};

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t p_half[2];  // first 64 keys of P written (tree mode)
  uint64_t o_done;
  uint32_t tmem_base;
};

__device__ __forceinline__ uint64_t kdesc(uint32_t base, int kk) {
  // K-major operand (Q or K): 16-dim step kk lives in half kk/4 at +32*(kk%4) B.
  return sm100::sw128_desc(base + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}

__device__ __forceinline__ uint64_t vdesc(uint32_t base, int kk) {
  // MN-major V: 16-key step kk starts at row 16*kk; the two 64-dim halves are
  // kHalf apart (leading byte offset), 8-row groups 1024 B apart (stride).
  return sm100::sw128_desc(base + kk * 16 * 128, kHalf, 1024);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                   const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const Params p) {
  if (MODE == kTree) {
    // launched as a programmatic dependent of tree_order_kernel: nothing
    // below may be read before that grid (and all earlier work) completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }
  const int b = (MODE == kTree && p.order != nullptr) ? p.order[blockIdx.z] : blockIdx.z;
  const int g = blockIdx.y;
  const int split = blockIdx.x % p.nsplit;
  const int m = gridDim.x / p.nsplit - 1 - blockIdx.x / p.nsplit;  // heaviest row blocks first
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Tree mode hands P to the MMA warp in two 64-key halves, so the P V of the
  // first half overlaps the softmax of the second (measured: +4% on tree,
  // -2% on prefill, which keeps one hand-off).
  constexpr bool kSplitP = MODE == kTree;
  constexpr int kPolyEvery = MODE == kTree ? kPolyEveryTree : kPolyEveryPrefill;

  // ------------------------------------------------ sequence geometry
  const int q_begin = p.cu_q[b];
  int Lq = p.cu_q[b + 1] - q_begin;
  if (q_begin < 0 || q_begin > p.total_q) return;
  if (q_begin + static_cast<int64_t>(Lq) > p.total_q) Lq = static_cast<int>(p.total_q - q_begin);
  int Lk, k_begin = 0, ctx = 0;
  if (MODE == kTree) {
    ctx = p.ctx_lens[b];
    Lk = ctx + Lq;
  } else {
    k_begin = p.cu_k[b];
    Lk = p.cu_k[b + 1] - k_begin;
  }
  if (MODE != kDense && Lk > p.max_blocks * p.block_size) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(p.status, NVATTN_STATUS_BAD_BLOCK);
    const int cut = Lk - p.max_blocks * p.block_size;
    Lk -= cut;
    if (MODE == kTree) ctx = max(0, ctx - cut);
  }
  const int group = p.group;
  const int tok0 = m * 2 * p.tpt;  // first query token of this CTA
  if (Lq <= 0 || tok0 >= Lq) return;
  const int tok_hi = min(Lq - 1, tok0 + 2 * p.tpt - 1);
  const int diag = Lk - Lq;
  int kend;
  if (MODE == kTree)
    kend = Lk;
  else
    kend = p.causal ? min(Lk, diag + tok_hi + 1) : Lk;
  const int ntiles_all = kend > 0 ? (kend + kBN - 1) / kBN : 0;
  const int jb = split * p.split_tiles;  // first key tile of this CTA's split
  const int ntiles = max(0, min(ntiles_all, jb + p.split_tiles) - jb);
  if (p.nsplit > 1 && ntiles == 0) return;  // split past the keys: the merge skips it

  if (ntiles == 0) {
    // No visible key for any row of this CTA: the rows are zeros.
    for (int e = threadIdx.x; e < 2 * p.rpt * (kHeadDim / 8); e += blockDim.x) {
      const int r = e / (kHeadDim / 8), c = e % (kHeadDim / 8);
      const int tok = tok0 + (r / p.rpt) * p.tpt + (r % p.rpt) / group;
      if (tok >= Lq || tok > tok0 + 2 * p.tpt - 1) continue;
      __nv_bfloat16* o = p.out + static_cast<int64_t>(q_begin + tok) * p.o_stride_tok +
                         static_cast<int64_t>(g * group + (r % p.rpt) % group) * p.o_stride_head;
      for (int d = 0; d < 8; ++d) o[c * 8 + d] = __float2bfloat16_rn(0.f);
    }
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kSmemData);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_s[2] = {sbase, sbase + kOperand};
  auto k_s = [&](int st) { return sbase + kQBytes + st * 2 * kOperand; };
  auto v_s = [&](int st) { return sbase + kQBytes + st * 2 * kOperand + kOperand; };

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 4);
      mbar_init(&bars->p_half[i], 4);
    }
    mbar_init(&bars->o_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(&bars->tmem_base, kTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::fence_before_sync();
  __syncthreads();
  sm100::fence_after_sync();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensor_map(&qmap);
      prefetch_tensor_map(&kmap);
      prefetch_tensor_map(&vmap);
      const uint32_t qbytes = 2u * 2u * static_cast<uint32_t>(p.rpt) * 128u;
      mbar_arrive_expect_tx(&bars->q_full, qbytes);
      for (int i = 0; i < 2; ++i) {
        const int row = q_begin + tok0 + i * p.tpt;
        tma_load_3d(smem + i * kOperand, &qmap, &bars->q_full, 0, g * group, row);
        tma_load_3d(smem + i * kOperand + kHalf, &qmap, &bars->q_full, 64, g * group, row);
      }
      const int32_t* bt =
          (MODE == kDense) ? nullptr : p.block_table + static_cast<int64_t>(b) * p.bt_stride;
      int issued = 0;
      bool ok = true;
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % kStages;
        const uint32_t par = ((j / kStages) & 1) ^ 1;
        const int j0 = (jb + j) * kBN;
        uint8_t* kd = smem + kQBytes + st * 2 * kOperand;
        uint8_t* vd = kd + kOperand;
        int c2 = 0, c3 = 0;  // token coordinate / block coordinate of the tile
        if (MODE == kDense) {
          c2 = k_begin + j0;
        } else {
          int blk = bt[j0 / p.block_size];
          if (blk < 0 || blk >= p.num_blocks) {
            set_status(p.status, NVATTN_STATUS_BAD_BLOCK);
            blk = 0;
          }
          c2 = j0 % p.block_size;
          c3 = blk;
        }
        // Warm L2 with the tile kPrefetch ahead: the ring holds one tile of
        // lookahead, far less than the HBM latency of a cold paged tile.
        if (j + kPrefetch < ntiles) {
          const int pj0 = (jb + j + kPrefetch) * kBN;
          if (MODE == kDense) {
            const int pc2 = k_begin + pj0;
            tma_prefetch_3d(&kmap, 0, g, pc2);
            tma_prefetch_3d(&kmap, 64, g, pc2);
            tma_prefetch_3d(&vmap, 0, g, pc2);
            tma_prefetch_3d(&vmap, 64, g, pc2);
          } else {
            const int pblk = bt[pj0 / p.block_size];
            if (pblk >= 0 && pblk < p.num_blocks) {
              const int pc2 = pj0 % p.block_size;
              tma_prefetch_4d(&kmap, 0, g, pc2, pblk);
              tma_prefetch_4d(&kmap, 64, g, pc2, pblk);
              tma_prefetch_4d(&vmap, 0, g, pc2, pblk);
              tma_prefetch_4d(&vmap, 64, g, pc2, pblk);
            }
          }
        }
        // K ring slot frees after S1 of the tile two back; V after its PV1.
        if (!mbar_wait(&bars->k_empty[st], par)) { ok = false; break; }
        mbar_arrive_expect_tx(&bars->k_full[st], kOperand);
        if (MODE == kDense) {
          tma_load_3d(kd, &kmap, &bars->k_full[st], 0, g, c2);
          tma_load_3d(kd + kHalf, &kmap, &bars->k_full[st], 64, g, c2);
        } else {
          tma_load_4d(kd, &kmap, &bars->k_full[st], 0, g, c2, c3);
          tma_load_4d(kd + kHalf, &kmap, &bars->k_full[st], 64, g, c2, c3);
        }
        if (!mbar_wait(&bars->v_empty[st], par)) { ok = false; issued = -(j + 1); break; }
        mbar_arrive_expect_tx(&bars->v_full[st], kOperand);
        if (MODE == kDense) {
          tma_load_3d(vd, &vmap, &bars->v_full[st], 0, g, c2);
          tma_load_3d(vd + kHalf, &vmap, &bars->v_full[st], 64, g, c2);
        } else {
          tma_load_4d(vd, &vmap, &bars->v_full[st], 0, g, c2, c3);
          tma_load_4d(vd + kHalf, &vmap, &bars->v_full[st], 64, g, c2, c3);
        }
        issued = j + 1;
      }
      if (!ok) set_status(p.status, NVATTN_STATUS_TIMEOUT);
      // Drain: no copy of ours may still be in flight when the CTA ends. The
      // last use of each ring slot is the last phase that barrier completes.
      mbar_wait(&bars->q_full, 0);
      const int k_issued = issued < 0 ? -issued : issued;  // K of tile |issued|-1 went out
      const int v_issued = issued < 0 ? -issued - 1 : issued;
      for (int j = max(0, k_issued - kStages); j < k_issued; ++j)
        mbar_wait(&bars->k_full[j % kStages], (j / kStages) & 1);
      for (int j = max(0, v_issued - kStages); j < v_issued; ++j)
        mbar_wait(&bars->v_full[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc_s = sm100::idesc_bf16_f32(kBM, kBN, false);
      constexpr uint32_t idesc_o = sm100::idesc_bf16_f32(kBM, kHeadDim, true);
      bool ok = mbar_wait(&bars->q_full, 0);
      auto issue_s = [&](int i, int st) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          sm100::mma_ss(tmem + col_s(i), kdesc(q_s[i], kk), kdesc(k_s(st), kk), idesc_s,
                        kk > 0 ? 1u : 0u);
        sm100::commit(&bars->s_full[i]);
      };
      auto issue_pv = [&](int i, int st, int j, int k0, int k1) {
#pragma unroll
        for (int kk = k0; kk < k1; ++kk)
          sm100::mma_ts(tmem + col_o(i), tmem + col_s(i) + kk * 8, vdesc(v_s(st), kk), idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
      };
      if (ok) ok = mbar_wait(&bars->k_full[0], 0);
      if (ok) {
        sm100::fence_after_sync();
        issue_s(0, 0);
        issue_s(1, 0);
        sm100::commit(&bars->k_empty[0]);
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % kStages;
        const int nst = (j + 1) % kStages;
        const bool more = j + 1 < ntiles;
        if (kSplitP) {
          ok = mbar_wait(&bars->p_half[0], j & 1) &&
               mbar_wait(&bars->v_full[st], (j / kStages) & 1);
          if (!ok) break;
          sm100::fence_after_sync();
          issue_pv(0, st, j, 0, 4);
          ok = mbar_wait(&bars->p_full[0], j & 1);
          if (!ok) break;
          sm100::fence_after_sync();
          issue_pv(0, st, j, 4, 8);
        } else {
          ok = mbar_wait(&bars->p_full[0], j & 1) &&
               mbar_wait(&bars->v_full[st], (j / kStages) & 1);
          if (!ok) break;
          sm100::fence_after_sync();
          issue_pv(0, st, j, 0, 8);
        }
        if (more) {
          ok = mbar_wait(&bars->k_full[nst], ((j + 1) / kStages) & 1);
          if (!ok) break;
          sm100::fence_after_sync();
          issue_s(0, nst);
        }
        if (kSplitP) {
          ok = mbar_wait(&bars->p_half[1], j & 1);
          if (!ok) break;
          sm100::fence_after_sync();
          issue_pv(1, st, j, 0, 4);
        }
        ok = mbar_wait(&bars->p_full[1], j & 1);
        if (!ok) break;
        sm100::fence_after_sync();
        issue_pv(1, st, j, kSplitP ? 4 : 0, 8);
        sm100::commit(&bars->v_empty[st]);
        if (more) {
          issue_s(1, nst);
          sm100::commit(&bars->k_empty[nst]);
        }
      }
      if (!ok) set_status(p.status, NVATTN_STATUS_TIMEOUT);
      // All MMAs done -> O final; also makes sure none is in flight at exit.
      sm100::commit(&bars->o_done);
      mbar_wait(&bars->o_done, 0);
    }
  } else {
    // ----------------------------------------------------------- softmax
    const int wg = (warp - 2) >> 2;            // Q tile 0 or 1
    const int quarter = warp & 3;              // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;         // row inside the Q tile
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int tok = tok0 + wg * p.tpt + r / group;
    const int hh = r % group;
    const bool valid = r < p.rpt && tok < Lq;
    const int lim = valid ? ((MODE != kTree && p.causal) ? min(Lk - 1, diag + tok) : Lk - 1) : -1;
    uint64_t mword = 0;
    if (MODE == kTree && valid) mword = p.tree_mask[q_begin + tok];
    // first key index at which this row needs masking
    const int mask_from = !valid ? 0 : (MODE == kTree ? ctx : lim + 1);
    // A warp whose rows all lie past the sequence (short drafts, the last row
    // block) computes nothing: its P and O rows are never read. It still
    // zeroes its share of the stale V rows and hands the tile on.
    const bool warp_live = __any_sync(0xffffffffu, valid);

    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      // warp-uniform: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[wg], j & 1))) {
        ok = false;
        break;
      }
      sm100::fence_after_sync();
      const int j0 = (jb + j) * kBN;
      if (!warp_live) {
        if (MODE != kDense && wg == 0 && j == ntiles - 1 && kend - j0 < kBN) {
          const int vlim = kend - j0;
          __all_sync(0xffffffffu, mbar_wait(&bars->v_full[j % kStages], (j / kStages) & 1));
          if (r >= vlim) {
            uint8_t* vrow = smem + kQBytes + (j % kStages) * 2 * kOperand + kOperand + r * 128;
            const int4 z = make_int4(0, 0, 0, 0);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              reinterpret_cast<int4*>(vrow)[c] = z;
              reinterpret_cast<int4*>(vrow + kHalf)[c] = z;
            }
          }
          fence_proxy_async();
        }
        __syncwarp();
        if (lane == 0) {
          if (kSplitP) mbar_arrive(&bars->p_half[wg]);
          mbar_arrive(&bars->p_full[wg]);
        }
        continue;
      }
      // no key of this tile is masked; rows past the sequence count as
      // unmasked (their P and O rows are never read)
      const bool full_row = !valid || j0 + kBN <= mask_from;
      // Raw score or -inf where masked (scale is applied later: it is > 0).
      auto masked = [&](uint32_t raw, int key) -> float {
        const float x = __uint_as_float(raw);
        bool okk;
        if (MODE == kTree) {
          const int t = key - ctx;
          okk = valid && (t < 0 || (t < Lq && ((mword >> t) & 1ull)));
        } else {
          okk = key <= lim;
        }
        return okk ? x : -INFINITY;
      };
      // Tiles where no row of the warp is masked take the lean path.
      const bool wfull = __all_sync(0xffffffffu, full_row);
      // The last paged tile may hold stale rows whose V this warpgroup zeroes:
      // that tile always takes the two passes below.
      const bool zero_v_tile = MODE != kDense && j == ntiles - 1 && kend - j0 < kBN;
      // Single pass (prefill modes): on a lean tile after the row's first,
      // the exponentials are taken against the current reference max while
      // the tile's max is found, with P kept in registers until the max is
      // known. If no row of the warp grew its max by more than the rescale
      // threshold (the usual case once a row has seen a few tiles), those P
      // are exactly what the two passes below compute (same FMA, same exp2
      // split) and they are stored; otherwise the warp redoes the tile in the
      // two passes, from S, which nothing has overwritten yet. Tree mode
      // keeps the two passes: it hands the first 64 keys of P to the MMA warp
      // before the second 64 are computed, which a deferred store would undo.
      if (!kSplitP && wfull && !zero_v_tile &&
          __all_sync(0xffffffffu, m_used != -INFINITY || !valid)) {
        const float base1 = (m_used == -INFINITY) ? 0.f : m_used;  // rows past the sequence
        const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2);
        const uint64_t nbase2 = pack_f32x2(-base1, -base1);
        uint64_t sum2[2] = {pack_f32x2(0.f, 0.f), pack_f32x2(0.f, 0.f)};
        float mx2[2] = {-INFINITY, -INFINITY};
        uint32_t pk[64];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          uint32_t sr[32];
          sm100::tmem_ld32(t_lane + col_s(wg) + qq * 32, sr);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int ee = qq * 16 + e;  // pair index in the tile, 0..63
            const uint64_t x2 = fma_f32x2((static_cast<uint64_t>(sr[2 * e + 1]) << 32) | sr[2 * e],
                                          scale2, nbase2);
            const float2 xx = unpack_f32x2(x2);
            mx2[e & 1] = fmax3(mx2[e & 1], xx.x, xx.y);
            const uint64_t p2 = ((ee & 31) % kPolyEvery == kPolyEvery - 1) ? exp2_poly_f32x2(x2)
                                                                           : exp2_mufu_f32x2(x2);
            sum2[e & 1] = add_f32x2(sum2[e & 1], p2);
            const float2 pp = unpack_f32x2(p2);
            pk[ee] = pack_bf16x2(pp.x, pp.y);
          }
        }
        const float grow = fmaxf(mx2[0], mx2[1]);
        if (!__any_sync(0xffffffffu, valid && grow > kRescaleThreshold)) {
          sm100::tmem_st32(t_lane + col_s(wg), pk);
          sm100::tmem_st32(t_lane + col_s(wg) + 32, pk + 32);
          const float2 sm = unpack_f32x2(add_f32x2(sum2[0], sum2[1]));
          l += sm.x + sm.y;
          sm100::tmem_wait_st();
          sm100::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->p_full[wg]);
          continue;
        }
      }
      // Pass 1: row max of the raw scores, 64 columns per TMEM round trip,
      // in four independent chains (a single chain is 64 dependent maxes).
      float mr4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sr[64];
        sm100::tmem_ld32(t_lane + col_s(wg) + h * 64, sr);
        sm100::tmem_ld32(t_lane + col_s(wg) + h * 64 + 32, sr + 32);
        sm100::tmem_wait_ld();
        if (wfull) {
#pragma unroll
          for (int e = 0; e < 64; e += 2)
            mr4[(e >> 1) & 3] =
                fmax3(mr4[(e >> 1) & 3], __uint_as_float(sr[e]), __uint_as_float(sr[e + 1]));
        } else {
#pragma unroll
          for (int e = 0; e < 64; e += 2)
            mr4[(e >> 1) & 3] = fmax3(mr4[(e >> 1) & 3], masked(sr[e], j0 + h * 64 + e),
                                      masked(sr[e + 1], j0 + h * 64 + e + 1));
        }
      }
      // rows past the sequence never move their reference max (no rescales)
      const float mraw = valid ? fmaxf(fmaxf(mr4[0], mr4[1]), fmaxf(mr4[2], mr4[3])) : -INFINITY;
      const float mx = (mraw == -INFINITY) ? -INFINITY : mraw * p.scale_log2;
      // Lazy rescale: keep the reference max unless the row max grew by > 2^8.
      float alpha = 1.f;
      bool need = false;
      if (mx > m_used + kRescaleThreshold) {
        need = (m_used != -INFINITY);  // nothing accumulated yet otherwise
        alpha = need ? fast_exp2(m_used - mx) : 1.f;
        m_used = mx;
        l *= alpha;
      }
      if (kSplitP) {
        // O rescale and stale-V zeroing before any P is handed over: the P V
        // of the first half may start while the second half is computed.
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          uint32_t orr[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            sm100::tmem_ld32(t_lane + col_o(wg) + c * 32, orr);
            sm100::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e)
              orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
            sm100::tmem_st32(t_lane + col_o(wg) + c * 32, orr);
          }
        }
        if (MODE != kDense && wg == 0 && j == ntiles - 1 && kend - j0 < kBN) {
          // Stale cache rows past the end of the sequence: zero their V so that
          // 0 * NaN cannot reach O. Every tile row r is one 128-byte line in
          // each half. V_j must have landed first, or its TMA write would
          // overwrite the zeros (the slot's previous tile is already consumed:
          // its P V was issued before S0_j, whose completion brought us here).
          const int vlim = kend - j0;
          __all_sync(0xffffffffu, mbar_wait(&bars->v_full[j % kStages], (j / kStages) & 1));
          if (r >= vlim) {
            uint8_t* vrow = smem + kQBytes + (j % kStages) * 2 * kOperand + kOperand + r * 128;
            const int4 z = make_int4(0, 0, 0, 0);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              reinterpret_cast<int4*>(vrow)[c] = z;
              reinterpret_cast<int4*>(vrow + kHalf)[c] = z;
            }
          }
          fence_proxy_async();
        }
      }
      const float base = (m_used == -INFINITY) ? 0.f : m_used;
      // Pass 2: P = exp2(raw*scale - base), two columns per packed fp32x2 FMA,
      // written over S as bf16 pairs. Columns 64h..64h+63 of S become P
      // columns 32h..32h+31, which only overlap S columns already read.
      // In lean tiles one pair in kPolyEvery takes exp2 from a polynomial on
      // the FMA pipe instead of the MUFU unit, which both softmax warpgroups
      // of a sub-partition share.
      const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2);
      const uint64_t nbase2 = pack_f32x2(-base, -base);
      uint64_t sum2[4] = {pack_f32x2(0.f, 0.f), pack_f32x2(0.f, 0.f), pack_f32x2(0.f, 0.f),
                          pack_f32x2(0.f, 0.f)};  // four independent sum chains
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sr[64];
        sm100::tmem_ld32(t_lane + col_s(wg) + h * 64, sr);
        sm100::tmem_ld32(t_lane + col_s(wg) + h * 64 + 32, sr + 32);
        sm100::tmem_wait_ld();
        uint32_t pk[32];
        if (wfull) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint64_t x2 = fma_f32x2((static_cast<uint64_t>(sr[2 * e + 1]) << 32) | sr[2 * e],
                                          scale2, nbase2);
            const uint64_t p2 = (e % kPolyEvery == kPolyEvery - 1) ? exp2_poly_f32x2(x2)
                                                                    : exp2_mufu_f32x2(x2);
            sum2[e & 3] = add_f32x2(sum2[e & 3], p2);
            const float2 pp = unpack_f32x2(p2);
            pk[e] = pack_bf16x2(pp.x, pp.y);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = j0 + h * 64 + 2 * e;
            const uint64_t x2 = fma_f32x2(
                pack_f32x2(masked(sr[2 * e], key), masked(sr[2 * e + 1], key + 1)), scale2,
                nbase2);
            const uint64_t p2 = exp2_mufu_f32x2(x2);
            sum2[e & 3] = add_f32x2(sum2[e & 3], p2);
            const float2 pp = unpack_f32x2(p2);
            pk[e] = pack_bf16x2(pp.x, pp.y);
          }
        }
        sm100::tmem_st32(t_lane + col_s(wg) + h * 32, pk);
        if (kSplitP && h == 0) {
          sm100::tmem_wait_st();
          sm100::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->p_half[wg]);
        }
      }
      {
        const float2 sm =
            unpack_f32x2(add_f32x2(add_f32x2(sum2[0], sum2[1]), add_f32x2(sum2[2], sum2[3])));
        l += sm.x + sm.y;
      }
      // O rescale after P is out of registers (keeps the score row and this
      // buffer from being live together).
      if (!kSplitP && j > 0 && __any_sync(0xffffffffu, need)) {
        uint32_t orr[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          sm100::tmem_ld32(t_lane + col_o(wg) + c * 32, orr);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
          sm100::tmem_st32(t_lane + col_o(wg) + c * 32, orr);
        }
      }
      if (!kSplitP && MODE != kDense && wg == 0 && j == ntiles - 1 && kend - j0 < kBN) {
        // Stale cache rows past the end of the sequence: zero their V so that
        // 0 * NaN cannot reach O. Every tile row r is one 128-byte line in
        // each half. V_j must have landed first, or its TMA write would
        // overwrite the zeros (the slot's previous tile is already consumed:
        // its P V was issued before S0_j, whose completion brought us here).
        const int vlim = kend - j0;
        __all_sync(0xffffffffu, mbar_wait(&bars->v_full[j % kStages], (j / kStages) & 1));
        if (r >= vlim) {
          uint8_t* vrow = smem + kQBytes + (j % kStages) * 2 * kOperand + kOperand + r * 128;
          const int4 z = make_int4(0, 0, 0, 0);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            reinterpret_cast<int4*>(vrow)[c] = z;
            reinterpret_cast<int4*>(vrow + kHalf)[c] = z;
          }
        }
        fence_proxy_async();
      }
      sm100::tmem_wait_st();
      sm100::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[wg]);
    }
    if (!ok && lane == 0) set_status(p.status, NVATTN_STATUS_TIMEOUT);

    // ----------------------------------------------------------- epilogue
    const bool done = !warp_live || __all_sync(0xffffffffu, mbar_wait(&bars->o_done, 0));
    sm100::fence_after_sync();
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
    __nv_bfloat16* orow = p.out + static_cast<int64_t>(q_begin + (valid ? tok : 0)) * p.o_stride_tok +
                          static_cast<int64_t>(g * group + hh) * p.o_stride_head;
#pragma unroll
    for (int c = 0; c < 4 && warp_live; ++c) {
      uint32_t orr[32];
      sm100::tmem_ld32(t_lane + col_o(wg) + c * 32, orr);
      sm100::tmem_wait_ld();
      if (valid && done && p.nsplit > 1) {
        const int64_t slot =
            (static_cast<int64_t>(q_begin + tok) * p.num_heads + g * group + hh) * p.nsplit + split;
        float4* dst = reinterpret_cast<float4*>(p.ws_o + slot * kHeadDim + c * 32);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          dst[e] = make_float4(__uint_as_float(orr[4 * e]), __uint_as_float(orr[4 * e + 1]),
                               __uint_as_float(orr[4 * e + 2]), __uint_as_float(orr[4 * e + 3]));
        if (c == 0) p.ws_ml[slot] = make_float2(m_used, l);
      } else if (valid && done) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = pack_bf16x2(__uint_as_float(orr[2 * e]) * inv,
                              __uint_as_float(orr[2 * e + 1]) * inv);
        if (p.out_vec16) {
          int4* dst = reinterpret_cast<int4*>(orow + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            dst[e] = make_int4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
        } else {
          uint32_t* dst = reinterpret_cast<uint32_t*>(orow + c * 32);
#pragma unroll
          for (int e = 0; e < 16; ++e) dst[e] = pk[e];
        }
      }
    }
    if (!done && lane == 0) set_status(p.status, NVATTN_STATUS_TIMEOUT);
  }

  // Every TMEM access of this CTA is complete: release the allocation.
  sm100::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    sm100::fence_after_sync();
    sm100::tmem_dealloc(tmem, kTmemCols);
  }
}

// Tree mode: the order in which sequences' CTAs are dispatched, longest
// (most keys: context + draft) first, ties by index. With one wave or more of
// CTAs and no key split, the hardware's in-order dispatch to free SMs then
// schedules the items longest-processing-time first, which keeps the last SM
// to finish close to the average.
constexpr int kOrderMaxSeqs = 1024;

__global__ void __launch_bounds__(kOrderMaxSeqs)
    tree_order_kernel(const int32_t* __restrict__ ctx_lens, const int32_t* __restrict__ cu_q,
                      int num_seqs, int32_t* __restrict__ order) {
  __shared__ int32_t key[kOrderMaxSeqs];
  for (int i = threadIdx.x; i < num_seqs; i += blockDim.x)
    key[i] = max(0, ctx_lens[i]) + max(0, cu_q[i + 1] - cu_q[i]);
  __syncthreads();
  // Let the dependent attention grid launch now: it waits for this grid's
  // completion before it reads the order.
  asm volatile("griddepcontrol.launch_dependents;");
  for (int i = threadIdx.x; i < num_seqs; i += blockDim.x) {
    const int ki = key[i];
    int rank = 0;
    for (int j = 0; j < num_seqs; ++j) {
      const int kj = key[j];
      rank += (kj > ki) || (kj == ki && j < i);
    }
    order[rank] = i;
  }
}

// Merges the split-K partials of the tree mode: one warp per (node, query
// head); lane i owns dims 4i..4i+3. Splits past the sequence's keys were
// never run and are not read.
__global__ void __launch_bounds__(128)
    tree_combine_kernel(const Params p) {
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_begin = p.cu_q[b];
  int Lq = p.cu_q[b + 1] - q_begin;
  if (q_begin < 0 || q_begin > p.total_q) return;
  if (q_begin + static_cast<int64_t>(Lq) > p.total_q) Lq = static_cast<int>(p.total_q - q_begin);
  const int idx = blockIdx.x * 4 + warp;
  const int node = idx / p.num_heads, h = idx % p.num_heads;
  if (node >= Lq) return;
  int Lk = p.ctx_lens[b] + Lq;
  Lk = min(Lk, p.max_blocks * p.block_size);
  const int ntiles_all = Lk > 0 ? (Lk + kBN - 1) / kBN : 0;
  const int nact = min(p.nsplit, (ntiles_all + p.split_tiles - 1) / p.split_tiles);
  const int64_t base = (static_cast<int64_t>(q_begin + node) * p.num_heads + h) * p.nsplit;
  float mmax = -INFINITY;
  for (int s = 0; s < nact; ++s) mmax = fmaxf(mmax, p.ws_ml[base + s].x);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < nact; ++s) {
    const float2 ml = p.ws_ml[base + s];
    const float w = (ml.x == -INFINITY) ? 0.f : fast_exp2(ml.x - mmax);
    L += ml.y * w;
    const float4 o = reinterpret_cast<const float4*>(p.ws_o + (base + s) * kHeadDim)[lane];
    acc.x += o.x * w;
    acc.y += o.y * w;
    acc.z += o.z * w;
    acc.w += o.w * w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  __nv_bfloat16* orow = p.out + static_cast<int64_t>(q_begin + node) * p.o_stride_tok +
                        static_cast<int64_t>(h) * p.o_stride_head + lane * 4;
  const uint32_t lo = pack_bf16x2(acc.x * inv, acc.y * inv);
  const uint32_t hi = pack_bf16x2(acc.z * inv, acc.w * inv);
  if (p.out_vec16) {
    *reinterpret_cast<uint2*>(orow) = make_uint2(lo, hi);
  } else {
    reinterpret_cast<uint32_t*>(orow)[0] = lo;
    reinterpret_cast<uint32_t*>(orow)[1] = hi;
  }
}

int make_kv_map(CUtensorMap* map, const void* base, bool paged, int64_t total, int num_blocks,
                int block_size, int num_kv_heads, int64_t stride_tok, int64_t stride_head) {
  if (paged) {
    const uint64_t dims[4] = {static_cast<uint64_t>(kHeadDim),
                              static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(block_size),
                              static_cast<uint64_t>(num_blocks)};
    const uint64_t strides[3] = {
        static_cast<uint64_t>(kHeadDim) * 2, static_cast<uint64_t>(num_kv_heads) * kHeadDim * 2,
        static_cast<uint64_t>(block_size) * num_kv_heads * kHeadDim * 2};
    const uint32_t box[4] = {64, 1, static_cast<uint32_t>(kBN), 1};
    return make_tensor_map(map, base, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(num_kv_heads),
                            static_cast<uint64_t>(total)};
  const uint64_t strides[2] = {static_cast<uint64_t>(stride_head) * 2,
                               static_cast<uint64_t>(stride_tok) * 2};
  const uint32_t box[3] = {64, 1, static_cast<uint32_t>(kBN)};
  return make_tensor_map(map, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int make_q_map(CUtensorMap* map, const void* q, int64_t total_q, int num_heads, int64_t stride_tok,
               int64_t stride_head, int group, int tpt) {
  const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(num_heads),
                            static_cast<uint64_t>(total_q)};
  const uint64_t strides[2] = {static_cast<uint64_t>(stride_head) * 2,
                               static_cast<uint64_t>(stride_tok) * 2};
  const uint32_t box[3] = {64, static_cast<uint32_t>(group), static_cast<uint32_t>(tpt)};
  return make_tensor_map(map, q, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

constexpr int kSmemBytes = kSmemData + 1024 + static_cast<int>(sizeof(Barriers)) + 64;

// Per (mode, device): the kernel's dynamic shared-memory limit has been
// raised. File scope (internal linkage), so every copy of the library keeps
// its own flags.
static std::mutex g_attr_mu;
static bool g_attr_done[3][64];

template <int MODE>
int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Params& p,
           int num_seqs, int max_tokens, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(g_attr_mu);
    if (dev >= 64 || !g_attr_done[MODE][dev]) {
      cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<MODE>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmemBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attn_tc_kernel)");
      if (dev < 64) g_attr_done[MODE][dev] = true;
    }
  }
  const int blocks_m = (max_tokens + 2 * p.tpt - 1) / (2 * p.tpt);
  if (blocks_m <= 0) return NVATTN_OK;
  if (num_seqs > 65535) return fail(NVATTN_ERR_UNSUPPORTED, "more than 65535 sequences");
  dim3 grid(blocks_m * p.nsplit, p.num_kv_heads, num_seqs);
  cudaError_t e;
  if (MODE == kTree && p.order != nullptr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, attn_tc_kernel<MODE>, qm, km, vm, p);
  } else {
    attn_tc_kernel<MODE><<<grid, kThreads, kSmemBytes, stream>>>(qm, km, vm, p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return cuda_fail(e, "attn_tc_kernel launch");
  if (p.nsplit > 1) {
    const int per_seq = max_tokens * p.num_heads;
    tree_combine_kernel<<<dim3((per_seq + 3) / 4, num_seqs), 128, 0, stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "tree_combine_kernel launch");
  }
  return NVATTN_OK;
}

}  // namespace tc

// Shared argument checks of the two entry points; returns NVATTN_OK or a code.
static int tc_check_q_out(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                          const void* out, int64_t o_stride_tok, int64_t o_stride_head,
                          int num_heads, int num_kv_heads, int head_dim, const char* who) {
  if (!q || !out) return fail(NVATTN_ERR_INVALID, std::string(who) + ": NULL q/out");
  if (head_dim != kHeadDim)
    return fail(NVATTN_ERR_UNSUPPORTED, std::string(who) + ": head_dim must be 128");
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads)
    return fail(NVATTN_ERR_INVALID,
                std::string(who) + ": num_heads must be a multiple of num_kv_heads");
  if (num_heads / num_kv_heads > 16)
    return fail(NVATTN_ERR_UNSUPPORTED,
                std::string(who) + ": more than 16 query heads per KV head");
  if (!aligned16(q) || (q_stride_tok * 2) % 16 || (q_stride_head * 2) % 16)
    return fail(NVATTN_ERR_UNSUPPORTED,
                std::string(who) + ": q base and strides must be 16-byte multiples (TMA)");
  if ((reinterpret_cast<uintptr_t>(out) & 3) || (o_stride_tok & 1) || (o_stride_head & 1))
    return fail(NVATTN_ERR_UNSUPPORTED, std::string(who) + ": out rows must be 4-byte aligned");
  return NVATTN_OK;
}

static tc::Params tc_params(void* out, int64_t o_stride_tok, int64_t o_stride_head,
                            int num_heads, int num_kv_heads, float softmax_scale,
                            int64_t total_q, int32_t* status) {
  tc::Params p{};
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_stride_tok = o_stride_tok;
  p.o_stride_head = o_stride_head;
  p.total_q = total_q;
  p.num_kv_heads = num_kv_heads;
  p.group = num_heads / num_kv_heads;
  p.tpt = tc::kBM / p.group;
  p.rpt = p.tpt * p.group;
  p.out_vec16 = aligned16(out) && (o_stride_tok * 2) % 16 == 0 && (o_stride_head * 2) % 16 == 0;
  p.nsplit = 1;
  p.split_tiles = 1 << 30;
  p.num_heads = num_heads;
  p.scale_log2 = softmax_scale * kLog2e;
  p.status = status;
  return p;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Tree mode: split the key range when the (sequence, KV head, row block)
// CTAs alone cannot fill ~4 waves of the GPU; splits hold >= 8 key tiles.
// Depends only on host-side sizes (the block-table width bounds the keys).
static void tree_split(int num_seqs, int num_heads, int num_kv_heads, int max_nodes,
                       int max_blocks, int block_size, int* nsplit, int* split_tiles) {
  const int group = num_heads / num_kv_heads;
  const int tpt = tc::kBM / group;
  const int blocks_m = (max_nodes + 2 * tpt - 1) / (2 * tpt);
  const int64_t ctas = static_cast<int64_t>(num_seqs) * num_kv_heads * blocks_m;
  const int max_tiles = static_cast<int>(
      (static_cast<int64_t>(max_blocks) * block_size + tc::kBN - 1) / tc::kBN);
  // One wave or more of items: no split (no partials to write and merge);
  // the items are dispatched longest first instead (tree_order_kernel).
  // Fewer: split each item's keys just enough for the CTAs to cover the SMs,
  // twice that when the items are under a quarter of the SMs (measured at the
  // per-rank shapes of configs[4] at TP 2/4/8, 128/64/32 items: 146/95/62 us,
  // against 170/103/62 us for a 4-wave split target and 146/118/62 us for 2).
  int ns = 1;
  const int sms = sm_count();
  if (ctas < sms) {
    ns = static_cast<int>((sms + ctas - 1) / ctas);
    if (ctas * 4 <= sms) ns *= 2;
    ns = std::min(ns, std::max(1, max_tiles / 8));
  }
  *nsplit = std::max(1, ns);
  *split_tiles = (max_tiles + *nsplit - 1) / *nsplit;
}

// Tree workspace: the dispatch order (one int32 per sequence, when there are
// at most kOrderMaxSeqs sequences), then with a key split the fp32 partial O
// and the (max, sum) pairs; each region 256-byte aligned.
static size_t tree_order_bytes(int num_seqs) {
  return num_seqs <= tc::kOrderMaxSeqs ? (static_cast<size_t>(num_seqs) * 4 + 255) & ~size_t(255)
                                       : 0;
}

static size_t tree_ws_bytes(int num_seqs, int64_t total_q, int num_heads, int nsplit) {
  size_t bytes = tree_order_bytes(num_seqs);
  if (nsplit > 1) {
    const size_t n = static_cast<size_t>(total_q) * num_heads * nsplit;
    const size_t o_bytes = (n * kHeadDim * sizeof(float) + 255) & ~static_cast<size_t>(255);
    bytes += o_bytes + n * sizeof(float2);
  }
  return bytes;
}

}  // namespace nvattn

using namespace nvattn;

extern "C" size_t nvattn_tree_workspace_bytes(int32_t num_seqs, int32_t max_nodes, int64_t total_q,
                                              int32_t num_heads, int32_t num_kv_heads,
                                              int32_t max_blocks_per_seq, int32_t block_size) {
  if (num_seqs <= 0 || max_nodes <= 0 || total_q <= 0 || num_heads <= 0 || num_kv_heads <= 0 ||
      num_heads % num_kv_heads || max_blocks_per_seq <= 0 || block_size <= 0)
    return 0;
  int nsplit, split_tiles;
  tree_split(num_seqs, num_heads, num_kv_heads, max_nodes, max_blocks_per_seq, block_size, &nsplit,
             &split_tiles);
  return tree_ws_bytes(num_seqs, total_q, num_heads, nsplit);
}

extern "C" int nvattn_varlen_prefill(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* k,
    int64_t k_stride_tok, int64_t k_stride_head, const void* v, int64_t v_stride_tok,
    int64_t v_stride_head, void* out, int64_t o_stride_tok, int64_t o_stride_head,
    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t num_seqs,
    int32_t max_seqlen_q, int32_t max_seqlen_k, int64_t total_q, int64_t total_k,
    const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks_per_seq,
    int32_t num_blocks, int32_t block_size, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, float softmax_scale, int32_t causal, int32_t* status, void* stream) {
  clear_error();
  if (num_seqs < 0 || total_q < 0 || total_k < 0 || max_seqlen_q < 0 || max_seqlen_k < 0)
    return fail(NVATTN_ERR_INVALID, "varlen_prefill: negative size");
  if (num_seqs == 0 || total_q == 0 || max_seqlen_q == 0) return NVATTN_OK;
  int rc = tc_check_q_out(q, q_stride_tok, q_stride_head, out, o_stride_tok, o_stride_head,
                          num_heads, num_kv_heads, head_dim, "varlen_prefill");
  if (rc) return rc;
  if (!k || !v || !cu_seqlens_q || !cu_seqlens_k)
    return fail(NVATTN_ERR_INVALID, "varlen_prefill: NULL k/v/cu_seqlens");
  tc::Params p = tc_params(out, o_stride_tok, o_stride_head, num_heads, num_kv_heads,
                           softmax_scale, total_q, status);
  CUtensorMap qm, km, vm;
  rc = tc::make_q_map(&qm, q, total_q, num_heads, q_stride_tok, q_stride_head, p.group, p.tpt);
  if (rc) return rc;
  if (block_table) {
    if (block_size <= 0 || block_size % tc::kBN)
      return fail(NVATTN_ERR_UNSUPPORTED, "varlen_prefill: block_size must be a multiple of 128");
    if (num_blocks <= 0 || max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
      return fail(NVATTN_ERR_INVALID, "varlen_prefill: bad block table geometry");
    if (!aligned16(k) || !aligned16(v))
      return fail(NVATTN_ERR_INVALID, "varlen_prefill: caches must be 16-byte aligned");
    rc = tc::make_kv_map(&km, k, true, 0, num_blocks, block_size, num_kv_heads, 0, 0);
    if (rc) return rc;
    rc = tc::make_kv_map(&vm, v, true, 0, num_blocks, block_size, num_kv_heads, 0, 0);
    if (rc) return rc;
  } else {
    if (total_k <= 0) return fail(NVATTN_ERR_INVALID, "varlen_prefill: total_k must be > 0");
    if (!aligned16(k) || !aligned16(v) || (k_stride_tok * 2) % 16 || (k_stride_head * 2) % 16 ||
        (v_stride_tok * 2) % 16 || (v_stride_head * 2) % 16)
      return fail(NVATTN_ERR_UNSUPPORTED,
                  "varlen_prefill: k/v base and strides must be 16-byte multiples (TMA)");
    rc = tc::make_kv_map(&km, k, false, total_k, 0, 0, num_kv_heads, k_stride_tok, k_stride_head);
    if (rc) return rc;
    rc = tc::make_kv_map(&vm, v, false, total_k, 0, 0, num_kv_heads, v_stride_tok, v_stride_head);
    if (rc) return rc;
  }
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.max_blocks = block_table ? max_blocks_per_seq : 0;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.causal = causal ? 1 : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return block_table ? tc::launch<tc::kPaged>(qm, km, vm, p, num_seqs, max_seqlen_q, s)
                     : tc::launch<tc::kDense>(qm, km, vm, p, num_seqs, max_seqlen_q, s);
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
                                  void* workspace, size_t workspace_bytes, int32_t* status,
                                  void* stream) {
  clear_error();
  if (num_seqs < 0 || total_q < 0 || max_nodes < 0)
    return fail(NVATTN_ERR_INVALID, "tree_verify: negative size");
  if (num_seqs == 0 || total_q == 0 || max_nodes == 0) return NVATTN_OK;
  if (max_nodes > 64) return fail(NVATTN_ERR_UNSUPPORTED, "tree_verify: at most 64 tree nodes");
  int rc = tc_check_q_out(q, q_stride_tok, q_stride_head, out, o_stride_tok, o_stride_head,
                          num_heads, num_kv_heads, head_dim, "tree_verify");
  if (rc) return rc;
  if (!k_cache || !v_cache || !cu_seqlens_q || !context_lens || !tree_mask || !block_table)
    return fail(NVATTN_ERR_INVALID, "tree_verify: NULL pointer");
  if (block_size <= 0 || block_size % tc::kBN)
    return fail(NVATTN_ERR_UNSUPPORTED, "tree_verify: block_size must be a multiple of 128");
  if (num_blocks <= 0 || max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
    return fail(NVATTN_ERR_INVALID, "tree_verify: bad block table geometry");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(NVATTN_ERR_INVALID, "tree_verify: caches must be 16-byte aligned");
  tc::Params p = tc_params(out, o_stride_tok, o_stride_head, num_heads, num_kv_heads,
                           softmax_scale, total_q, status);
  CUtensorMap qm, km, vm;
  rc = tc::make_q_map(&qm, q, total_q, num_heads, q_stride_tok, q_stride_head, p.group, p.tpt);
  if (rc) return rc;
  rc = tc::make_kv_map(&km, k_cache, true, 0, num_blocks, block_size, num_kv_heads, 0, 0);
  if (rc) return rc;
  rc = tc::make_kv_map(&vm, v_cache, true, 0, num_blocks, block_size, num_kv_heads, 0, 0);
  if (rc) return rc;
  p.cu_q = cu_seqlens_q;
  p.ctx_lens = context_lens;
  p.tree_mask = tree_mask;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.max_blocks = max_blocks_per_seq;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.causal = 1;
  tree_split(num_seqs, num_heads, num_kv_heads, max_nodes, max_blocks_per_seq, block_size,
             &p.nsplit, &p.split_tiles);
  const size_t need = tree_ws_bytes(num_seqs, total_q, num_heads, p.nsplit);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes < need)
      return fail(NVATTN_ERR_WORKSPACE,
                  "tree_verify: workspace smaller than nvattn_tree_workspace_bytes()");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
      return fail(NVATTN_ERR_INVALID, "tree_verify: workspace must be 256-byte aligned");
    char* ws = static_cast<char*>(workspace);
    const size_t ob = tree_order_bytes(num_seqs);
    if (ob > 0) {
      int32_t* order = reinterpret_cast<int32_t*>(ws);
      tc::tree_order_kernel<<<1, tc::kOrderMaxSeqs, 0, s>>>(context_lens, cu_seqlens_q, num_seqs,
                                                             order);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(e, "tree_order_kernel launch");
      p.order = order;
    }
    if (p.nsplit > 1) {
      const size_t n = static_cast<size_t>(total_q) * num_heads * p.nsplit;
      const size_t o_bytes = (n * kHeadDim * sizeof(float) + 255) & ~static_cast<size_t>(255);
      p.ws_o = reinterpret_cast<float*>(ws + ob);
      p.ws_ml = reinterpret_cast<float2*>(ws + ob + o_bytes);
    }
  }
  return tc::launch<tc::kTree>(qm, km, vm, p, num_seqs, max_nodes, s);
}
