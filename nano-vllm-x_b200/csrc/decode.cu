// Paged split-K decode attention (replaces flash_attn_with_kvcache as called at
// nanovllm/layers/attention.py:72-74).
//
// Work decomposition: CTA (split s, KV head g, sequence b) owns the key range
// [s*split_tokens, min((s+1)*split_tokens, cache_seqlens[b])) of one KV head and
// computes it for ALL num_heads/num_kv_heads query heads of that group, so each
// KV byte is read from HBM exactly once per call.
//
// Data path: a producer warp streams 64-token K and V tiles of the paged cache
// into a STAGES-deep shared-memory ring with 4-D TMA loads (box d64 x 1 head x
// 64 tokens x 1 block, 128-byte swizzle, no multicast); completion is tracked
// by mbarriers with bounded waits. Four consumer warps each take 16 of the 64
// tokens of a tile and run S = Q K^T and O += P V on the tensor cores
// (mma.m16n8k16 bf16 -> fp32, the GQA group padded to the 16 M rows), with an
// online softmax in fp32 whose row reductions are quad warp shuffles. At the
// end the four warps merge through shared memory; with one split the CTA
// writes the bf16 output, otherwise it writes an fp32 partial (O, max, sum)
// that nvattn_decode_combine_kernel merges.
//
// The arithmetic intensity is ~2*GQA flop per KV byte, far below the B200
// ridge, so the kernel is HBM-bound by design; the tensor cores only keep the
// 2*GQA fp32 FMAs per KV element off the FMA pipe.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace nvattn {

constexpr int kTile = 64;                      // tokens per pipeline stage
constexpr int kDecStages = 3;                  // ring depth
constexpr int kHalfBytes = kTile * 128;        // one 64-token x 64-dim half tile (8 KB)
constexpr int kStageBytes = 4 * kHalfBytes;    // K lo/hi + V lo/hi (32 KB)
constexpr int kDecConsumerWarps = 4;
constexpr int kDecThreads = (kDecConsumerWarps + 1) * 32;
constexpr int kMaxGroup = 16;                  // query heads per KV head handled per CTA
constexpr int kOPad = 132;                     // fp32 row pitch of the merge buffer
// Split policy (see choose_split); overridable at build time for tuning sweeps.
#ifndef NVATTN_DEC_MIN_SPLIT_TILES
#define NVATTN_DEC_MIN_SPLIT_TILES 4
#endif
#ifndef NVATTN_DEC_SPLIT_CTAS_PER_SM
#define NVATTN_DEC_SPLIT_CTAS_PER_SM 8
#endif
constexpr int kMinSplitTiles = NVATTN_DEC_MIN_SPLIT_TILES;
constexpr int kSplitCtasPerSm = NVATTN_DEC_SPLIT_CTAS_PER_SM;

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_stride_tok, q_stride_head;
  __nv_bfloat16* out;
  int64_t o_stride_tok, o_stride_head;
  const int32_t* seqlens;
  const int32_t* block_table;
  int64_t bt_stride;
  int32_t num_blocks, block_size, num_heads, num_kv_heads, group;
  int32_t max_blocks;  // block-table width: keys past max_blocks*block_size are ignored
  int32_t nsplit, split_tiles;
  float scale_log2;
  float* ws_o;    // [batch][num_heads][nsplit][128]
  float2* ws_ml;  // [batch][num_heads][nsplit]  (running max (log2 units), sum)
  int32_t* status;
};

__device__ __forceinline__ float neg_inf() { return -INFINITY; }

__global__ void __launch_bounds__(kDecThreads, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const DecodeParams p) {
  const int split = blockIdx.x;
  const int g = blockIdx.y;
  const int b = blockIdx.z;
  int ctx = p.seqlens[b];
  if (ctx > p.max_blocks * p.block_size) {
    if (split == 0 && threadIdx.x == 0) set_status(p.status, NVATTN_STATUS_BAD_BLOCK);
    ctx = p.max_blocks * p.block_size;
  }
  const int tok_begin = split * p.split_tiles * kTile;
  const int tok_end = min(ctx, tok_begin + p.split_tiles * kTile);
  if (tok_end <= tok_begin) {
    // Whole CTA idle (uniform exit). Without a combine pass the empty
    // sequence's output rows still have to be written (as zeros).
    if (p.nsplit == 1 && split == 0) {
      for (int e = threadIdx.x; e < p.group * kHeadDim; e += blockDim.x) {
        const int h = g * p.group + e / kHeadDim;
        p.out[static_cast<int64_t>(b) * p.o_stride_tok + static_cast<int64_t>(h) * p.o_stride_head +
              e % kHeadDim] = __float2bfloat16_rn(0.f);
      }
    }
    return;
  }
  const int ntiles = (tok_end - tok_begin + kTile - 1) / kTile;
  // The combine kernel may be scheduled from now on (it waits for this grid's
  // completion before it reads anything).
  asm volatile("griddepcontrol.launch_dependents;");

  extern __shared__ uint8_t smem_raw[];
  // Swizzled TMA tiles need 1024-byte alignment.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecStages * kStageBytes);
  uint64_t* empty = full + kDecStages;
  float* ml_smem = reinterpret_cast<float*>(empty + kDecStages);  // [4][16][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kDecStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kDecConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDecConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensor_map(&kmap);
      prefetch_tensor_map(&vmap);
      const int32_t* bt = p.block_table + static_cast<int64_t>(b) * p.bt_stride;
      for (int it = 0; it < ntiles; ++it) {
        const int stage = it % kDecStages;
        const uint32_t phase = (it / kDecStages) & 1;
        if (!mbar_wait(&empty[stage], phase ^ 1)) {
          set_status(p.status, NVATTN_STATUS_TIMEOUT);
          break;
        }
        const int tok0 = tok_begin + it * kTile;
        int blk = bt[tok0 / p.block_size];
        if (blk < 0 || blk >= p.num_blocks) {
          set_status(p.status, NVATTN_STATUS_BAD_BLOCK);
          blk = 0;  // read a valid block; the result is flagged as invalid
        }
        const int tin = tok0 % p.block_size;
        uint8_t* st = smem + stage * kStageBytes;
        mbar_arrive_expect_tx(&full[stage], kStageBytes);
        tma_load_4d(st, &kmap, &full[stage], 0, g, tin, blk);
        tma_load_4d(st + kHalfBytes, &kmap, &full[stage], 64, g, tin, blk);
        tma_load_4d(st + 2 * kHalfBytes, &vmap, &full[stage], 0, g, tin, blk);
        tma_load_4d(st + 3 * kHalfBytes, &vmap, &full[stage], 64, g, tin, blk);
      }
    }
    // The producer warp takes no part in the merge below.
    return;
  }

  // -------------------------------------------------------------- consumers
  const int quad = lane & 3;   // column pair inside an 8-wide MMA tile
  const int rowa = lane >> 2;  // accumulator rows rowa and rowa + 8
  const int rowb = rowa + 8;
  const int h0 = g * p.group;

  // Q fragments (A operand, rows = query heads of the group, K = head dim).
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* qb = p.q + static_cast<int64_t>(b) * p.q_stride_tok;
    const bool va = rowa < p.group, vb = rowb < p.group;
    const uint32_t* qra =
        reinterpret_cast<const uint32_t*>(qb + static_cast<int64_t>(h0 + rowa) * p.q_stride_head);
    const uint32_t* qrb =
        reinterpret_cast<const uint32_t*>(qb + static_cast<int64_t>(h0 + rowb) * p.q_stride_head);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 8 + quad;  // uint32 index of d = 16kk + 2*quad
      qa[kk][0] = va ? qra[c] : 0u;
      qa[kk][1] = vb ? qrb[c] : 0u;
      qa[kk][2] = va ? qra[c + 4] : 0u;
      qa[kk][3] = vb ? qrb[c + 4] : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = neg_inf(), m_b = neg_inf(), l_a = 0.f, l_b = 0.f;

  const int r0 = warp * 16;  // this warp's first token row inside a tile
  bool timed_out = false;
  for (int it = 0; it < ntiles; ++it) {
    const int stage = it % kDecStages;
    const uint32_t phase = (it / kDecStages) & 1;
    if (!mbar_wait(&full[stage], phase)) {
      timed_out = true;
      break;
    }
    const int nvalid = min(kTile, tok_end - (tok_begin + it * kTile));
    if (r0 < nvalid) {
      const uint32_t kbase = smem_u32(smem + stage * kStageBytes);
      const uint32_t vbase = kbase + 2 * kHalfBytes;
      // ---- S = Q K^T for 16 tokens (two n8 tiles)
      float s[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
      {
        const int mi = lane >> 3;
        const int row = r0 + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t half = (kk >> 2) * kHalfBytes;
          const int chunk = ((kk & 3) << 1) + (mi & 1);
          uint32_t b00, b01, b10, b11;
          ldmatrix_x4(kbase + half + swz128(row, chunk), b00, b01, b10, b11);
          mma_bf16_16816(s[0], qa[kk], b00, b01);
          mma_bf16_16816(s[1], qa[kk], b10, b11);
        }
      }
      // ---- mask, scale, online softmax
      float mx_a = neg_inf(), mx_b = neg_inf();
#pragma unroll
      for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int t = r0 + n * 8 + quad * 2 + j;
          const bool ok = t < nvalid;
          s[n][j] = ok ? s[n][j] * p.scale_log2 : neg_inf();
          s[n][2 + j] = ok ? s[n][2 + j] * p.scale_log2 : neg_inf();
          mx_a = fmaxf(mx_a, s[n][j]);
          mx_b = fmaxf(mx_b, s[n][2 + j]);
        }
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      // r0 < nvalid guarantees at least one finite score per row.
      const float al_a = fast_exp2(m_a - mn_a), al_b = fast_exp2(m_b - mn_b);
      m_a = mn_a;
      m_b = mn_b;
      float ps_a = 0.f, ps_b = 0.f;
#pragma unroll
      for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          s[n][j] = fast_exp2(s[n][j] - mn_a);
          s[n][2 + j] = fast_exp2(s[n][2 + j] - mn_b);
          ps_a += s[n][j];
          ps_b += s[n][2 + j];
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
      // ---- O += P V
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[0][0], s[0][1]);
      pa[1] = pack_bf16x2(s[0][2], s[0][3]);
      pa[2] = pack_bf16x2(s[1][0], s[1][1]);
      pa[3] = pack_bf16x2(s[1][2], s[1][3]);
      // Tokens past nvalid in the last tile hold stale cache bytes (maybe
      // NaN): zero their V elements so 0 * NaN never reaches the sum.
      const bool full_tile = (r0 + 16) <= nvalid;
      const int t_lo = r0 + quad * 2;
      const uint32_t mlo = full_tile ? 0xffffffffu
                                     : ((t_lo < nvalid ? 0x0000ffffu : 0u) |
                                        (t_lo + 1 < nvalid ? 0xffff0000u : 0u));
      const uint32_t mhi = full_tile ? 0xffffffffu
                                     : ((t_lo + 8 < nvalid ? 0x0000ffffu : 0u) |
                                        (t_lo + 9 < nvalid ? 0xffff0000u : 0u));
      {
        const int mi = lane >> 3;
        const int row = r0 + ((mi & 1) << 3) + (lane & 7);
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
  if (timed_out && lane == 0) set_status(p.status, NVATTN_STATUS_TIMEOUT);

  // ---------------------------------------------------------------- merge
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);

  // All consumer warps are past their last ring read: reuse the ring.
  asm volatile("bar.sync 1, %0;" ::"r"(kDecConsumerWarps * 32));
  float* obuf = reinterpret_cast<float*>(smem);  // [4 warps][16 rows][kOPad]
  float* ow = obuf + warp * kMaxGroup * kOPad;
  if (quad == 0) {
    ml_smem[(warp * kMaxGroup + rowa) * 2 + 0] = m_a;
    ml_smem[(warp * kMaxGroup + rowa) * 2 + 1] = l_a;
    ml_smem[(warp * kMaxGroup + rowb) * 2 + 0] = m_b;
    ml_smem[(warp * kMaxGroup + rowb) * 2 + 1] = l_b;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = j * 8 + quad * 2;
    *reinterpret_cast<float2*>(ow + rowa * kOPad + d) = make_float2(o[j][0], o[j][1]);
    *reinterpret_cast<float2*>(ow + rowb * kOPad + d) = make_float2(o[j][2], o[j][3]);
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kDecConsumerWarps * 32));

  const int d = threadIdx.x;  // 0..127: one head-dim column per thread
  for (int r = 0; r < p.group; ++r) {
    float mw[kDecConsumerWarps];
    float mmax = neg_inf();
#pragma unroll
    for (int w = 0; w < kDecConsumerWarps; ++w) {
      mw[w] = ml_smem[(w * kMaxGroup + r) * 2];
      mmax = fmaxf(mmax, mw[w]);
    }
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kDecConsumerWarps; ++w) {
      // A warp with no valid token keeps m = -inf, l = 0, o = 0.
      const float f = (mw[w] == neg_inf()) ? 0.f : fast_exp2(mw[w] - mmax);
      L += ml_smem[(w * kMaxGroup + r) * 2 + 1] * f;
      acc += obuf[(w * kMaxGroup + r) * kOPad + d] * f;
    }
    const int h = h0 + r;
    if (p.nsplit == 1) {
      const float v = (L > 0.f) ? acc / L : 0.f;
      p.out[static_cast<int64_t>(b) * p.o_stride_tok + static_cast<int64_t>(h) * p.o_stride_head +
            d] = __float2bfloat16_rn(v);
    } else {
      const int64_t slot = (static_cast<int64_t>(b) * p.num_heads + h) * p.nsplit + split;
      p.ws_o[slot * kHeadDim + d] = acc;
      if (d == 0) p.ws_ml[slot] = make_float2(mmax, L);
    }
  }
}

// Merges the split-K partials of one (sequence, query head) per warp-group.
__global__ void __launch_bounds__(128)
    decode_combine_kernel(const DecodeParams p) {
  // Launched as a programmatic dependent of paged_decode_kernel: it may start
  // while the last decode CTAs run; this waits until that grid has completed
  // and its partials are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int d = threadIdx.x;
  const int ctx = min(p.seqlens[b], p.max_blocks * p.block_size);
  const int split_tokens = p.split_tiles * kTile;
  const int nact = min(p.nsplit, (max(ctx, 0) + split_tokens - 1) / split_tokens);
  const int64_t base = (static_cast<int64_t>(b) * p.num_heads + h) * p.nsplit;
  float mmax = -INFINITY;
  for (int s = 0; s < nact; ++s) mmax = fmaxf(mmax, p.ws_ml[base + s].x);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < nact; ++s) {
    const float2 ml = p.ws_ml[base + s];
    const float f = (ml.x == -INFINITY) ? 0.f : fast_exp2(ml.x - mmax);
    L += ml.y * f;
    acc += p.ws_o[(base + s) * kHeadDim + d] * f;
  }
  const float v = (L > 0.f) ? acc / L : 0.f;
  p.out[static_cast<int64_t>(b) * p.o_stride_tok + static_cast<int64_t>(h) * p.o_stride_head + d] =
      __float2bfloat16_rn(v);
}

static int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Split size (in 64-token tiles): the largest of 64/32/16/8/4 tiles that
// still gives >= 8 CTAs per SM when every sequence is at the block-table
// width (longer splits amortise each CTA's pipeline fill and shrink the
// partials the combine reads; when one split covers the table, the kernel
// writes the output itself and no combine runs).
// Depends only on host-side sizes, so a captured graph keeps its grid.
static void choose_split(int batch, int num_kv_heads, int max_blocks, int block_size,
                         int* nsplit, int* split_tiles) {
  const int sms = device_sm_count();
  const int64_t max_tiles = (static_cast<int64_t>(max_blocks) * block_size + kTile - 1) / kTile;
  const int64_t pairs = static_cast<int64_t>(batch) * num_kv_heads;
  int st = 64;
  while (st > kMinSplitTiles) {
    const int64_t ns = (max_tiles + st - 1) / st;
    if (pairs * ns >= static_cast<int64_t>(kSplitCtasPerSm) * sms) break;
    st >>= 1;
  }
  *split_tiles = st;
  *nsplit = static_cast<int>(std::max<int64_t>(1, (max_tiles + st - 1) / st));
}

static size_t decode_ws_bytes(int batch, int num_heads, int nsplit) {
  if (nsplit <= 1) return 0;
  const size_t n = static_cast<size_t>(batch) * num_heads * nsplit;
  // partial O (128 fp32 per slot) followed by (max, sum) pairs; keep 256-B alignment.
  const size_t o_bytes = (n * kHeadDim * sizeof(float) + 255) & ~static_cast<size_t>(255);
  return o_bytes + n * sizeof(float2);
}

static int set_smem_attr(const void* fn, int bytes) {
  // Per device: the attribute must be set once in every context that launches.
  static std::mutex mu;
  static int done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && done[dev] >= bytes) return NVATTN_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  if (dev < 64) done[dev] = bytes;
  return NVATTN_OK;
}

int make_cache_map(CUtensorMap* map, const void* cache, int num_blocks, int block_size,
                   int num_kv_heads) {
  // dims innermost first: head_dim, kv head, token-in-block, block
  const uint64_t dims[4] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(num_kv_heads),
                            static_cast<uint64_t>(block_size),
                            static_cast<uint64_t>(num_blocks)};
  const uint64_t strides[3] = {
      static_cast<uint64_t>(kHeadDim) * 2, static_cast<uint64_t>(num_kv_heads) * kHeadDim * 2,
      static_cast<uint64_t>(block_size) * num_kv_heads * kHeadDim * 2};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(kTile), 1};
  return make_tensor_map(map, cache, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Argument checks shared by both decode entry points (a negative batch is an
// error; the caller handles batch == 0 before).
static int check_decode_args(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                             const void* k_cache, const void* v_cache, const void* out,
                             const int32_t* cache_seqlens, const int32_t* block_table,
                             int64_t block_table_stride, int32_t max_blocks_per_seq,
                             int32_t num_blocks, int32_t block_size, int32_t batch,
                             int32_t num_heads, int32_t num_kv_heads, int32_t head_dim) {
  if (batch < 0) return fail(NVATTN_ERR_INVALID, "paged_decode: negative batch");
  if (!q || !k_cache || !v_cache || !out || !cache_seqlens || !block_table)
    return fail(NVATTN_ERR_INVALID, "paged_decode: NULL pointer");
  if (head_dim != kHeadDim) return fail(NVATTN_ERR_UNSUPPORTED, "paged_decode: head_dim must be 128");
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads)
    return fail(NVATTN_ERR_INVALID, "paged_decode: num_heads must be a multiple of num_kv_heads");
  if (num_heads / num_kv_heads > kMaxGroup)
    return fail(NVATTN_ERR_UNSUPPORTED, "paged_decode: more than 16 query heads per KV head");
  if (block_size <= 0 || block_size % kTile)
    return fail(NVATTN_ERR_UNSUPPORTED, "paged_decode: block_size must be a multiple of 64");
  if (num_blocks <= 0 || max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
    return fail(NVATTN_ERR_INVALID, "paged_decode: bad block table geometry");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(NVATTN_ERR_INVALID, "paged_decode: caches must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_stride_tok & 1) || (q_stride_head & 1))
    return fail(NVATTN_ERR_UNSUPPORTED, "paged_decode: q rows must be 4-byte aligned");
  return NVATTN_OK;
}

}  // namespace nvattn

using namespace nvattn;

extern "C" size_t nvattn_decode_workspace_bytes(int32_t batch, int32_t num_heads,
                                                int32_t num_kv_heads, int32_t max_blocks_per_seq,
                                                int32_t block_size) {
  if (batch <= 0 || num_heads <= 0 || num_kv_heads <= 0 || max_blocks_per_seq <= 0 ||
      block_size <= 0)
    return 0;
  int nsplit, split_tiles;
  choose_split(batch, num_kv_heads, max_blocks_per_seq, block_size, &nsplit, &split_tiles);
  return decode_ws_bytes(batch, num_heads, nsplit);
}

extern "C" int nvattn_paged_decode(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                   const void* k_cache, const void* v_cache, void* out,
                                   int64_t o_stride_tok, int64_t o_stride_head,
                                   const int32_t* cache_seqlens, const int32_t* block_table,
                                   int64_t block_table_stride, int32_t max_blocks_per_seq,
                                   int32_t num_blocks, int32_t block_size, int32_t batch,
                                   int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                   float softmax_scale, void* workspace, size_t workspace_bytes,
                                   int32_t* status, void* stream) {
  clear_error();
  if (batch == 0) return NVATTN_OK;
  int rc = check_decode_args(q, q_stride_tok, q_stride_head, k_cache, v_cache, out,
                             cache_seqlens, block_table, block_table_stride, max_blocks_per_seq,
                             num_blocks, block_size, batch, num_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  const int group = num_heads / num_kv_heads;

  int nsplit, split_tiles;
  choose_split(batch, num_kv_heads, max_blocks_per_seq, block_size, &nsplit, &split_tiles);
  const size_t need = decode_ws_bytes(batch, num_heads, nsplit);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(NVATTN_ERR_WORKSPACE, "paged_decode: workspace smaller than "
                                      "nvattn_decode_workspace_bytes()");
  if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(NVATTN_ERR_INVALID, "paged_decode: workspace must be 256-byte aligned");

  CUtensorMap kmap, vmap;
  rc = make_cache_map(&kmap, k_cache, num_blocks, block_size, num_kv_heads);
  if (rc) return rc;
  rc = make_cache_map(&vmap, v_cache, num_blocks, block_size, num_kv_heads);
  if (rc) return rc;

  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride_tok = q_stride_tok;
  p.q_stride_head = q_stride_head;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_stride_tok = o_stride_tok;
  p.o_stride_head = o_stride_head;
  p.seqlens = cache_seqlens;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = group;
  p.max_blocks = max_blocks_per_seq;
  p.nsplit = nsplit;
  p.split_tiles = split_tiles;
  p.scale_log2 = softmax_scale * kLog2e;
  p.status = status;
  if (need > 0) {
    const size_t n = static_cast<size_t>(batch) * num_heads * nsplit;
    const size_t o_bytes = (n * kHeadDim * sizeof(float) + 255) & ~static_cast<size_t>(255);
    p.ws_o = static_cast<float*>(workspace);
    p.ws_ml = reinterpret_cast<float2*>(static_cast<char*>(workspace) + o_bytes);
  } else {
    p.ws_o = nullptr;
    p.ws_ml = nullptr;
  }

  const int smem = kDecStages * kStageBytes + 1024 + 2 * kDecStages * 8 +
                   kDecConsumerWarps * kMaxGroup * 2 * 4;
  rc = set_smem_attr(reinterpret_cast<const void*>(paged_decode_kernel), smem);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (batch > 65535) return fail(NVATTN_ERR_UNSUPPORTED, "paged_decode: batch > 65535");
  dim3 grid(nsplit, num_kv_heads, batch);
  paged_decode_kernel<<<grid, kDecThreads, smem, s>>>(kmap, vmap, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
  if (nsplit > 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_heads, batch);
    cfg.blockDim = dim3(128);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_combine_kernel, p);
    if (e != cudaSuccess) return cuda_fail(e, "decode_combine launch");
  }
  return NVATTN_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free decode.
//
// nvattn_paged_decode needs a split-K workspace from its caller. Some callers
// cannot allocate device memory at the point where they run decode: a host
// whose memory manager has already handed the rest of the GPU to the KV cache
// (Nano-vLLM-X sizes its cache to fill gpu_memory_utilization of the device,
// model_runner.py:103-121), a path that must not take cudaMalloc's implicit
// device-wide synchronisation, or a foreign-language host that only holds
// pointers and has no CUDA allocator. For them this variant keeps the
// workspace in a fixed array of device memory that belongs to the library:
// each GPU that loads libnvattn.so holds kNoAllocScratchBytes of it until the
// process exits.
namespace nvattn {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device. In host code the
// symbol itself is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
static int noalloc_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[kNoAllocMaxDevices] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(NVATTN_ERR_UNSUPPORTED, "paged_decode_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "paged_decode_noalloc: cudaGetSymbolAddress");
    addr[dev] = p;
  }
  *out = addr[dev];
  return NVATTN_OK;
}

}  // namespace nvattn

extern "C" int nvattn_paged_decode_noalloc(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* k_cache,
    const void* v_cache, void* out, int64_t o_stride_tok, int64_t o_stride_head,
    const int32_t* cache_seqlens, const int32_t* block_table, int64_t block_table_stride,
    int32_t max_blocks_per_seq, int32_t num_blocks, int32_t block_size, int32_t batch,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
    int32_t* status, void* stream) {
  using namespace nvattn;
  clear_error();
  if (batch == 0) return NVATTN_OK;
  // The same argument checks as nvattn_paged_decode come first, so a bad call
  // gets the same error from both entry points.
  const int bad = check_decode_args(q, q_stride_tok, q_stride_head, k_cache, v_cache, out,
                                    cache_seqlens, block_table, block_table_stride,
                                    max_blocks_per_seq, num_blocks, block_size, batch, num_heads,
                                    num_kv_heads, head_dim);
  if (bad) return bad;
  const size_t need = nvattn_decode_workspace_bytes(batch, num_heads, num_kv_heads,
                                                    max_blocks_per_seq, block_size);
  if (need > kNoAllocScratchBytes) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "paged_decode_noalloc: this batch needs %zu bytes of split-K workspace, more than "
             "the library's fixed %zu-byte scratch; use nvattn_paged_decode with a workspace",
             need, kNoAllocScratchBytes);
    return fail(NVATTN_ERR_WORKSPACE, buf);
  }
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch_address(&scratch);
    if (rc) return rc;
  }
  // Same kernels as nvattn_paged_decode; only the workspace differs. Every
  // partial a call reads is written earlier in that same call, so the
  // scratch needs no clearing between calls.
  return nvattn_paged_decode(q, q_stride_tok, q_stride_head, k_cache, v_cache, out, o_stride_tok,
                             o_stride_head, cache_seqlens, block_table, block_table_stride,
                             max_blocks_per_seq, num_blocks, block_size, batch, num_heads,
                             num_kv_heads, head_dim, softmax_scale, scratch,
                             need > 0 ? kNoAllocScratchBytes : 0, status, stream);
}
