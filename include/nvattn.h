/*
 * nvattn — B200 (sm_100a) paged-KV attention for Nano-vLLM-X, C ABI.
 *
 * This is the drop-in boundary for the attention hot path of Nano-vLLM-X
 * (nanovllm/layers/attention.py). The reference reaches three GPU routines
 * from that file; each entry point below replaces one of them with the same
 * argument meaning:
 *
 *   store_kvcache_kernel / store_kvcache   attention.py:10-40  -> nvattn_store_kvcache
 *   flash_attn_varlen_func (dense, paged)  attention.py:64-70  -> nvattn_varlen_prefill
 *   flash_attn_with_kvcache (decode)       attention.py:71-74  -> nvattn_paged_decode
 *
 * plus two entry points with no counterpart in the reference, for EAGLE-style
 * speculative verification over the same cache layout:
 *
 *   nvattn_tree_verify   ancestor-masked attention of draft-tree nodes
 *   nvattn_kv_move       compaction of the accepted path's K/V slots
 *
 * and one entry point that fuses the producer side of the path, the steps of
 * Qwen3Attention.forward between the QKV projection and attention
 * (nanovllm/models/qwen3.py:82-86 plus the scatter at attention.py:62-63):
 *
 *   q_norm/k_norm + rotary_emb + store_kvcache  -> nvattn_qk_norm_rope_store
 *
 * and one for the consumer side, the sampler (nanovllm/layers/sampler.py:5-12):
 *
 *   Sampler.forward / greedy argmax              -> nvattn_sample
 *   ParallelLMHead gather + sampling at TP > 1   -> nvattn_sample_shard
 *     (embed_head.py:56-66, sampler.py:5-12)        + nvattn_sample_merge
 *
 * and one for the decode step's metadata (ModelRunner.prepare_decode plus
 * the copies into the decode graph's inputs, model_runner.py:172-188,
 * 204-210):
 *
 *   prepare_decode + graph_vars copies           -> nvattn_decode_prepare
 *
 * and one for the collective next to attention, the all-reduce of the
 * row-parallel linears (o_proj, down_proj; linear.py:152-155), for
 * decode-sized messages:
 *
 *   dist.all_reduce(y) of RowParallelLinear      -> nvattn_allreduce
 *     (+ nvattn_ar_buffer_bytes / _alloc / _open / _close / _free)
 *
 * Conventions (all entry points):
 *   - Pointers are device pointers unless stated otherwise; no torch types.
 *   - Strides are in ELEMENTS (like torch.Tensor.stride()).
 *   - Element type is bf16 (2 bytes); head_dim must be 128.
 *   - KV cache layout is the engine's (nanovllm/engine/model_runner.py:115):
 *     one layer's cache is [num_blocks][block_size][num_kv_heads][head_dim],
 *     contiguous; slot s lives at row s of the [num_blocks*block_size]
 *     x [num_kv_heads*head_dim] view.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). All work is
 *     asynchronous on that stream: no host synchronisation, no allocation,
 *     so every call can be captured in a CUDA graph.
 *   - `status` (nullable) is a device int32. Kernels never trap; when they
 *     meet an input they cannot honour (a slot or block id outside the cache,
 *     a wait that timed out) they skip the offending access and OR a bit from
 *     nvattn_status_bits into *status.
 *   - Return value: NVATTN_OK, or an error code with a message available from
 *     nvattn_last_error() (thread-local). Argument errors are detected on the
 *     host before any launch.
 */
#ifndef NVATTN_H_
#define NVATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NVATTN_API __attribute__((visibility("default")))
#else
#define NVATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum nvattn_error {
  NVATTN_OK = 0,
  NVATTN_ERR_INVALID = 1,     /* bad argument: shape, stride, alignment, NULL */
  NVATTN_ERR_UNSUPPORTED = 2, /* valid for the reference but not built here   */
  NVATTN_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed            */
  NVATTN_ERR_WORKSPACE = 4    /* caller-provided workspace too small          */
};

enum nvattn_status_bits {
  NVATTN_STATUS_BAD_SLOT = 1,   /* slot_mapping entry outside [-1, num_slots)  */
  NVATTN_STATUS_BAD_BLOCK = 2,  /* block_table entry outside [0, num_blocks)   */
  NVATTN_STATUS_TIMEOUT = 4,    /* a pipeline wait gave up (bounded spin)      */
  NVATTN_STATUS_BAD_POSITION = 8 /* position outside [0, max_position) (clamped) */
};

/* Message of the last failed call on this host thread ("" if none). */
NVATTN_API const char* nvattn_last_error(void);

/* ABI version of this library: (major << 16) | minor. */
NVATTN_API int nvattn_version(void);

/*
 * KV-cache scatter. Replaces store_kvcache (nanovllm/layers/attention.py:33-40)
 * and its Triton kernel store_kvcache_kernel (attention.py:10-30):
 *
 *   for i in [0, num_tokens): if slot_mapping[i] != -1:
 *     k_cache[slot_mapping[i]*D : +D] = key[i*key_stride : +D]
 *     v_cache[slot_mapping[i]*D : +D] = value[i*value_stride : +D]
 *
 * D = num_kv_heads*head_dim elements (the reference asserts key.stride(1) ==
 * head_dim, so a token's D elements are contiguous); key_stride/value_stride
 * are the token strides (value is a strided view of the qkv projection in the
 * engine). num_slots = num_blocks*block_size bounds the slot ids: entries
 * outside [-1, num_slots) are skipped and flagged NVATTN_STATUS_BAD_SLOT.
 * Bit-exact copy.
 */
NVATTN_API int nvattn_store_kvcache(const void* key, int64_t key_stride,
                         const void* value, int64_t value_stride,
                         void* k_cache, void* v_cache,
                         const int32_t* slot_mapping, int64_t num_tokens,
                         int64_t D, int64_t num_slots, int32_t* status,
                         void* stream);

/*
 * Variable-length causal prefill. Replaces the call
 *   flash_attn_varlen_func(q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k,
 *                          cu_seqlens_k, softmax_scale, causal=True,
 *                          block_table)
 * at nanovllm/layers/attention.py:67-70.
 *
 *   q   [total_q][num_heads][head_dim]      strides (q_stride_tok, q_stride_head, 1)
 *   out [total_q][num_heads][head_dim]      strides (o_stride_tok, o_stride_head, 1)
 *   block_table == NULL (dense; attention.py:67 with block_tables None):
 *     k, v [total_k][num_kv_heads][head_dim] strides (*_stride_tok, *_stride_head, 1)
 *   block_table != NULL (prefix-cache hit; attention.py:65-66 swaps k,v for
 *   the caches): k, v are the caches [num_blocks][block_size][num_kv_heads]
 *     [head_dim] (contiguous; stride arguments ignored) and sequence b's key j
 *     lives in block block_table[b*block_table_stride + j/block_size];
 *     max_blocks_per_seq is the table width (keys beyond width*block_size are
 *     ignored and flagged NVATTN_STATUS_BAD_BLOCK).
 *
 * cu_seqlens_q must stay within total_q rows (rows past it are not touched).
 *
 * Sequence b owns query rows [cu_seqlens_q[b], cu_seqlens_q[b+1]) and
 * seqlen_k = cu_seqlens_k[b+1]-cu_seqlens_k[b] keys. With causal != 0 the mask
 * is aligned to the bottom-right corner (flash-attn >= 2.1 semantics): query i
 * of a sequence sees keys [0, seqlen_k - seqlen_q + i]; rows that see no key
 * produce 0. Query head h reads KV head h / (num_heads/num_kv_heads).
 * Scores and softmax are fp32; the output is rounded to bf16 once.
 */
NVATTN_API int nvattn_varlen_prefill(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                          const void* k, int64_t k_stride_tok, int64_t k_stride_head,
                          const void* v, int64_t v_stride_tok, int64_t v_stride_head,
                          void* out, int64_t o_stride_tok, int64_t o_stride_head,
                          const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                          int32_t num_seqs, int32_t max_seqlen_q, int32_t max_seqlen_k,
                          int64_t total_q, int64_t total_k,
                          const int32_t* block_table, int64_t block_table_stride,
                          int32_t max_blocks_per_seq, int32_t num_blocks, int32_t block_size,
                          int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                          float softmax_scale, int32_t causal,
                          int32_t* status, void* stream);

/*
 * Paged decode (one query token per sequence). Replaces the call
 *   flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
 *                           cache_seqlens=context_lens, block_table=block_tables,
 *                           softmax_scale, causal=True)
 * at nanovllm/layers/attention.py:72-74.
 *
 *   q   [batch][num_heads][head_dim]   strides (q_stride_tok, q_stride_head, 1)
 *   out [batch][num_heads][head_dim]   strides (o_stride_tok, o_stride_head, 1)
 *   k_cache, v_cache [num_blocks][block_size][num_kv_heads][head_dim]
 *   cache_seqlens[b] keys are read through block_table row b; a row with
 *   cache_seqlens[b] == 0 (CUDA-graph padding, model_runner.py:206-209)
 *   produces zeros. max_blocks_per_seq = block_table width; it fixes the
 *   split-K grid, so the launch shape depends only on host-side sizes.
 *
 * Split-K partials go to `workspace` (device, >= nvattn_decode_workspace_bytes
 * of the same sizes); the library allocates nothing.
 */
NVATTN_API size_t nvattn_decode_workspace_bytes(int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                                     int32_t max_blocks_per_seq, int32_t block_size);

NVATTN_API int nvattn_paged_decode(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                        const void* k_cache, const void* v_cache,
                        void* out, int64_t o_stride_tok, int64_t o_stride_head,
                        const int32_t* cache_seqlens,
                        const int32_t* block_table, int64_t block_table_stride,
                        int32_t max_blocks_per_seq, int32_t num_blocks, int32_t block_size,
                        int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                        int32_t head_dim, float softmax_scale,
                        void* workspace, size_t workspace_bytes,
                        int32_t* status, void* stream);

/*
 * Allocation-free paged decode (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory when they run decode: a host
 * whose allocator already gave the free device memory to the KV cache, a path
 * that must not take cudaMalloc's implicit device-wide synchronisation, or a
 * foreign-language host that holds only pointers. Arguments and results are
 * those of nvattn_paged_decode without the workspace: the split-K partials go
 * to a fixed array of device memory inside the library, 16 MiB
 * (16777216 bytes) on every GPU that loads the library, held until the
 * process exits. A batch whose
 * workspace (nvattn_decode_workspace_bytes) exceeds it is rejected with
 * NVATTN_ERR_WORKSPACE before any launch. Nothing is allocated, by the library
 * or by anything it calls.
 *
 * The first call on a device looks up the array's device address (with that
 * device current) and caches it; make that first call before any stream
 * capture on the device. All calls on a device share the one array and it
 * keeps the last call's contents (nothing in it has to start at zero): calls
 * whose executions can overlap on the GPU (different streams without
 * ordering between them) race on it and must be serialised by the caller.
 */
NVATTN_API int nvattn_paged_decode_noalloc(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                const void* k_cache, const void* v_cache,
                                void* out, int64_t o_stride_tok, int64_t o_stride_head,
                                const int32_t* cache_seqlens,
                                const int32_t* block_table, int64_t block_table_stride,
                                int32_t max_blocks_per_seq, int32_t num_blocks, int32_t block_size,
                                int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                                int32_t head_dim, float softmax_scale,
                                int32_t* status, void* stream);

/*
 * Tree-verification attention (no counterpart in the reference: EAGLE3-style
 * speculative verification, new in this library).
 *
 * Sequence b has context_lens[b] committed tokens in the cache followed by
 * n_b = cu_seqlens_q[b+1]-cu_seqlens_q[b] (<= 64) draft-tree nodes whose K/V
 * were already scattered to cache positions context_lens[b] .. +n_b-1 (node i
 * at position context_lens[b]+i, e.g. by nvattn_store_kvcache). Query row
 * r = cu_seqlens_q[b]+j is node j; it attends every committed token and the
 * tree nodes i whose bit i is set in tree_mask[r] (ancestors and itself).
 * A chain mask (tree_mask[r] = 2^(j+1)-1) is ordinary causal prefill.
 *
 *   q, out [total_q][num_heads][head_dim]; caches and block_table as in
 *   nvattn_varlen_prefill's paged mode; tree_mask [total_q] uint64.
 *
 * `workspace` (device, 256-byte aligned, >= nvattn_tree_workspace_bytes of
 * the same sizes) holds the order in which sequences are dispatched, longest
 * first (written by a small kernel on every call, for up to 1024 sequences),
 * and, when the (sequence, KV head) items are fewer than the SMs, the fp32
 * partials of the context split across CTAs, which a second kernel merges.
 * 0 bytes (more than 1024 sequences and no split) accepts NULL. The split
 * depends only on host-side sizes, so a captured graph keeps its grid.
 */
NVATTN_API size_t nvattn_tree_workspace_bytes(int32_t num_seqs, int32_t max_nodes, int64_t total_q,
                                              int32_t num_heads, int32_t num_kv_heads,
                                              int32_t max_blocks_per_seq, int32_t block_size);

NVATTN_API int nvattn_tree_verify(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                       const void* k_cache, const void* v_cache,
                       void* out, int64_t o_stride_tok, int64_t o_stride_head,
                       const int32_t* cu_seqlens_q, const int32_t* context_lens,
                       const uint64_t* tree_mask,
                       const int32_t* block_table, int64_t block_table_stride,
                       int32_t max_blocks_per_seq, int32_t num_blocks, int32_t block_size,
                       int32_t num_seqs, int32_t max_nodes, int64_t total_q,
                       int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                       float softmax_scale, void* workspace, size_t workspace_bytes,
                       int32_t* status, void* stream);

/*
 * In-cache slot moves, grouped (no counterpart in the reference: compaction
 * of an accepted speculative path). Group g moves rows
 *   src_slots[i] -> dst_slots[i], i in [cu_moves[g], cu_moves[g+1])
 * of both caches (row = D contiguous elements). Every source row of a group is
 * read before any destination row of that group is written, so a group may
 * shift rows onto positions its own sources occupy; different groups must
 * touch disjoint slots. At most 64 moves per group; num_moves is the length of
 * src_slots/dst_slots (group bounds past it are clamped and flagged).
 */
NVATTN_API int nvattn_kv_move(void* k_cache, void* v_cache,
                   const int32_t* src_slots, const int32_t* dst_slots,
                   const int32_t* cu_moves, int32_t num_groups, int32_t num_moves,
                   int64_t D, int64_t num_slots, int32_t* status, void* stream);

/*
 * Fused per-head RMSNorm of q and k, rotary embedding of both, and the K/V
 * cache scatter: one launch for the four steps of
 *   q = q_norm(q); k = k_norm(k)                  (layernorm.py:16-26)
 *   q, k = rotary_emb(positions, q, k)            (rotary_embedding.py:6-14,37-48)
 *   store_kvcache(k, v, k_cache, v_cache, slots)  (attention.py:10-40)
 * q (num_tokens x num_heads x 128), k and v (num_tokens x num_kv_heads x 128)
 * are bf16 rows with the given token strides (views of the fused QKV
 * projection); heads are contiguous within a token. q_weight/k_weight are the
 * bf16 RMSNorm weights (128), `cos_sin` the module's fp32 cache
 * [max_position][cos(64) | sin(64)], `positions` int64 per token.
 * Writes q_out (contiguous num_tokens x num_heads x 128) and, when non-NULL,
 * k_out (contiguous num_tokens x num_kv_heads x 128); when slot_mapping is
 * non-NULL also rotated K and the V row into the caches at each token's slot
 * (slot -1 skipped, as attention.py:23). All arithmetic is fp32, each step
 * rounded (no FMA contraction), in the fixed order documented in
 * csrc/qk_norm_rope.cu, so results are bit-reproducible. Rows, weights,
 * outputs and cos_sin must be 16-byte aligned.
 */
NVATTN_API int nvattn_qk_norm_rope_store(
    const void* q, int64_t q_stride_tok, const void* k, int64_t k_stride_tok,
    const void* v, int64_t v_stride_tok, const void* q_weight, const void* k_weight,
    const float* cos_sin, int64_t max_position, const int64_t* positions,
    const int32_t* slot_mapping, void* q_out, void* k_out, void* k_cache, void* v_cache,
    int64_t num_slots, int64_t num_tokens, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, float eps, int32_t* status, void* stream);

/*
 * One token per row of bf16 logits (num_rows x vocab, row stride in
 * elements): with temperatures[r] > 0 a sample from softmax(logits[r] / T)
 * drawn as argmax(logits/T + Gumbel noise), the same law as the reference's
 * exponential race (sampler.py:9-11), the noise from Philox4x32-10 keyed by
 * `seed` with counter (column/4, row, offset) (23-bit uniforms, exact in
 * fp32 and strictly inside (0, 1), so every noise value is finite);
 * otherwise (temperatures NULL or T <= 0) greedy argmax, first index on
 * ties. NaN and -inf logits are never picked; a row
 * with nothing else gives column 0. Writes out_tokens[r] (int64, 8-byte
 * aligned; it holds intermediate keys until the call's last kernel).
 * Columns must number below 2^32.
 */
NVATTN_API int nvattn_sample(const void* logits, int64_t row_stride, int64_t num_rows,
                             int64_t vocab, const float* temperatures, uint64_t seed,
                             uint64_t offset, int64_t* out_tokens, void* stream);

/*
 * The same pick over one vocabulary shard: logits hold global columns
 * [vocab_offset, vocab_offset + vocab_shard) of each row (the rank's slice of
 * ParallelLMHead's output, embed_head.py:56-61), and the noise of column c is
 * the one nvattn_sample gives column c of the whole row. Writes one 64-bit
 * key per row (unsigned order = pick order: monotone score bits, then
 * 0xFFFFFFFF - column; 0 = no candidate). With the same seed, offset and
 * temperatures on every rank, the largest key over the shards is the key of
 * nvattn_sample's pick on the gathered row, so ranks exchange num_rows x 8
 * bytes instead of the logits. vocab_offset % 4 == 0 keeps the vector path.
 */
NVATTN_API int nvattn_sample_shard(const void* logits, int64_t row_stride, int64_t num_rows,
                                   int64_t vocab_shard, int64_t vocab_offset,
                                   const float* temperatures, uint64_t seed, uint64_t offset,
                                   uint64_t* out_keys, void* stream);

/*
 * keys: num_shards x num_rows keys from nvattn_sample_shard (e.g. an
 * all-gather over the ranks). out_tokens[r] = the column of the largest
 * keys[s][r] over s, or 0 when no shard has a candidate.
 */
NVATTN_API int nvattn_sample_merge(const uint64_t* keys, int64_t num_shards, int64_t num_rows,
                                   int64_t* out_tokens, void* stream);

/*
 * Decode-step metadata from one packed host record per sequence.
 * packed layout (num_seqs = B, table_width = W, 8-byte aligned):
 *   int64 last_token[B] | int32 num_tokens[B] | int32 table_len[B] |
 *   int32 block_table[B][W]  (each row padded with -1)
 * num_tokens is len(seq) with the new token (sequence.py:33), table_len is
 * len(seq.block_table). If packed_host is non-NULL the call first copies the
 * record (nvattn_decode_prepare_bytes(B, W) bytes) into packed_dev on the
 * stream (use pinned memory, and keep it unchanged until the copy is done);
 * with packed_host NULL, packed_dev already holds it. Then one kernel writes,
 * for r < B:
 *   input_ids[r] = last_token, positions[r] = num_tokens - 1,
 *   context_lens[r] = num_tokens,
 *   slot_mapping[r] = block_table[r][table_len-1] * block_size
 *       + num_tokens - (ceil(num_tokens / block_size) - 1) * block_size - 1,
 *   block_tables[r][0:W] = block_table[r] (row stride bt_row_stride),
 * exactly as ModelRunner.prepare_decode (model_runner.py:172-188) and its
 * graph-input copies (:204-210) leave them, and for B <= r < pad_rows
 * slot_mapping = -1 and context_lens = 0 (the padding rows of a captured
 * batch). Any output pointer may be NULL (not written). A record that
 * cannot give a slot (table_len outside [1, W], num_tokens < 1 or beyond
 * the table, a negative block id) gets slot -1 and sets
 * NVATTN_STATUS_BAD_SLOT.
 */
NVATTN_API size_t nvattn_decode_prepare_bytes(int64_t num_seqs, int32_t table_width);

NVATTN_API int nvattn_decode_prepare(const void* packed_host, void* packed_dev, int64_t num_seqs,
                                     int32_t table_width, int32_t block_size, int64_t pad_rows,
                                     int64_t* input_ids, int64_t* positions,
                                     int32_t* slot_mapping, int32_t* context_lens,
                                     int32_t* block_tables, int64_t bt_row_stride,
                                     int32_t* status, void* stream);

/*
 * One-shot all-reduce (sum) of bf16 partials over NVLink peer memory, for
 * the dist.all_reduce of RowParallelLinear.forward (linear.py:152-155).
 *
 * Set-up, once per process (not per step): each rank allocates one buffer of
 * nvattn_ar_buffer_bytes(capacity_elems) with nvattn_ar_alloc (zeroed; it
 * returns the 64-byte CUDA IPC handle), the ranks exchange handles, and each
 * rank opens its peers' with nvattn_ar_open. A buffer is a 4096-byte header
 * of flags, two data halves of capacity_elems bf16 each, then two receive
 * areas of 8 slots (one per sending rank) of 16 bytes per 4 elements of
 * min(capacity_elems, 262144); calls alternate between the halves and areas.
 * Small messages (at most 262144 elements and (world - 1) * 4 * num_elems
 * bytes of pushed traffic within 4 MiB) are pushed into the peers' receive
 * areas with the launch number beside every 4-byte word; larger ones are
 * published in the rank's own half and read by the peers.
 *
 * Per call: `in` holds the rank's partial (num_elems bf16, written by earlier
 * work on `stream`); buffers[p] is rank p's buffer as mapped in this process
 * (own buffer at [rank]). Every rank of the group must make the same sequence
 * of calls with the same num_elems. out receives the sum over ranks,
 * accumulated in fp32 in rank order from rank 0's value and rounded once to
 * bf16: the same bits on every rank (with two ranks, the single rounded add
 * of NCCL's bf16 sum). in and out are 16-byte aligned, outside the shared
 * buffer, and may be the same tensor (in place). The kernel copies `in` into
 * the shared buffer itself, so `in` may be rewritten as soon as the call's
 * kernel has run. Waits on peers are bounded (about a second by default;
 * nvattn_ar_set_wait_limit changes it): on expiry NVATTN_STATUS_TIMEOUT is
 * set, the kernel finishes, and that call's output is not valid.
 * Graph-capturable: the launch count lives in the buffer header.
 */
NVATTN_API size_t nvattn_ar_buffer_bytes(int64_t capacity_elems);
NVATTN_API int nvattn_ar_alloc(size_t bytes, void** buffer, void* ipc_handle);
NVATTN_API int nvattn_ar_open(const void* ipc_handle, void** peer_buffer);
NVATTN_API int nvattn_ar_close(void* peer_buffer);
NVATTN_API int nvattn_ar_free(void* buffer);
NVATTN_API int nvattn_allreduce(const uint64_t* buffers, int32_t rank, int32_t world,
                                int64_t num_elems, int64_t capacity_elems, const void* in,
                                void* out, int32_t* status, void* stream);
/*
 * Sets the limit, in SM clock cycles, of every later nvattn_allreduce
 * launch's waits on its peers (a launch captured in a CUDA graph keeps the
 * limit it was captured with); cycles <= 0 restores the default of 2e9
 * (about a second). Returns the previous limit. Tests shorten it to see a
 * wait on a peer that never arrives end with NVATTN_STATUS_TIMEOUT.
 */
NVATTN_API int64_t nvattn_ar_set_wait_limit(int64_t cycles);
/*
 * Which protocol nvattn_allreduce takes for num_elems over world ranks with
 * buffers of capacity_elems: 1 = words pushed into the peers' receive areas
 * (small messages; the faster one), 0 = halves published and read by the
 * peers, -1 = such a call is invalid. Lets a caller keep another all-reduce
 * for the sizes where this one is not the faster.
 */
NVATTN_API int32_t nvattn_ar_protocol(int32_t world, int64_t num_elems, int64_t capacity_elems);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* NVATTN_H_ */
