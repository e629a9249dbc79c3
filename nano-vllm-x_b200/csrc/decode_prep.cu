// Decode-step metadata on the device (replaces ModelRunner.prepare_decode,
// nanovllm/engine/model_runner.py:172-188, and the copies into the captured
// graph's static inputs, model_runner.py:204-210).
//
// The reference builds five Python lists per decode step, turns each into a
// pinned tensor, copies each to the GPU, then (CUDA-graph path) runs seven
// small copy/fill operations into the graph's static buffers. Here the host
// packs only what it alone knows, one record per sequence, into one buffer:
//
//   int64 last_token[B] | int32 num_tokens[B] | int32 table_len[B] |
//   int32 block_table[B][W]   (rows padded with -1, W = widest table)
//
// One copy moves it to the device and one kernel derives the rest, writing
// straight into the caller's buffers (the graph's static inputs):
//
//   input_ids[r]    = last_token[r]                          (:178)
//   positions[r]    = num_tokens[r] - 1                      (:179)
//   context_lens[r] = num_tokens[r]                          (:180)
//   slot_mapping[r] = table[r][table_len-1] * block_size
//                     + num_tokens - (ceil(num_tokens / block_size) - 1) * block_size - 1
//                                                            (:181, sequence.py:56-61)
//   block_tables[r][0:W] = table[r][0:W]                     (:123-127, :209)
//
// and, for rows B <= r < pad_rows, slot_mapping = -1 and context_lens = 0
// (the fill_(-1) / zero_() of :205-208); input ids, positions and table
// columns past W are left as they are, as the reference leaves them.
// A record whose table_len is outside [1, W], whose num_tokens is below 1 or
// beyond its table, or whose last block id is negative gets slot -1 (the
// scatter skips it) and sets NVATTN_STATUS_BAD_SLOT.
#include "common.cuh"

namespace nvattn {

constexpr int kPrepThreads = 256;

struct PrepArgs {
  const int64_t* last_token;
  const int32_t* num_tokens;
  const int32_t* table_len;
  const int32_t* tables;  // [B][W]
  int64_t B;
  int32_t W;
  int32_t block_size;
  int64_t pad_rows;
  int64_t* input_ids;
  int64_t* positions;
  int32_t* slot_mapping;
  int32_t* context_lens;
  int32_t* block_tables;
  int64_t bt_stride;
  int32_t* status;
};

// One thread per (row, table column) for the table copy; column-0 threads
// also write the row's scalars. Rows past B only get their padding.
__global__ void __launch_bounds__(kPrepThreads) decode_prepare_kernel(const PrepArgs a) {
  const int64_t cols = a.W > 0 ? a.W : 1;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kPrepThreads + threadIdx.x;
  const int64_t r = i / cols, c = i - r * cols;
  if (r >= a.pad_rows) return;
  if (r >= a.B) {
    if (c == 0) {
      if (a.slot_mapping) a.slot_mapping[r] = -1;
      if (a.context_lens) a.context_lens[r] = 0;
    }
    return;
  }
  if (a.block_tables && c < a.W) a.block_tables[r * a.bt_stride + c] = a.tables[r * a.W + c];
  if (c != 0) return;
  const int32_t n = a.num_tokens[r];
  const int32_t len = a.table_len[r];
  if (a.input_ids) a.input_ids[r] = a.last_token[r];
  if (a.positions) a.positions[r] = static_cast<int64_t>(n) - 1;
  if (a.context_lens) a.context_lens[r] = n;
  if (a.slot_mapping) {
    const int64_t bs = a.block_size;
    const int64_t nblocks = (static_cast<int64_t>(n) + bs - 1) / bs;
    int32_t slot = -1;
    bool ok = n >= 1 && len >= 1 && len <= a.W && nblocks <= len;
    if (ok) {
      const int64_t last = a.tables[r * a.W + (len - 1)];
      const int64_t s = last * bs + n - (nblocks - 1) * bs - 1;
      ok = last >= 0 && s <= 0x7fffffffLL;
      if (ok) slot = static_cast<int32_t>(s);
    }
    a.slot_mapping[r] = slot;
    if (!ok && a.status) atomicOr(a.status, NVATTN_STATUS_BAD_SLOT);
  }
}

}  // namespace nvattn

using namespace nvattn;

extern "C" NVATTN_API size_t nvattn_decode_prepare_bytes(int64_t num_seqs, int32_t table_width) {
  if (num_seqs < 0 || table_width < 0) return 0;
  return static_cast<size_t>(num_seqs) * (16 + 4 * static_cast<size_t>(table_width));
}

extern "C" NVATTN_API int nvattn_decode_prepare(
    const void* packed_host, void* packed_dev, int64_t num_seqs, int32_t table_width,
    int32_t block_size, int64_t pad_rows, int64_t* input_ids, int64_t* positions,
    int32_t* slot_mapping, int32_t* context_lens, int32_t* block_tables, int64_t bt_row_stride,
    int32_t* status, void* stream) {
  clear_error();
  if (num_seqs < 0 || table_width < 0 || block_size <= 0 || pad_rows < num_seqs)
    return fail(NVATTN_ERR_INVALID, "decode_prepare: bad sizes (need pad_rows >= num_seqs)");
  if (num_seqs > 0 && table_width == 0)
    return fail(NVATTN_ERR_INVALID, "decode_prepare: a sequence needs a block table");
  if (block_tables && bt_row_stride < table_width)
    return fail(NVATTN_ERR_INVALID, "decode_prepare: block_tables row stride below the width");
  if (pad_rows == 0) return NVATTN_OK;
  if (num_seqs > 0 && !packed_dev) return fail(NVATTN_ERR_INVALID, "decode_prepare: NULL packed_dev");
  if (reinterpret_cast<uintptr_t>(packed_dev) % 8 != 0 ||
      reinterpret_cast<uintptr_t>(packed_host) % 8 != 0)
    return fail(NVATTN_ERR_INVALID, "decode_prepare: packed buffers must be 8-byte aligned");
  const int64_t cols = table_width > 0 ? table_width : 1;
  if (pad_rows > (0x7fffffffLL * kPrepThreads) / cols)
    return fail(NVATTN_ERR_INVALID, "decode_prepare: too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t bytes = nvattn_decode_prepare_bytes(num_seqs, table_width);
  if (packed_host && bytes > 0) {
    cudaError_t e = cudaMemcpyAsync(packed_dev, packed_host, bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "decode_prepare: host-to-device copy");
  }
  PrepArgs a;
  const char* base = static_cast<const char*>(packed_dev);
  a.last_token = reinterpret_cast<const int64_t*>(base);
  a.num_tokens = reinterpret_cast<const int32_t*>(base + 8 * num_seqs);
  a.table_len = reinterpret_cast<const int32_t*>(base + 12 * num_seqs);
  a.tables = reinterpret_cast<const int32_t*>(base + 16 * num_seqs);
  a.B = num_seqs;
  a.W = table_width;
  a.block_size = block_size;
  a.pad_rows = pad_rows;
  a.input_ids = input_ids;
  a.positions = positions;
  a.slot_mapping = slot_mapping;
  a.context_lens = context_lens;
  a.block_tables = block_tables;
  a.bt_stride = bt_row_stride;
  a.status = status;
  const int64_t threads = pad_rows * cols;
  const unsigned grid = static_cast<unsigned>((threads + kPrepThreads - 1) / kPrepThreads);
  decode_prepare_kernel<<<grid, kPrepThreads, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode_prepare_kernel");
  return NVATTN_OK;
}
