// One-shot all-reduce over NVLink peer memory for the row-parallel linears
// (replaces the dist.all_reduce of RowParallelLinear.forward,
// nanovllm/layers/linear.py:152-155, for decode-sized messages).
//
// Every rank owns one IPC-shared buffer: a 4 KB header of flags, then the
// data region. The rank's GEMM writes its partial product into its own data
// region (local memory only), then one launch of allreduce_oneshot_kernel
//
//   1. announces "partial of launch e ready" to every rank (a release store
//      of e into start[rank] of each rank's header) and waits until every
//      rank has announced e (acquire loads of its own header);
//   2. sums the partials of all ranks, read over NVLink, in rank order in
//      fp32 starting from rank 0's value, rounded once to bf16: every rank
//      computes the same bits, and with two ranks the result is the single
//      rounded bf16 add that NCCL's bf16 sum gives;
//   3. when its last block is done, announces "finished reading launch e"
//      (end[rank] on every rank) and waits for every rank's end flag before
//      the launch completes, so the next GEMM may overwrite the partial.
//
// The launch count e lives in the header (the last block stores it), so a
// captured CUDA graph replays correctly. Every wait is bounded: after about
// a second it records NVATTN_STATUS_TIMEOUT and the kernel finishes.
#include <string.h>

#include "common.cuh"

namespace nvattn {

constexpr int kArMaxRanks = 8;
constexpr int kArThreads = 256;
constexpr size_t kArHeaderBytes = 4096;

struct ArHeader {
  uint32_t start[kArMaxRanks];  // start[p]: last launch whose partial rank p announced
  uint32_t end[kArMaxRanks];    // end[p]: last launch rank p finished reading
  uint32_t epoch;               // launches this rank has completed
  uint32_t done;                // blocks of the running launch that have finished
};

struct ArPeers {
  char* base[kArMaxRanks];  // each rank's buffer (this rank's own at [rank])
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *flag has reached e (wrap-safe), at most kWaitLimitCycles.
__device__ __forceinline__ bool wait_reached(const uint32_t* flag, uint32_t e) {
  const long long t0 = clock64();
  while (static_cast<int32_t>(ld_acquire_sys(flag) - e) < 0) {
    if (clock64() - t0 > kWaitLimitCycles) return false;
    __nanosleep(64);
  }
  return true;
}

// Loads of peer data: volatile (relaxed, system scope), so every launch reads
// what the owner wrote for it and never a line cached from an earlier one.
__device__ __forceinline__ int4 ld_sys_v4(const int4* p) {
  int4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_sys_u16(const unsigned short* p) {
  unsigned short v;
  asm volatile("ld.volatile.global.u16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void add8(float acc[8], const int4 v) {
  const uint32_t w[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y),
                         static_cast<uint32_t>(v.z), static_cast<uint32_t>(v.w)};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t bits = (e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16);
    acc[e] += __uint_as_float(bits);
  }
}

__device__ __forceinline__ void load8(float acc[8], const int4 v) {
  const uint32_t w[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y),
                         static_cast<uint32_t>(v.z), static_cast<uint32_t>(v.w)};
#pragma unroll
  for (int e = 0; e < 8; ++e)
    acc[e] = __uint_as_float((e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16));
}

__device__ __forceinline__ int4 pack8(const float acc[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_int4(static_cast<int>(w[0]), static_cast<int>(w[1]), static_cast<int>(w[2]),
                   static_cast<int>(w[3]));
}

__global__ void __launch_bounds__(kArThreads)
    allreduce_oneshot_kernel(const ArPeers peers, int rank, int world, int64_t n,
                             __nv_bfloat16* __restrict__ out, int32_t* status) {
  ArHeader* mine = reinterpret_cast<ArHeader*>(peers.base[rank]);
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&mine->epoch) + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_epoch;

  // 1. this rank's partial (written by the kernels before this one) is ready;
  // every block announces it, so no block depends on another being resident
  if (threadIdx.x < world) {
    __threadfence_system();
    ArHeader* peer = reinterpret_cast<ArHeader*>(peers.base[threadIdx.x]);
    st_release_sys(&peer->start[rank], e);
    if (!wait_reached(&mine->start[threadIdx.x], e)) s_ok = 0;
  }
  __syncthreads();
  __threadfence_system();  // every thread's data loads come after the flags it waited on
  if (!s_ok && threadIdx.x == 0 && status) atomicOr(status, NVATTN_STATUS_TIMEOUT);

  // 2. sum in rank order (fp32, from rank 0's value), one rounding to bf16
  const int64_t nvec = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kArThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kArThreads + threadIdx.x; i < nvec;
       i += stride) {
    float acc[8];
    load8(acc, ld_sys_v4(reinterpret_cast<const int4*>(peers.base[0] + kArHeaderBytes) + i));
    for (int p = 1; p < world; ++p)
      add8(acc, ld_sys_v4(reinterpret_cast<const int4*>(peers.base[p] + kArHeaderBytes) + i));
    reinterpret_cast<int4*>(out)[i] = pack8(acc);
  }
  if (blockIdx.x == 0) {
    for (int64_t j = nvec * 8 + threadIdx.x; j < n; j += kArThreads) {
      const unsigned short* d0 =
          reinterpret_cast<const unsigned short*>(peers.base[0] + kArHeaderBytes);
      float a = __uint_as_float(ld_sys_u16(d0 + j) << 16);
      for (int p = 1; p < world; ++p) {
        const unsigned short* dp =
            reinterpret_cast<const unsigned short*>(peers.base[p] + kArHeaderBytes);
        a += __uint_as_float(ld_sys_u16(dp + j) << 16);
      }
      out[j] = __float2bfloat16_rn(a);
    }
  }

  // 3. the last block of this rank: finished reading every partial of launch
  // e; wait until every rank has, then record the launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&mine->done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int p = 0; p < world; ++p)
        st_release_sys(&reinterpret_cast<ArHeader*>(peers.base[p])->end[rank], e);
      bool ok = true;
      for (int p = 0; p < world; ++p) ok = wait_reached(&mine->end[p], e) && ok;
      if (!ok && status) atomicOr(status, NVATTN_STATUS_TIMEOUT);
      *reinterpret_cast<volatile uint32_t*>(&mine->done) = 0u;
      *reinterpret_cast<volatile uint32_t*>(&mine->epoch) = e;
      __threadfence();
    }
  }
}

static int ar_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

}  // namespace nvattn

using namespace nvattn;

extern "C" NVATTN_API size_t nvattn_ar_buffer_bytes(int64_t capacity_elems) {
  if (capacity_elems < 0) return 0;
  return kArHeaderBytes + (static_cast<size_t>(capacity_elems) * 2 + 15) / 16 * 16;
}

extern "C" NVATTN_API int nvattn_ar_alloc(size_t bytes, void** buffer, void* ipc_handle) {
  clear_error();
  if (!buffer || !ipc_handle || bytes <= kArHeaderBytes)
    return fail(NVATTN_ERR_INVALID, "ar_alloc: NULL output or size without a data region");
  *buffer = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "ar_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "ar_alloc: zeroing or IPC handle");
  }
  *buffer = p;
  return NVATTN_OK;
}

extern "C" NVATTN_API int nvattn_ar_open(const void* ipc_handle, void** peer_buffer) {
  clear_error();
  if (!ipc_handle || !peer_buffer) return fail(NVATTN_ERR_INVALID, "ar_open: NULL argument");
  *peer_buffer = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "ar_open: cudaIpcOpenMemHandle");
  return NVATTN_OK;
}

extern "C" NVATTN_API int nvattn_ar_close(void* peer_buffer) {
  clear_error();
  if (!peer_buffer) return NVATTN_OK;
  cudaError_t e = cudaIpcCloseMemHandle(peer_buffer);
  if (e != cudaSuccess) return cuda_fail(e, "ar_close: cudaIpcCloseMemHandle");
  return NVATTN_OK;
}

extern "C" NVATTN_API int nvattn_ar_free(void* buffer) {
  clear_error();
  if (!buffer) return NVATTN_OK;
  cudaError_t e = cudaFree(buffer);
  if (e != cudaSuccess) return cuda_fail(e, "ar_free: cudaFree");
  return NVATTN_OK;
}

extern "C" NVATTN_API int nvattn_allreduce(const uint64_t* buffers, int32_t rank, int32_t world,
                                           int64_t num_elems, int64_t capacity_elems, void* out,
                                           int32_t* status, void* stream) {
  clear_error();
  if (world < 1 || world > kArMaxRanks || rank < 0 || rank >= world)
    return fail(NVATTN_ERR_INVALID, "allreduce: world must be 1..8 and 0 <= rank < world");
  if (num_elems < 0 || num_elems > capacity_elems)
    return fail(NVATTN_ERR_INVALID, "allreduce: num_elems outside [0, capacity]");
  if (!buffers || !out) return fail(NVATTN_ERR_INVALID, "allreduce: NULL buffers or out");
  ArPeers peers;
  for (int p = 0; p < kArMaxRanks; ++p) peers.base[p] = nullptr;
  for (int p = 0; p < world; ++p) {
    if (!buffers[p] || buffers[p] % 16 != 0)
      return fail(NVATTN_ERR_INVALID, "allreduce: buffers must be non-NULL and 16-byte aligned");
    peers.base[p] = reinterpret_cast<char*>(buffers[p]);
  }
  if (!aligned16(out)) return fail(NVATTN_ERR_INVALID, "allreduce: out must be 16-byte aligned");
  const uintptr_t own = static_cast<uintptr_t>(buffers[rank]);
  const uintptr_t o = reinterpret_cast<uintptr_t>(out);
  if (o + static_cast<uintptr_t>(num_elems) * 2 > own && o < own + nvattn_ar_buffer_bytes(capacity_elems))
    return fail(NVATTN_ERR_INVALID, "allreduce: out overlaps the shared buffer");
  if (num_elems == 0) return NVATTN_OK;
  const int64_t nvec = num_elems / 8;
  int64_t grid = (nvec + kArThreads - 1) / kArThreads;
  const int64_t cap = 2LL * ar_sms();
  grid = grid < 1 ? 1 : (grid > cap ? cap : grid);
  allreduce_oneshot_kernel<<<static_cast<unsigned>(grid), kArThreads, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(
      peers, rank, world, num_elems, static_cast<__nv_bfloat16*>(out), status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "allreduce_oneshot_kernel");
  return NVATTN_OK;
}
