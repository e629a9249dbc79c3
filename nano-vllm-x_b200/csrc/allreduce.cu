// One-shot all-reduce over NVLink peer memory for the row-parallel linears
// (replaces the dist.all_reduce of RowParallelLinear.forward,
// nanovllm/layers/linear.py:152-155, for decode-sized messages).
//
// Every rank owns one IPC-shared buffer: a 4 KB header of flags, then two
// data halves of `capacity` bf16 each. Launch e (the rank's e-th call)
// uses half e % 2. The message is cut into one contiguous chunk per block,
// and block b of every rank handles chunk b:
//
//   1. copies its chunk of this rank's input into half e % 2 of the rank's
//      own buffer (local memory only);
//   2. publishes it: a system-scope fence, then a release store of e into
//      flag[rank][b] of every rank's header (one thread per rank);
//   3. waits until flag[p][b] of its own header has reached e for every
//      rank p (acquire loads, bounded);
//   4. sums chunk b of half e % 2 of every rank's buffer, read over NVLink,
//      in rank order in fp32 starting from rank 0's value, rounded once to
//      bf16: every rank computes the same bits, and with two ranks the result
//      is the single rounded bf16 add that NCCL's bf16 sum gives.
//
// No block waits for another block of its own launch, so nothing depends on
// the blocks being co-resident. There is no closing barrier: a rank next
// writes half e % 2 in launch e + 2, which starts after its launch e + 1
// completed; every block of launch e + 1 waited for every peer's launch-e+1
// flags, which a peer publishes only after its own launch e (and its reads of
// half e % 2) completed. The last block to finish records e in the header,
// so a captured CUDA graph replays correctly. Every wait is bounded: after
// the wait limit (about a second by default) it records
// NVATTN_STATUS_TIMEOUT and the kernel finishes; that launch's output is then
// not valid.
//
// Messages up to NVATTN_AR_LL_MAX_ELEMS whose push traffic stays small take a
// second protocol, allreduce_ll_kernel, that carries its flags inside the
// data: every 4-byte word of the message travels in one 64-bit store together
// with the launch number e, so a word is valid as soon as it is seen with e,
// and neither a fence nor a flag round trip nor a read over NVLink lies on
// the path. Each rank pushes its input into its slot of every peer's receive
// area (half e % 2, a slot per sending rank), then waits for every peer's
// words of the same lines in its own memory and sums them in rank order. The
// two halves make overwriting safe by the argument above: a rank reaches
// launch e + 2 only after its launch e + 1 saw every peer's launch-e+1
// words, which a peer pushes only after its own launch e completed. Both
// protocols share the launch count and give the same bits.
#include <string.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"

namespace nvattn {

constexpr int kArMaxRanks = 8;
#ifndef NVATTN_AR_THREADS
#define NVATTN_AR_THREADS 512
#endif
#ifndef NVATTN_AR_VECS_PER_THREAD
#define NVATTN_AR_VECS_PER_THREAD 2
#endif
#ifndef NVATTN_AR_LL_MAX_ELEMS
#define NVATTN_AR_LL_MAX_ELEMS 262144
#endif
#ifndef NVATTN_AR_LL_MAX_TRAFFIC
#define NVATTN_AR_LL_MAX_TRAFFIC (4 << 20)
#endif
#ifndef NVATTN_AR_LL_THREADS
#define NVATTN_AR_LL_THREADS 256
#endif
constexpr int kArThreads = NVATTN_AR_THREADS;
constexpr int64_t kArLLMaxElems = NVATTN_AR_LL_MAX_ELEMS;       // largest message of the LL protocol
// Push bytes per rank the LL protocol may cost: (world - 1) x 4 x elements.
// Measured (max over ranks, 200 back-to-back calls): at 4 ranks 512 KB took
// 13.9 us pushed against 16.7 published; at 8 ranks 256 KB 15.7 against 18.1,
// and 512 KB (7 MB pushed) 23.0 against 20.8.
constexpr int64_t kArLLMaxTraffic = NVATTN_AR_LL_MAX_TRAFFIC;
constexpr int kArLLThreads = NVATTN_AR_LL_THREADS;
constexpr int kArMaxBlocks = 120;
constexpr int kArVecsPerThread = NVATTN_AR_VECS_PER_THREAD;  // 16-byte vectors per thread and rank in flight
constexpr size_t kArHeaderBytes = 4096;

struct ArHeader {
  uint32_t flag[kArMaxRanks][kArMaxBlocks];  // flag[p][b]: last launch whose chunk b rank p published
  uint32_t epoch;                            // launches this rank has completed
  uint32_t done;                             // blocks of the running launch that have finished
};
static_assert(sizeof(ArHeader) <= kArHeaderBytes, "all-reduce header exceeds 4 KB");

struct ArPeers {
  char* base[kArMaxRanks];  // each rank's buffer (this rank's own at [rank])
};

static std::atomic<long long> g_ar_wait_limit{kWaitLimitCycles};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *flag has reached e (wrap-safe), at most `limit` SM cycles.
__device__ __forceinline__ bool wait_reached(const uint32_t* flag, uint32_t e, long long limit) {
  const long long t0 = clock64();
  while (static_cast<int32_t>(ld_acquire_sys(flag) - e) < 0) {
    if (clock64() - t0 > limit) return false;
    __nanosleep(32);
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
                             int64_t half_bytes, int64_t per_block,
                             const __nv_bfloat16* in, __nv_bfloat16* out, int32_t* status,
                             long long wait_limit) {
  ArHeader* mine = reinterpret_cast<ArHeader*>(peers.base[rank]);
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&mine->epoch) + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int b = blockIdx.x;
  const int64_t off = kArHeaderBytes + static_cast<int64_t>(e & 1u) * half_bytes;
  const int64_t nvec = n / 8;
  const int64_t lo = static_cast<int64_t>(b) * per_block;
  const int64_t hi = lo + per_block < nvec ? lo + per_block : nvec;
  const bool tail_block = (b == static_cast<int>(gridDim.x) - 1);

  // 1. this rank's chunk into its own shared half (in may be out: each block
  // reads its chunk of in here, before it writes the same chunk of out)
  int4* own = reinterpret_cast<int4*>(peers.base[rank] + off);
  for (int64_t i = lo + threadIdx.x; i < hi; i += kArThreads)
    own[i] = reinterpret_cast<const int4*>(in)[i];
  if (tail_block) {
    unsigned short* own16 = reinterpret_cast<unsigned short*>(peers.base[rank] + off);
    const unsigned short* in16 = reinterpret_cast<const unsigned short*>(in);
    for (int64_t j = nvec * 8 + threadIdx.x; j < n; j += kArThreads) own16[j] = in16[j];
  }
  __syncthreads();

  // 2-3. publish chunk b of launch e to every rank; wait for every rank's
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(&reinterpret_cast<ArHeader*>(peers.base[threadIdx.x])->flag[rank][b], e);
    if (!wait_reached(&mine->flag[threadIdx.x][b], e, wait_limit)) s_ok = 0;
  }
  __syncthreads();
  if (!s_ok && threadIdx.x == 0 && status) atomicOr(status, NVATTN_STATUS_TIMEOUT);

  // 4. sum in rank order (fp32, from rank 0's value), one rounding to bf16;
  // every rank's loads are issued before the adds
  for (int64_t i0 = lo + threadIdx.x; i0 < hi; i0 += kArThreads * kArVecsPerThread) {
    int4 v[kArVecsPerThread][kArMaxRanks];
#pragma unroll
    for (int u = 0; u < kArVecsPerThread; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * kArThreads;
#pragma unroll
      for (int p = 0; p < kArMaxRanks; ++p)
        if (p < world && i < hi)
          v[u][p] = ld_sys_v4(reinterpret_cast<const int4*>(peers.base[p] + off) + i);
    }
#pragma unroll
    for (int u = 0; u < kArVecsPerThread; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * kArThreads;
      if (i >= hi) break;
      float acc[8];
      load8(acc, v[u][0]);
#pragma unroll
      for (int p = 1; p < kArMaxRanks; ++p)
        if (p < world) add8(acc, v[u][p]);
      reinterpret_cast<int4*>(out)[i] = pack8(acc);
    }
  }
  if (tail_block) {
    for (int64_t j = nvec * 8 + threadIdx.x; j < n; j += kArThreads) {
      float a = __uint_as_float(
          ld_sys_u16(reinterpret_cast<const unsigned short*>(peers.base[0] + off) + j) << 16);
      for (int p = 1; p < world; ++p)
        a += __uint_as_float(
            ld_sys_u16(reinterpret_cast<const unsigned short*>(peers.base[p] + off) + j) << 16);
      out[j] = __float2bfloat16_rn(a);
    }
  }

  // the last block of this rank records launch e
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&mine->done, 1u);
    if (prev == gridDim.x - 1) {
      *reinterpret_cast<volatile uint32_t*>(&mine->done) = 0u;
      *reinterpret_cast<volatile uint32_t*>(&mine->epoch) = e;
      __threadfence();
    }
  }
}

__device__ __forceinline__ void st_sys_v2u64(void* p, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void ld_sys_v2u64(const void* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Four bf16 of the message starting at element 4 * line (zeros past n).
__device__ __forceinline__ uint2 ll_read_line(const __nv_bfloat16* in, int64_t line, int64_t n) {
  const int64_t e0 = line * 4;
  if (e0 + 4 <= n) return reinterpret_cast<const uint2*>(in)[line];
  const unsigned short* in16 = reinterpret_cast<const unsigned short*>(in);
  uint32_t h[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = (e0 + k < n) ? in16[e0 + k] : 0u;
  return make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
}

__device__ __forceinline__ void ll_add(float acc[4], uint2 w, bool first) {
  const float v[4] = {__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                      __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u)};
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k] = first ? v[k] : acc[k] + v[k];
}

// LL protocol. A line is 16 bytes of a receive slot: two 64-bit words, each
// {4 bytes of the message, launch number e}, so 8 bytes of message per line.
// Receive area of a rank: two halves of kArMaxRanks slots (one per sending
// rank) of slot_bytes each, at ll_off in its buffer.
__global__ void __launch_bounds__(kArLLThreads)
    allreduce_ll_kernel(const ArPeers peers, int rank, int world, int64_t n, int64_t ll_off,
                        int64_t slot_bytes, const __nv_bfloat16* in, __nv_bfloat16* out,
                        int32_t* status, long long wait_limit) {
  ArHeader* mine = reinterpret_cast<ArHeader*>(peers.base[rank]);
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&mine->epoch) + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int64_t area = ll_off + static_cast<int64_t>(e & 1u) * kArMaxRanks * slot_bytes;
  const int64_t lines = (n + 3) / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t tag = static_cast<uint64_t>(e) << 32;

  // push this rank's lines into its slot of every peer's receive area
  for (int64_t i = first; i < lines; i += stride) {
    const uint2 w = ll_read_line(in, i, n);
    const uint64_t a = tag | w.x, b = tag | w.y;
#pragma unroll
    for (int p = 0; p < kArMaxRanks; ++p)
      if (p < world && p != rank)
        st_sys_v2u64(peers.base[p] + area + static_cast<int64_t>(rank) * slot_bytes + i * 16, a, b);
  }

  // the same lines from every rank, summed in rank order (fp32, one rounding)
  bool ok = true;
  const long long t0 = clock64();
  for (int64_t i = first; i < lines; i += stride) {
    const uint2 own = ll_read_line(in, i, n);
    float acc[4];
#pragma unroll
    for (int p = 0; p < kArMaxRanks; ++p) {
      if (p >= world) break;
      uint2 w = own;
      if (p != rank) {
        const char* src = peers.base[rank] + area + static_cast<int64_t>(p) * slot_bytes + i * 16;
        uint64_t a = 0, b = 0;
        while (ok) {
          ld_sys_v2u64(src, a, b);
          if ((a >> 32) == e && (b >> 32) == e) break;
          if (clock64() - t0 > wait_limit) ok = false;
        }
        w = make_uint2(static_cast<uint32_t>(a), static_cast<uint32_t>(b));
      }
      ll_add(acc, w, p == 0);
    }
    const int64_t e0 = i * 4;
    const __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0], acc[1]);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2], acc[3]);
    if (e0 + 4 <= n) {
      reinterpret_cast<uint2*>(out)[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                                                    *reinterpret_cast<const uint32_t*>(&hi));
    } else {
      const __nv_bfloat16 v[4] = {lo.x, lo.y, hi.x, hi.y};
      for (int k = 0; k < 4 && e0 + k < n; ++k) out[e0 + k] = v[k];
    }
    if (!ok) break;
  }
  if (!ok) s_ok = 0;
  __syncthreads();
  if (!s_ok && threadIdx.x == 0 && status) atomicOr(status, NVATTN_STATUS_TIMEOUT);

  // the last block of this rank records launch e
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&mine->done, 1u);
    if (prev == gridDim.x - 1) {
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

static size_t ar_half_bytes(int64_t capacity_elems) {
  return (static_cast<size_t>(capacity_elems) * 2 + 15) / 16 * 16;
}

// Bytes of one LL receive slot: a 16-byte line per 4 elements of the largest
// LL message the buffer takes.
static size_t ar_ll_slot_bytes(int64_t capacity_elems) {
  const int64_t cap = std::min<int64_t>(capacity_elems, kArLLMaxElems);
  return static_cast<size_t>((cap + 3) / 4) * 16;
}

extern "C" NVATTN_API size_t nvattn_ar_buffer_bytes(int64_t capacity_elems) {
  if (capacity_elems < 0) return 0;
  return kArHeaderBytes + 2 * ar_half_bytes(capacity_elems) +
         2 * kArMaxRanks * ar_ll_slot_bytes(capacity_elems);
}

// 1 when a call of num_elems over world ranks (buffers of capacity_elems)
// takes the pushed-words protocol, 0 for the published halves, -1 when such a
// call is invalid.
static int ar_protocol(int32_t world, int64_t num_elems, int64_t capacity_elems) {
  if (world < 1 || world > kArMaxRanks || num_elems < 0 || num_elems > capacity_elems) return -1;
  const int64_t ll_cap = std::min<int64_t>(capacity_elems, kArLLMaxElems);
  return (num_elems <= ll_cap && (world - 1) * num_elems * 4 <= kArLLMaxTraffic) ? 1 : 0;
}

extern "C" NVATTN_API int32_t nvattn_ar_protocol(int32_t world, int64_t num_elems,
                                                 int64_t capacity_elems) {
  return ar_protocol(world, num_elems, capacity_elems);
}

extern "C" NVATTN_API int64_t nvattn_ar_set_wait_limit(int64_t cycles) {
  return g_ar_wait_limit.exchange(cycles > 0 ? cycles : kWaitLimitCycles);
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
                                           int64_t num_elems, int64_t capacity_elems,
                                           const void* in, void* out, int32_t* status,
                                           void* stream) {
  clear_error();
  if (world < 1 || world > kArMaxRanks || rank < 0 || rank >= world)
    return fail(NVATTN_ERR_INVALID, "allreduce: world must be 1..8 and 0 <= rank < world");
  if (num_elems < 0 || num_elems > capacity_elems)
    return fail(NVATTN_ERR_INVALID, "allreduce: num_elems outside [0, capacity]");
  if (!buffers || !in || !out) return fail(NVATTN_ERR_INVALID, "allreduce: NULL buffers, in or out");
  ArPeers peers;
  for (int p = 0; p < kArMaxRanks; ++p) peers.base[p] = nullptr;
  for (int p = 0; p < world; ++p) {
    if (!buffers[p] || buffers[p] % 16 != 0)
      return fail(NVATTN_ERR_INVALID, "allreduce: buffers must be non-NULL and 16-byte aligned");
    peers.base[p] = reinterpret_cast<char*>(buffers[p]);
  }
  if (!aligned16(in) || !aligned16(out))
    return fail(NVATTN_ERR_INVALID, "allreduce: in and out must be 16-byte aligned");
  const uintptr_t own = static_cast<uintptr_t>(buffers[rank]);
  const uintptr_t own_end = own + nvattn_ar_buffer_bytes(capacity_elems);
  const uintptr_t bytes = static_cast<uintptr_t>(num_elems) * 2;
  const uintptr_t o = reinterpret_cast<uintptr_t>(out);
  const uintptr_t i = reinterpret_cast<uintptr_t>(in);
  if ((o + bytes > own && o < own_end) || (i + bytes > own && i < own_end))
    return fail(NVATTN_ERR_INVALID, "allreduce: in or out overlaps the shared buffer");
  if (num_elems == 0) return NVATTN_OK;
  if (ar_protocol(world, num_elems, capacity_elems) == 1) {
    const int64_t lines = (num_elems + 3) / 4;
    int64_t grid = (lines + kArLLThreads - 1) / kArLLThreads;
    grid = std::max<int64_t>(1, std::min<int64_t>(grid, ar_sms()));
    allreduce_ll_kernel<<<static_cast<unsigned>(grid), kArLLThreads, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(
        peers, rank, world, num_elems,
        static_cast<int64_t>(kArHeaderBytes + 2 * ar_half_bytes(capacity_elems)),
        static_cast<int64_t>(ar_ll_slot_bytes(capacity_elems)),
        static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), status,
        g_ar_wait_limit.load());
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "allreduce_ll_kernel");
    return NVATTN_OK;
  }
  const int64_t nvec = num_elems / 8;
  const int64_t per_launch = static_cast<int64_t>(kArThreads) * kArVecsPerThread;
  int64_t grid = (nvec + per_launch - 1) / per_launch;
  const int64_t cap = std::min<int64_t>(kArMaxBlocks, ar_sms());
  grid = grid < 1 ? 1 : (grid > cap ? cap : grid);
  const int64_t per_block = (nvec + grid - 1) / grid;
  allreduce_oneshot_kernel<<<static_cast<unsigned>(grid), kArThreads, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(
      peers, rank, world, num_elems, static_cast<int64_t>(ar_half_bytes(capacity_elems)),
      per_block, static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), status,
      g_ar_wait_limit.load());
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "allreduce_oneshot_kernel");
  return NVATTN_OK;
}
