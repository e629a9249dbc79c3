// Host-side helpers shared by all entry points: thread-local error strings and
// TMA descriptor encoding through the runtime's driver entry point.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace nvattn {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                  cudaGetErrorString(err) + ")";
  set_error(m);
  return NVATTN_ERR_CUDA;
}

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

int make_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box,
                    CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return fail(NVATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gstride[i] = strides_bytes[i];
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), gdim,
                   gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d, rank %d)", (int)r,
             rank);
    return fail(NVATTN_ERR_CUDA, buf);
  }
  return NVATTN_OK;
}

}  // namespace nvattn

extern "C" const char* nvattn_last_error(void) { return nvattn::g_last_error.c_str(); }

extern "C" int nvattn_version(void) { return (1 << 16) | 0; }
