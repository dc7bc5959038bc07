// Host runtime of the C ABI: error state, device properties, version.
#include <cstdarg>
#include <cstdio>

#include <atomic>

#include <cudaTypedefs.h>

#include "fxp_common.cuh"
#include "tma.cuh"

namespace fxpr {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
    return FXPR_ERR_CUDA;
  }
  return FXPR_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

namespace tma {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> fn{nullptr};
  PFN_cuTensorMapEncodeTiled_v12000 f = fn.load(std::memory_order_acquire);
  if (f == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
      return nullptr;
    f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    fn.store(f, std::memory_order_release);
  }
  return f;
}

bool encode_4d_u16(CUtensorMap* map, const void* base, const uint64_t dims[4],
                   const uint64_t strides_bytes[3], const uint32_t box[4]) {
  PFN_cuTensorMapEncodeTiled_v12000 f = encode_fn();
  if (f == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  const cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  cuuint64_t gd[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gs[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  const CUresult r = f(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(base), gd, gs, bx,
                       elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return false;
  }
  return true;
}

}  // namespace tma

}  // namespace fxpr

extern "C" int fxpr_abi_version(void) { return FXPR_ABI_VERSION; }
extern "C" const char* fxpr_last_error(void) { return fxpr::g_err; }
