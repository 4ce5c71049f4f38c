// capi.cu -- C-ABI utilities (status strings, device status, version) and the
// host helpers declared in host_util.h.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "host_util.h"

namespace thm {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess && fn != nullptr) {
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
}  // namespace

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) return THM_ERR_NO_DRIVER;
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
  CUresult r = g_encode(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? THM_OK : THM_ERR_INVALID;
}

int check_launch() { return cudaGetLastError() == cudaSuccess ? THM_OK : THM_ERR_CUDA; }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace thm

extern "C" {

const char* thm_status_string(int status) {
  switch (status) {
    case THM_OK: return "THM_OK";
    case THM_ERR_INVALID: return "THM_ERR_INVALID (bad shape, size or null pointer)";
    case THM_ERR_UNSUPPORTED: return "THM_ERR_UNSUPPORTED (size or dtype not built for sm_100a here)";
    case THM_ERR_ALIGNMENT: return "THM_ERR_ALIGNMENT (pointer not 16-byte aligned)";
    case THM_ERR_CUDA: return "THM_ERR_CUDA (CUDA launch or runtime error)";
    case THM_ERR_TIMEOUT: return "THM_ERR_TIMEOUT (an in-kernel wait ran out of time)";
    case THM_ERR_NO_DRIVER: return "THM_ERR_NO_DRIVER (cuTensorMapEncodeTiled unavailable)";
    default: return "THM_ERR_UNKNOWN";
  }
}

int thm_get_device_status(int* device_status, int reset) {
  if (device_status == nullptr) return THM_ERR_INVALID;
  if (cudaDeviceSynchronize() != cudaSuccess) return THM_ERR_CUDA;
  unsigned acc = 0, s = 0;
  int (*readers[])(unsigned*, int) = {thm_internal_status_conv, thm_internal_status_wu, thm_internal_status_h,
                                      thm_internal_status_o, thm_internal_status_ho,
                                      thm_internal_status_selftest};
  for (auto rd : readers) {
    int r = rd(&s, reset);
    if (r != THM_OK) return r;
    if (acc == 0) acc = s;
  }
  *device_status = (int)acc;
  return THM_OK;
}

int thm_version(void) { return (0 << 16) | 1; }

}  // extern "C"
