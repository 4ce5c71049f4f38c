// host_util.h -- host-side helpers shared by the C-ABI entry points.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/theorem_b200.h"

namespace thm {

// Encode a tiled TMA descriptor (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the library does not link libcuda directly).
//   dims[0] is the innermost (contiguous) extent; strides_bytes has rank-1
//   entries (stride of dims[1..rank-1]); box[i] <= 256. The default swizzle
//   (128 B, 16-B chunks) matches UMMA layout 2; MN-major tf32 operands need
//   CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B (UMMA layout 1).
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// THM_OK, or THM_ERR_CUDA if the last launch failed.
int check_launch();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace thm

// Per translation unit device-status readers (defined next to each kernel).
int thm_internal_status_conv(unsigned* s, int reset);
int thm_internal_status_wu(unsigned* s, int reset);
int thm_internal_status_h(unsigned* s, int reset);
int thm_internal_status_o(unsigned* s, int reset);
int thm_internal_status_ho(unsigned* s, int reset);
int thm_internal_status_selftest(unsigned* s, int reset);

// Reads (optionally clears) a TU's status symbol.
#define THM_STATUS_READER(fn, sym)                                                   \
  int fn(unsigned* s, int reset) {                                                   \
    unsigned v = 0;                                                                  \
    if (cudaMemcpyFromSymbol(&v, sym, sizeof(v)) != cudaSuccess) return THM_ERR_CUDA; \
    if (reset) {                                                                     \
      unsigned z = 0;                                                                \
      if (cudaMemcpyToSymbol(sym, &z, sizeof(z)) != cudaSuccess) return THM_ERR_CUDA; \
    }                                                                                \
    *s = v;                                                                          \
    return THM_OK;                                                                   \
  }
