// runtime.hpp -- lazily created per-device state of the library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/bjf.h"

namespace bjf {

struct DeviceInfo {
  int device = -1;
  int cc_major = 0;
  int cc_minor = 0;
  int sm_count = 0;
  size_t max_smem_optin = 0;
  int* error_flag = nullptr;  // device int: non-zero after a kernel gave up on a bounded wait
};

// State of the current device (cudaGetDevice()), created on first use.
bjf_status current_device(const DeviceInfo** out);

// cuTensorMapEncodeTiled from the driver (resolved once through the runtime).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
bjf_status encode_tiled_fn(EncodeTiledFn* out);

}  // namespace bjf
