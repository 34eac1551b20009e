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

// State of device `dev` if current_device() has created it, else nullptr (creates nothing).
const DeviceInfo* peek_device(int dev);

// Device address of the timeout flag of bjf_front_end_step_no_alloc on device `dev`, or
// nullptr when that step has never been set up there (front_end_no_alloc.cu).
int* no_alloc_error_flag(int dev);

// Time limit of the bounded pipeline waits of the gather-GEMM kernels, and the stall switch
// of bjf_set_bounded_wait (launches enqueued after a change use the new values).
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;
struct BoundedWait {
  uint64_t limit_ns;
  int32_t stall;
};
BoundedWait bounded_wait();

// Stream-ordered device memory from the library's own pool on device `dev` (a pool per
// device, created on first use, that keeps freed memory for the next call instead of
// returning it to the driver).  Capturable in a CUDA graph.
bjf_status stream_alloc(int dev, size_t bytes, cudaStream_t st, void** out);
bjf_status stream_free(void* p, cudaStream_t st);

// cuTensorMapEncodeTiled from the driver (resolved once through the runtime).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
bjf_status encode_tiled_fn(EncodeTiledFn* out);

}  // namespace bjf
