// status.hpp -- error reporting shared by the C ABI entry points.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/bjf.h"

namespace bjf {

// Records `msg` as this thread's last error and returns `code`.
bjf_status fail(bjf_status code, const std::string& msg);

// Maps a CUDA error to BJF_ERR_CUDA with a message naming `what`.
bjf_status cuda_status(cudaError_t err, const char* what);

// Returns BJF_OK or the status of the last launch on this thread.
inline bjf_status check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? BJF_OK : cuda_status(err, what);
}

inline cudaStream_t as_cuda(bjf_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Shape formatting helpers for messages that mirror the reference's wording.
std::string dims_str(const int64_t* dims, int n);

// Message of the last failing call on this thread.
const std::string& last_error();

}  // namespace bjf
