// status.cpp -- thread-local last-error storage for the C ABI.
#include "status.hpp"

#include <cstring>

namespace bjf {

namespace {
thread_local std::string g_last_error;
}

bjf_status fail(bjf_status code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

bjf_status cuda_status(cudaError_t err, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")";
  return BJF_ERR_CUDA;
}

std::string dims_str(const int64_t* dims, int n) {
  std::string s = "[";
  for (int i = 0; i < n; ++i) {
    if (i) s += ",";
    s += std::to_string(dims[i]);
  }
  return s + "]";
}

const std::string& last_error() { return g_last_error; }

}  // namespace bjf

extern "C" {

int32_t bjf_abi_version(void) { return BJF_ABI_VERSION; }

size_t bjf_get_last_error_string(char* buf, size_t len) {
  const std::string& e = bjf::last_error();
  if (buf && len > 0) {
    size_t n = e.size() < len - 1 ? e.size() : len - 1;
    std::memcpy(buf, e.data(), n);
    buf[n] = '\0';
  }
  return e.size();
}

}  // extern "C"
