// runtime.cpp -- per-device state and driver entry points.
#include "runtime.hpp"

#include <mutex>

#include "status.hpp"

namespace bjf {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceInfo g_devices[kMaxDevices];
EncodeTiledFn g_encode = nullptr;
}  // namespace

bjf_status current_device(const DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(BJF_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_devices[dev];
  if (d.device < 0) {
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
    int* flag = nullptr;
    e = cudaMalloc(&flag, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "cudaMalloc(error flag)");
    e = cudaMemset(flag, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "cudaMemset(error flag)");
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.sm_count = prop.multiProcessorCount;
    d.max_smem_optin = prop.sharedMemPerBlockOptin;
    d.error_flag = flag;
    d.device = dev;
  }
  *out = &d;
  return BJF_OK;
}

bjf_status encode_tiled_fn(EncodeTiledFn* out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(BJF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *out = g_encode;
  return BJF_OK;
}

}  // namespace bjf

extern "C" bjf_status bjf_device_error_check(bjf_stream_t stream, int32_t* flag_out) {
  const bjf::DeviceInfo* d = nullptr;
  bjf_status rc = bjf::current_device(&d);
  if (rc) return rc;
  cudaStream_t st = bjf::as_cuda(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, d->error_flag, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return bjf::cuda_status(e, "device error check");
  if (host) {
    e = cudaMemsetAsync(d->error_flag, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return bjf::cuda_status(e, "device error reset");
  }
  if (flag_out) *flag_out = host;
  return BJF_OK;
}
