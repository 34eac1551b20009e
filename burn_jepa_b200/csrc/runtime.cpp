// runtime.cpp -- per-device state and driver entry points.
#include "runtime.hpp"

#include <atomic>
#include <mutex>

#include "status.hpp"

namespace bjf {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceInfo g_devices[kMaxDevices];
EncodeTiledFn g_encode = nullptr;
std::atomic<uint64_t> g_wait_limit_ns{kDefaultWaitLimitNs};
std::atomic<int32_t> g_wait_stall{0};
cudaMemPool_t g_pools[kMaxDevices] = {};
}  // namespace

bjf_status stream_alloc(int dev, size_t bytes, cudaStream_t st, void** out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(BJF_ERR_UNSUPPORTED, "device ordinal out of range");
  cudaMemPool_t pool;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_pools[dev]) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      cudaError_t e = cudaMemPoolCreate(&g_pools[dev], &props);
      if (e != cudaSuccess) {
        g_pools[dev] = nullptr;
        return cuda_status(e, "cudaMemPoolCreate");
      }
      uint64_t keep = UINT64_MAX;
      e = cudaMemPoolSetAttribute(g_pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
      if (e != cudaSuccess) return cuda_status(e, "cudaMemPoolSetAttribute");
    }
    pool = g_pools[dev];
  }
  const cudaError_t e = cudaMallocFromPoolAsync(out, bytes, pool, st);
  return e == cudaSuccess ? BJF_OK : cuda_status(e, "cudaMallocFromPoolAsync");
}

bjf_status stream_free(void* p, cudaStream_t st) {
  if (!p) return BJF_OK;
  const cudaError_t e = cudaFreeAsync(p, st);
  return e == cudaSuccess ? BJF_OK : cuda_status(e, "cudaFreeAsync");
}

const DeviceInfo* peek_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  return g_devices[dev].device < 0 ? nullptr : &g_devices[dev];
}

BoundedWait bounded_wait() { return BoundedWait{g_wait_limit_ns.load(), g_wait_stall.load()}; }

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

namespace {

// Reads the device int at `flag` through `st` (synchronising it) and clears it when set.
bjf_status read_and_clear(int* flag, cudaStream_t st, int* out) {
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, flag, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return bjf::cuda_status(e, "device error check");
  if (host) {
    e = cudaMemsetAsync(flag, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return bjf::cuda_status(e, "device error reset");
  }
  *out = host;
  return BJF_OK;
}

}  // namespace

// Reads the flag of every path that has run on the current device: the per-device flag of the
// workspace entry points (only if their state exists -- a device none of them ran on has no
// flag to set) and the no-alloc step's flag in its fixed scratch.  Allocates nothing.
extern "C" bjf_status bjf_device_error_check(bjf_stream_t stream, int32_t* flag_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return bjf::cuda_status(e, "cudaGetDevice");
  cudaStream_t st = bjf::as_cuda(stream);
  int* flags[2] = {nullptr, bjf::no_alloc_error_flag(dev)};
  if (const bjf::DeviceInfo* d = bjf::peek_device(dev)) flags[0] = d->error_flag;
  int any = 0;
  for (int* f : flags) {
    if (!f) continue;
    int v = 0;
    bjf_status rc = read_and_clear(f, st, &v);
    if (rc) return rc;
    any |= v;
  }
  if (!flags[0] && !flags[1]) {  // nothing to read: still the documented synchronisation
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return bjf::cuda_status(e, "device error check");
  }
  if (flag_out) *flag_out = any;
  return BJF_OK;
}

extern "C" bjf_status bjf_set_bounded_wait(uint64_t limit_ns, int32_t stall) {
  if (stall != 0 && stall != 1) return bjf::fail(BJF_ERR_INVALID_ARGUMENT, "stall must be 0 or 1");
  bjf::g_wait_limit_ns.store(limit_ns ? limit_ns : bjf::kDefaultWaitLimitNs);
  bjf::g_wait_stall.store(stall);
  return BJF_OK;
}
