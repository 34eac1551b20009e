// front_end_no_alloc.cu -- bjf_front_end_step for callers that cannot allocate
// device memory.
//
// Some hosts of this front end cannot hand the library a workspace: a Burn/CubeCL
// application whose device memory is owned by the framework's caching allocator and
// which exposes no raw allocation to plugins, or a real-time camera loop that forbids
// allocation after start-up because an allocation can synchronise the device and stall
// the frame.  For them this variant keeps its scratch (patch-diff scores, mask indices,
// counts) in a file-scope __device__ array
// instead of a caller-provided workspace, so a call allocates nothing.  The launches are those
// of bjf_front_end_step: scores -> selection -> gather-GEMM reading its rows from the indices
// and per-stream counts, chained with programmatic dependent launch.
//
// Rules a caller must know:
//  * The array is kNoAllocScratchBytes (4 MiB) per device and lives as long as the
//    library is loaded, on every GPU that loads it.  Steps whose scratch would not fit
//    (streams x tokens above about 520k) are rejected with BJF_ERR_UNSUPPORTED.
//  * Every call on a device shares the one array, and each call overwrites it: calls
//    whose work overlaps on the GPU (different streams, or different host threads
//    without ordering) race and corrupt each other.  Serialise them on one stream.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and clears the array's timeout
//    flag; make that first call before any stream capture begins.  The address is kept
//    for the life of the process, so a device reset (cudaDeviceReset) while the library
//    is loaded is not supported: the array would move and the kept address go stale.
//  * A bounded-wait timeout in the GEMM sets the array's first int, which stays set until
//    bjf_device_error_check reads and clears it (as the workspace step's flag does); no
//    call clears it on entry, so no evidence is lost between calls.
#include <mutex>
#include <string>

#include "common.cuh"
#include "gather_gemm.hpp"
#include "patch_diff.hpp"
#include "runtime.hpp"
#include "status.hpp"

namespace bjf {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

// Scratch of bjf_front_end_step_no_alloc.  Bytes [0, 256) hold the bounded-wait
// timeout flag (cleared once, at set-up; then only by bjf_device_error_check); the step's
// buffers follow.
static __device__ __align__(256) unsigned char g_no_alloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_no_alloc_scratch on the current device `dev`, looked up once per
// device; the set-up also clears the timeout flag (on `st`, ahead of the first step).
bjf_status scratch_address(int dev, cudaStream_t st, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_no_alloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(no-alloc front-end scratch)");
    e = cudaMemsetAsync(p, 0, sizeof(int), st);
    if (e != cudaSuccess) return cuda_status(e, "clear no-alloc scratch flag");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return BJF_OK;
}

struct Carve {
  size_t scores, indices, counts, bytes;
};

Carve carve(int64_t S, int64_t N) {
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  Carve c{};
  size_t off = 256;  // timeout flag
  c.scores = off;
  off = up(off + sizeof(float) * S * N);
  c.indices = off;
  off = up(off + sizeof(int32_t) * S * N);
  c.counts = off;
  off = up(off + sizeof(int32_t) * S);
  c.bytes = off;
  return c;
}

}  // namespace

int* no_alloc_error_flag(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  return static_cast<int*>(g_scratch_addr[dev]);
}

}  // namespace bjf

using namespace bjf;

extern "C" bjf_status bjf_front_end_step_no_alloc(const bjf_front_end_desc* d, const void* video,
                                                  const void* weight, const float* bias, void* caches,
                                                  float* observed, float* age_frames, int32_t age_observed,
                                                  int32_t* counts_out, bjf_stream_t stream) {
  if (!d) return fail(BJF_ERR_INVALID_ARGUMENT, "front-end descriptor must not be null");
  const int64_t v[8] = {d->streams, d->channels, d->frames, d->height, d->width,
                        d->tubelet_size, d->patch_size, d->embed_dim};
  for (int64_t x : v)
    if (x <= 0 || x > (1 << 30)) return fail(BJF_ERR_INVALID_ARGUMENT, "front-end sizes must be positive");
  if (d->frames % d->tubelet_size || d->height % d->patch_size || d->width % d->patch_size)
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "patch-diff sparsity requires frames/height/width divisible by tubelet and patch sizes");
  const int64_t grid[3] = {d->frames / d->tubelet_size, d->height / d->patch_size, d->width / d->patch_size};
  const int64_t N = grid[0] * grid[1] * grid[2];
  const int64_t S = d->streams;
  if (S > 4096 || S * N > INT32_MAX)
    return fail(BJF_ERR_UNSUPPORTED, "the no-alloc front-end step supports up to 4096 streams");
  const Carve c = carve(S, N);
  if (c.bytes > kNoAllocScratchBytes)
    return fail(BJF_ERR_UNSUPPORTED,
                "no-alloc front-end step: streams x tokens = " + std::to_string(S * N) + " needs " +
                    std::to_string(c.bytes) + " bytes of scratch, above the fixed " +
                    std::to_string(kNoAllocScratchBytes) + "-byte limit; use bjf_front_end_step with a workspace");
  if (dtype_size(d->cache_dtype) == 0 || d->cache_dtype == BJF_DTYPE_I32)
    return fail(BJF_ERR_INVALID_ARGUMENT, "cache dtype must be f32, f16 or bf16");
  if (!video || !weight || !caches || !observed || !age_frames)
    return fail(BJF_ERR_INVALID_ARGUMENT, "front-end buffers must not be null");
  SelectParams sel;
  bjf_status rc = resolve_select(&d->mask, grid, sel);
  if (rc) return rc;

  int dev_id = 0;
  cudaError_t e = cudaGetDevice(&dev_id);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev_id < 0 || dev_id >= kMaxDevices) return fail(BJF_ERR_UNSUPPORTED, "device ordinal out of range");
  cudaStream_t st = as_cuda(stream);
  void* base = nullptr;
  rc = scratch_address(dev_id, st, &base);
  if (rc) return rc;
  // Device properties by attribute queries only (nothing here allocates).
  DeviceInfo dev;
  dev.device = dev_id;
  int optin = 0;
  if ((e = cudaDeviceGetAttribute(&dev.cc_major, cudaDevAttrComputeCapabilityMajor, dev_id)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&dev.cc_minor, cudaDevAttrComputeCapabilityMinor, dev_id)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&dev.sm_count, cudaDevAttrMultiProcessorCount, dev_id)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev_id)) != cudaSuccess)
    return cuda_status(e, "cudaDeviceGetAttribute");
  dev.max_smem_optin = (size_t)optin;

  char* ws = static_cast<char*>(base);
  dev.error_flag = reinterpret_cast<int*>(ws);
  float* scores = reinterpret_cast<float*>(ws + c.scores);
  int32_t* indices = reinterpret_cast<int32_t*>(ws + c.indices);
  int32_t* counts = counts_out ? counts_out : reinterpret_cast<int32_t*>(ws + c.counts);

  // The previous call's contents stay in the array.  Every buffer but the timeout flag is
  // fully written before it is read; the flag is left as it is, so a timeout of an earlier
  // call stays visible to bjf_device_error_check.

  const int64_t vd[5] = {1, d->channels, d->frames, d->height, d->width};
  // the cache aging rides at the end of the scores pass when it can, else in the selection
  const ScoresAging aging{age_frames, observed, (long long)(S * N)};
  bool aged = false;
  rc = launch_scores(video, d->video_dtype, vd, S, d->tubelet_size, d->patch_size, scores, st, true, nullptr,
                     age_observed ? &aging : nullptr, &aged);
  if (rc) return rc;
  if (age_observed && !aged) {
    sel.age = age_frames;
    sel.observed = observed;
  }
  rc = launch_select(scores, S, sel, indices, counts, st, true);
  if (rc) return rc;

  GatherGeometry g{};
  g.C = (int)d->channels;
  g.T = (int)d->frames;
  g.H = (int)d->height;
  g.W = (int)d->width;
  g.kt = (int)d->tubelet_size;
  g.ph = (int)d->patch_size;
  g.pw = (int)d->patch_size;
  g.batch = (int)S;
  g.depth = (int)grid[0];
  g.gh = (int)grid[1];
  g.gw = (int)grid[2];
  g.K = (int)(d->channels * d->tubelet_size * d->patch_size * d->patch_size);
  g.D = (int)d->embed_dim;
  EpilogueArgs ep{};
  ep.mode = kEpilogueScatter;
  ep.out = caches;
  ep.out_dtype = d->cache_dtype;
  ep.out_elem_bytes = (int)dtype_size(d->cache_dtype);
  ep.ldo = d->embed_dim;
  ep.dense_tokens = N;
  ep.observed = observed;
  ep.age = age_frames;
  ep.bias = bias;
  const RowSource rows{nullptr, indices, counts, (int)N, (int)S};  // the GEMM scans the counts
  // f32 operands stay on the SIMT kernel here: their tensor-core split needs scratch memory
  return launch_gather_gemm(dev, video, d->video_dtype, weight, d->weight_dtype, g, rows, nullptr, S * N, ep, st,
                            true, /*may_allocate=*/false);
}
