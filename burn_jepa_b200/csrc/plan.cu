// plan.cu -- device-resident sparse patchify plans.
//
// `SparsePatchifyPlan::new` / `SparsePatchifyBatchPlan::new` (burn_jepa
// src/sparse_patchify.rs:236-330) build the coords table (batch, tubelet, row,
// col) on the host and upload it every time the mask changes.  Here the table is
// written on the device straight from the mask kernel's compacted indices, so a
// new mask never crosses PCIe.  Token index -> (tubelet, row, col) follows
// token_index_to_coords (src/positional.rs:10-17).
#include "common.cuh"
#include "patch_diff.hpp"
#include "status.hpp"

namespace bjf {
namespace {

constexpr int kPlanThreads = 256;
constexpr int kMaxPlanBatch = 4096;

__global__ void __launch_bounds__(kPlanThreads)
    plan_coords_kernel(const int32_t* __restrict__ indices, int index_stride,
                       const int32_t* __restrict__ counts, int mask_rows, int batch, int depth,
                       int gh, int gw, int4* __restrict__ coords, long long capacity,
                       int32_t* __restrict__ total_rows) {
  __shared__ long long offsets[kMaxPlanBatch + 1];
  pdl_wait();  // indices / counts come from the kernel before (the selection)
  // Row offsets: exclusive prefix of the per-batch-row lengths (computed by every CTA).
  if (threadIdx.x == 0) {
    long long acc = 0;
    for (int b = 0; b < batch; ++b) {
      offsets[b] = acc;
      int mr = mask_rows == 1 ? 0 : b;
      int c = counts ? counts[mr] : index_stride;
      c = c < 0 ? 0 : (c > index_stride ? index_stride : c);
      acc += c;
    }
    offsets[batch] = acc;
  }
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 && total_rows) {
    long long t = offsets[batch];
    total_rows[0] = t > 0x7fffffffLL ? 0x7fffffff : (int32_t)t;
  }
  const int tpf = gh * gw;
  const int n = depth * tpf;
  for (int b = blockIdx.x; b < batch; b += gridDim.x) {
    const int mr = mask_rows == 1 ? 0 : b;
    const long long base = offsets[b];
    const int cnt = (int)(offsets[b + 1] - base);
    const int32_t* src = indices + (long long)mr * index_stride;
    for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
      long long row = base + i;
      if (row >= capacity) break;
      int idx = src[i];
      int4 c;
      c.x = b;
      if (idx < 0 || idx >= n) {
        c.y = -1; c.z = -1; c.w = -1;
      } else {
        int t = idx / tpf;
        int rem = idx - t * tpf;
        int r = rem / gw;
        c.y = t;
        c.z = r;
        c.w = rem - r * gw;
      }
      coords[row] = c;
    }
  }
}

}  // namespace
}  // namespace bjf

using namespace bjf;

namespace bjf {

bjf_status launch_plan(const int32_t* indices, int64_t index_stride, const int32_t* counts, int64_t mask_rows,
                       int64_t batch, const int64_t grid[3], int32_t* coords, int64_t coords_capacity,
                       int32_t* total_rows, cudaStream_t st, bool pdl) {
  if (batch <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify batch must be nonzero");
  if (!grid || grid[0] <= 0 || grid[1] <= 0 || grid[2] <= 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify grid must be non-empty");
  if (mask_rows != 1 && mask_rows != batch)
    return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify mask rows must be 1 or equal the batch");
  if (index_stride < 0 || index_stride > INT32_MAX) return fail(BJF_ERR_INVALID_ARGUMENT, "index stride out of range");
  if (batch > kMaxPlanBatch) return fail(BJF_ERR_UNSUPPORTED, "sparse patchify plans support up to 4096 batch rows");
  if (grid[0] * grid[1] * grid[2] > INT32_MAX) return fail(BJF_ERR_UNSUPPORTED, "token grid too large");
  if (coords_capacity < 0) return fail(BJF_ERR_INVALID_ARGUMENT, "coords capacity must be non-negative");
  if ((index_stride > 0 && !indices) || (coords_capacity > 0 && !coords))
    return fail(BJF_ERR_INVALID_ARGUMENT, "indices and coords must not be null");
  if (reinterpret_cast<uintptr_t>(coords) % 16 != 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "coords must be 16-byte aligned");
  int blocks = (int)(batch < 1184 ? batch : 1184);
  cudaError_t e = launch_kernel(pdl, plan_coords_kernel, dim3(blocks), dim3(kPlanThreads), 0, st, indices,
                                (int)index_stride, counts, (int)mask_rows, (int)batch, (int)grid[0], (int)grid[1],
                                (int)grid[2], reinterpret_cast<int4*>(coords), (long long)coords_capacity,
                                total_rows);
  return e == cudaSuccess ? BJF_OK : cuda_status(e, "sparse patchify plan launch");
}

}  // namespace bjf

extern "C" bjf_status bjf_sparse_patchify_plan_coords(const int32_t* indices, int64_t index_stride,
                                                      const int32_t* counts, int64_t mask_rows,
                                                      int64_t batch, const int64_t grid[3],
                                                      int32_t* coords, int64_t coords_capacity,
                                                      int32_t* total_rows, bjf_stream_t stream) {
  return launch_plan(indices, index_stride, counts, mask_rows, batch, grid, coords, coords_capacity, total_rows,
                     as_cuda(stream), false);
}
