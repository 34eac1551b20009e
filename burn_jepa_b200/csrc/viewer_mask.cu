// viewer_mask.cu -- the live viewer's patch-diff mask policy on the device (burn_jepa
// src/viewer.rs:780-885, 946-961): after the threshold selection of each stream (the "direct"
// mask, selected without dilation),
//
//   1. dense fallback   every token once the direct mask reaches ceil(len * density) tokens
//                       (patch_diff_dense_fallback, :780-793)
//   2. dilation         every token within `dilation` tiles of a direct token, same tubelet,
//                       no cap (dilate_sparse_patch_mask, :796-816, :844-869)  -> write mask
//   3. encode buckets   the write mask padded to the first configured bucket width that holds
//                       it: evenly spaced tokens first, then the lowest missing ones
//                       (bucket_sparse_mask_with_config, :927-944 -> SparseTokenMask::padded_to_len,
//                       src/tokens.rs:94-128)                                    -> encode mask
//
// One 1024-thread CTA per stream holds a keep flag per token in shared memory; every step is
// a parallel mark followed by an ordered block scan, so both masks come out ascending and
// unique as SparseTokenMask::new makes them.
#include <algorithm>
#include <cmath>
#include <string>

#include "../../include/bjf.h"
#include "common.cuh"
#include "patch_diff.hpp"
#include "runtime.hpp"
#include "status.hpp"

namespace bjf {
namespace {

constexpr int kViewerThreads = 1024;
constexpr int kMaxViewerTokens = 32768;
constexpr int kMaxBucketWidths = 32;  // bucket densities; one more width for the grid

struct ViewerParams {
  int n, gh, gw;
  int fallback_tokens;  // ceil(len * clamp(density, 0, 1)), computed as the reference does
  int dilation;
  int bucket_multiple;  // > 0: widths are its multiples below n, then n (no densities)
  int n_widths;         // > 0: the ascending widths below; both 0: encode mask = write mask
  int widths[kMaxBucketWidths + 1];
  // the RGBA mask node's dense shortcuts (crates/bevy_jepa/src/mask.rs:151-168)
  int force_dense;             // patch_diff_can_use_dense_fast_path (src/viewer.rs:1031-1036)
  const float* sample_scores;  // non-null: patch_diff_sampled_dense_fast_path_from_rgba (:1160-1195)
  float sample_threshold;
  int sample_stride, sample_rows, sample_cols, sample_required;
};
// Exclusive scan of one int per thread in thread order; *total gets the block sum.
__device__ __forceinline__ int viewer_scan(int v, int* sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  __syncthreads();
  if (lane == 31) sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < (int)(blockDim.x >> 5) ? sums[lane] : 0;
    int winc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc += y;
    }
    sums[lane] = winc - w;
    if (lane == 31) sums[32] = winc;
  }
  __syncthreads();
  const int r = sums[warp] + inc - v;
  *total = sums[32];
  __syncthreads();
  return r;
}

// Writes the ascending indices of the set flags to out and returns their count.  Each thread
// owns a contiguous segment so the scan order is index order.
__device__ __forceinline__ int compact_flags(const unsigned char* keep, int n, int32_t* out, int* sums) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int b = min(n, (int)threadIdx.x * per), e = min(n, b + per);
  int local = 0;
  for (int i = b; i < e; ++i) local += keep[i] != 0;
  int total;
  int pos = viewer_scan(local, sums, &total);
  for (int i = b; i < e; ++i)
    if (keep[i]) out[pos++] = i;
  return total;
}

__device__ __forceinline__ void write_all(int n, int32_t* out) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = i;
}

// direct_idx / direct_cnt may alias write_idx / write_cnt: every direct index and count is
// read before the write mask is stored.
__global__ void __launch_bounds__(kViewerThreads)
    viewer_mask_kernel(const int32_t* direct_idx, const int32_t* direct_cnt, ViewerParams p, int32_t* write_idx,
                       int32_t* write_cnt, int32_t* __restrict__ enc_idx, int32_t* __restrict__ enc_cnt) {
  extern __shared__ unsigned char keep[];
  __shared__ int sums[33];
  __shared__ int taken_sh;
  pdl_wait();
  const int n = p.n;
  const long long s = blockIdx.x;
  const int m = min(max(direct_cnt[s], 0), n);
  const int32_t* direct = direct_idx + s * n;
  int32_t* wout = write_idx + s * n;
  int32_t* eout = enc_idx + s * n;

  // 0. dense shortcuts of the RGBA mask node: every sampled patch score of the frame is the
  // full scorer's, so the sampled decision reads the stream's scores
  bool dense = p.force_dense != 0;
  if (!dense && p.sample_scores) {
    const int sampled = p.sample_rows * p.sample_cols;
    int local = 0;
    for (int i = threadIdx.x; i < sampled; i += blockDim.x) {
      const int row = (i / p.sample_cols) * p.sample_stride, col = (i % p.sample_cols) * p.sample_stride;
      local += p.sample_scores[s * n + row * p.gw + col] >= p.sample_threshold;
    }
    int active;
    viewer_scan(local, sums, &active);
    dense = sampled > 0 && active >= max(p.sample_required, 1);
  }
  // 1. dense fallback (a dense-ordered mask stays dense through dilation and bucketing)
  if (dense || m == n || (p.fallback_tokens < n && m >= max(p.fallback_tokens, 1))) {
    __syncthreads();  // all direct reads (none here) before the in-place write
    write_all(n, wout);
    write_all(n, eout);
    if (threadIdx.x == 0) {
      write_cnt[s] = n;
      enc_cnt[s] = n;
    }
    return;
  }

  // 2. dilation without a cap (dilation 0: the direct mask itself)
  for (int i = threadIdx.x; i < n; i += blockDim.x) keep[i] = 0;
  __syncthreads();
  const int tpf = p.gh * p.gw;
  for (int j = threadIdx.x; j < m; j += blockDim.x) {
    const int index = direct[j];
    if (index < 0 || index >= n) continue;
    const int t = index / tpf, local = index - t * tpf, row = local / p.gw, col = local - row * p.gw;
    const int r0 = max(row - p.dilation, 0), r1 = min(row + p.dilation, p.gh - 1);
    const int c0 = max(col - p.dilation, 0), c1 = min(col + p.dilation, p.gw - 1);
    for (int r = r0; r <= r1; ++r)
      for (int c = c0; c <= c1; ++c) keep[t * tpf + r * p.gw + c] = 1;
  }
  __syncthreads();
  const int count = compact_flags(keep, n, wout, sums);
  if (threadIdx.x == 0) write_cnt[s] = count;

  // 3. encode bucket: the first configured width that holds the write mask
  int target = count;
  if (count < n && p.bucket_multiple > 0) {
    const int b = p.bucket_multiple;
    const long long t = count <= b ? b : (long long)((count + b - 1) / b) * b;
    target = t >= n ? n : (int)t;
  } else if (count < n) {
    for (int w = 0; w < p.n_widths; ++w)
      if (p.widths[w] >= count) {
        target = p.widths[w];
        break;
      }
  }
  if (target <= count) {
    compact_flags(keep, n, eout, sums);  // the write mask again
    if (threadIdx.x == 0) enc_cnt[s] = count;
    return;
  }
  if (target >= n) {
    write_all(n, eout);
    if (threadIdx.x == 0) enc_cnt[s] = n;
    return;
  }
  // padded_to_len(target): evenly spaced candidates (i (n - 1) + target / 2) / target in i
  // order, the first `need` of them not yet kept; then the lowest tokens still missing.
  const int need = target - count;
  {
    const int per = (target + blockDim.x - 1) / blockDim.x;
    const int b = min(target, (int)threadIdx.x * per), e = min(target, b + per);
    int local = 0;
    for (int i = b; i < e; ++i) {
      const int c = (int)(((long long)i * (n - 1) + target / 2) / target);
      local += keep[c] == 0;
    }
    int total;
    int rank = viewer_scan(local, sums, &total);
    for (int i = b; i < e && rank < need; ++i) {
      const int c = (int)(((long long)i * (n - 1) + target / 2) / target);
      if (keep[c] == 0) {
        keep[c] = 2;  // candidates are distinct, so marking does not change another's test
        ++rank;
      }
    }
    if (threadIdx.x == 0) taken_sh = min(total, need);
  }
  __syncthreads();
  const int need2 = need - taken_sh;
  if (need2 > 0) {
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int b = min(n, (int)threadIdx.x * per), e = min(n, b + per);
    int local = 0;
    for (int i = b; i < e; ++i) local += keep[i] == 0;
    int total;
    int rank = viewer_scan(local, sums, &total);
    __syncthreads();
    for (int i = b; i < e && rank < need2; ++i)
      if (keep[i] == 0) {
        keep[i] = 3;
        ++rank;
      }
  }
  __syncthreads();
  const int enc = compact_flags(keep, n, eout, sums);
  if (threadIdx.x == 0) enc_cnt[s] = enc;
}

bjf_status viewer_params(const int64_t* grid, const bjf_viewer_mask_policy* policy, ViewerParams& p) {
  if (!grid || grid[0] <= 0 || grid[1] <= 0 || grid[2] <= 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must be non-empty");
  if (!policy) return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask policy must not be null");
  const int64_t n = grid[0] * grid[1] * grid[2];
  if (n > kMaxViewerTokens) return fail(BJF_ERR_UNSUPPORTED, "viewer masks support grids up to 32768 tokens");
  if (policy->dilation < 0) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff dilation must be non-negative");
  if (policy->bucket_density_count < 0 || policy->bucket_density_count > kMaxBucketWidths)
    return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask policy holds 0..32 bucket densities");
  p.n = (int)n;
  p.gh = (int)grid[1];
  p.gw = (int)grid[2];
  float d = policy->dense_fallback_density;
  d = d < 0.0f ? 0.0f : (d > 1.0f ? 1.0f : d);
  // (grid.len() as f32 * density).ceil() as usize (src/viewer.rs:787); a NaN density casts to 0
  p.fallback_tokens = std::isnan(d) ? 0 : (int)std::ceil((float)n * d);
  p.dilation = (int)std::min<int64_t>(policy->dilation, 1 << 20);
  p.bucket_multiple = 0;
  p.n_widths = 0;
  p.force_dense = 0;
  p.sample_scores = nullptr;
  // bucket_sparse_mask_with_config (src/viewer.rs:927-944) pads only grids of 256 tokens or more
  if (!policy->bucketed_encode || n < 256) return BJF_OK;
  if (policy->bucket_density_count == 0) {
    // the legacy fixed-width step (:893-901); bucket_tokens <= 1 leaves the single width n
    if (policy->bucket_tokens > 1) {
      p.bucket_multiple = (int)std::min<int64_t>(policy->bucket_tokens, std::max<int64_t>(n / 4, 1));
      return BJF_OK;
    }
  } else {
    // density_tokens(len, density, Ceil, 0.0) of every finite positive density (:902-916, 739-752)
    for (int i = 0; i < policy->bucket_density_count; ++i) {
      float b = policy->bucket_densities[i];
      if (!std::isfinite(b) || !(b > 0.0f)) continue;
      b = b > 1.0f ? 1.0f : b;
      const int64_t t = (int64_t)std::ceil((float)n * b);
      p.widths[p.n_widths++] = (int)std::min<int64_t>(std::max<int64_t>(t, 1), n);
    }
  }
  p.widths[p.n_widths++] = (int)n;
  std::sort(p.widths, p.widths + p.n_widths);
  p.n_widths = (int)(std::unique(p.widths, p.widths + p.n_widths) - p.widths);
  return BJF_OK;
}

bjf_status launch_viewer_masks(const int32_t* direct_idx, const int32_t* direct_cnt, int64_t streams,
                               const ViewerParams& p, int32_t* write_idx, int32_t* write_cnt, int32_t* enc_idx,
                               int32_t* enc_cnt, cudaStream_t st) {
  const size_t smem = (size_t)p.n;
  cudaError_t e = cudaSuccess;
  if (smem > 48 * 1024)
    e = cudaFuncSetAttribute(viewer_mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "viewer mask attribute");
  viewer_mask_kernel<<<(unsigned)streams, kViewerThreads, smem, st>>>(direct_idx, direct_cnt, p, write_idx, write_cnt,
                                                                      enc_idx, enc_cnt);
  return check_launch("viewer mask launch");
}

}  // namespace
}  // namespace bjf

using namespace bjf;

extern "C" bjf_status bjf_viewer_patch_diff_masks(const int32_t* direct_indices, const int32_t* direct_counts,
                                                  int64_t streams, const int64_t grid[3],
                                                  const bjf_viewer_mask_policy* policy, int32_t* write_indices,
                                                  int32_t* write_counts, int32_t* encode_indices,
                                                  int32_t* encode_counts, bjf_stream_t stream) {
  if (streams <= 0 || streams > (int64_t(1) << 31) - 1) return fail(BJF_ERR_INVALID_ARGUMENT, "stream count must be positive");
  if (!direct_indices || !direct_counts || !write_indices || !write_counts || !encode_indices || !encode_counts)
    return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask buffers must not be null");
  ViewerParams p{};
  const bjf_status rc = viewer_params(grid, policy, p);
  if (rc) return rc;
  return launch_viewer_masks(direct_indices, direct_counts, streams, p, write_indices, write_counts, encode_indices,
                             encode_counts, as_cuda(stream));
}

extern "C" bjf_status bjf_viewer_patch_diff_masks_from_scores(const float* scores, int64_t streams,
                                                              const int64_t grid[3],
                                                              const bjf_patch_diff_config* config,
                                                              const bjf_viewer_mask_policy* policy,
                                                              int32_t* write_indices, int32_t* write_counts,
                                                              int32_t* encode_indices, int32_t* encode_counts,
                                                              bjf_stream_t stream) {
  if (!config) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff config must not be null");
  if (!grid || grid[0] <= 0 || grid[1] <= 0 || grid[2] <= 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must be non-empty");
  if (streams <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "stream count must be positive");
  if (!scores || !write_indices || !write_counts || !encode_indices || !encode_counts)
    return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask buffers must not be null");
  // patch_diff_base_mask_from_scores (src/viewer.rs:819-829): the threshold selection
  // without dilation, then the policy (which dilates the direct mask)
  if (!policy) return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask policy must not be null");
  bjf_patch_diff_config direct = *config;
  direct.dilation = 0;
  bjf_viewer_mask_policy dilated = *policy;  // the dilation is the sparsity config's (:828)
  dilated.dilation = config->dilation;
  SelectParams sp;
  bjf_status rc = resolve_select(&direct, grid, sp);
  if (rc) return rc;
  ViewerParams vp{};
  rc = viewer_params(grid, &dilated, vp);
  if (rc) return rc;
  cudaStream_t st = as_cuda(stream);
  rc = launch_select(scores, streams, sp, write_indices, write_counts, st);
  if (rc) return rc;
  return launch_viewer_masks(write_indices, write_counts, streams, vp, write_indices, write_counts, encode_indices,
                             encode_counts, st);
}

namespace {
size_t rgba_masks_scores_offset(int64_t streams, const int64_t grid[3]) {
  return (bjf_rgba_patch_diff_workspace_bytes(streams, grid) + 255) & ~size_t(255);
}
}  // namespace

extern "C" size_t bjf_viewer_rgba_masks_workspace_bytes(int64_t streams, const int64_t grid[3]) {
  if (!grid || grid[0] != 1 || grid[1] <= 0 || grid[2] <= 0 || grid[1] * grid[2] > kMaxViewerTokens) return 0;
  if (bjf_rgba_patch_diff_workspace_bytes(streams, grid) == 0) return 0;
  return rgba_masks_scores_offset(streams, grid) + sizeof(float) * (size_t)streams * (size_t)(grid[1] * grid[2]);
}

extern "C" bjf_status bjf_viewer_patch_diff_masks_from_rgba(
    const uint8_t* prev, const uint8_t* current, int64_t streams, int64_t width, int64_t height, int64_t patch_size,
    const int64_t grid[3], const bjf_patch_diff_config* config, const bjf_viewer_mask_policy* policy,
    int32_t* write_indices, int32_t* write_counts, int32_t* encode_indices, int32_t* encode_counts,
    bjf_rgba_frame_stats* stats_out, void* workspace, size_t workspace_bytes, bjf_stream_t stream) {
  if (!config) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff config must not be null");
  if (!policy) return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask policy must not be null");
  if (!grid) return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must not be null");
  // patch_diff_mask_from_rgba (crates/bevy_jepa/src/mask.rs:126-149)
  if (grid[0] != 1) return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff mask expects a single-frame token grid");
  if (patch_size <= 0 || height != grid[1] * patch_size || width != grid[2] * patch_size)
    return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff frame size must match the V-JEPA patch grid");
  if (!write_indices || !write_counts || !encode_indices || !encode_counts)
    return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask buffers must not be null");
  const size_t need = bjf_viewer_rgba_masks_workspace_bytes(streams, grid);
  if (need == 0) return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA viewer masks support 1..65535 streams and grids up to 32768 tokens");
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "RGBA viewer mask workspace must be 256-byte aligned and hold " + std::to_string(need) + " bytes");
  bjf_patch_diff_config direct = *config;
  direct.dilation = 0;
  SelectParams sp;
  bjf_status rc = resolve_select(&direct, grid, sp);
  if (rc) return rc;
  bjf_viewer_mask_policy dilated = *policy;
  dilated.dilation = config->dilation;
  ViewerParams vp{};
  rc = viewer_params(grid, &dilated, vp);
  if (rc) return rc;
  const int64_t n = grid[1] * grid[2];
  // patch_diff_sparsity_config's dense shortcuts (crates/bevy_jepa/src/mask.rs:151-168)
  const bool full_context = config->allow_full_context != 0 && config->context_tokens >= n;
  vp.force_dense = config->threshold <= 0.0f && full_context;
  float fb = policy->dense_fallback_density;
  fb = fb < 0.0f ? 0.0f : (fb > 1.0f ? 1.0f : fb);
  float* scores = reinterpret_cast<float*>(static_cast<char*>(workspace) + rgba_masks_scores_offset(streams, grid));
  if (!(fb >= 1.0f) && config->threshold > 0.0f && full_context) {  // a NaN density takes the path
    // stride = ceil(sqrt(len / 64)) in f32, the sampled grid its multiples (src/viewer.rs:1178-1193)
    const int stride = std::max(1, (int)std::ceil(std::sqrt((float)n / 64.0f)));
    vp.sample_scores = scores;
    vp.sample_threshold = config->threshold;
    vp.sample_stride = stride;
    vp.sample_rows = (int)((grid[1] + stride - 1) / stride);
    vp.sample_cols = (int)((grid[2] + stride - 1) / stride);
    vp.sample_required = std::isnan(fb) ? 0 : (int)std::ceil((float)(vp.sample_rows * vp.sample_cols) * fb);
  }
  cudaStream_t st = as_cuda(stream);
  rc = bjf_rgba_patch_diff_scores(prev, current, streams, width, height, patch_size, grid, scores, stats_out,
                                  workspace, workspace_bytes, stream);
  if (rc) return rc;
  rc = launch_select(scores, streams, sp, write_indices, write_counts, st);
  if (rc) return rc;
  return launch_viewer_masks(write_indices, write_counts, streams, vp, write_indices, write_counts, encode_indices,
                             encode_counts, st);
}
