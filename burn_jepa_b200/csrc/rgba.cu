// rgba.cu -- the live viewer's patch-diff scorer for RGBA u8 camera frames
// (burn_jepa src/viewer.rs:1069-1270: rgba_patch_diff_frame_stats, patch_diff_scores_from_rgba,
// rgba_patch_diff_pixel_score), batched over S independent streams.
//
//   1. lighting means      per stream: mean RGB delta, mean luma delta, mean per-pixel |delta|
//   2. lighting residual   mean per-pixel |delta - mean delta|; compensate the global lighting
//                          shift when raw > 1e-4 and residual <= 0.35 raw
//   3. scores              per patch: mean over its pixels of
//                          max(|rgb delta| / 3, |luma delta|, relative luma / 4, chroma delta / 2)
//                          with the global shift removed when compensating
//
// Each pass is a grid over (pixel ranges, streams); the frame-wide sums are reduced in a fixed
// order from per-block partials (f64) kept in the caller's workspace, so results do not
// depend on timing and no counters need resetting.  Every per-pixel operation is rounded as
// the reference's f32 code does (no contraction); only the summation order of the means and
// patch sums differs from the reference's sequential loops.
#include <string>

#include "../../include/bjf.h"
#include "common.cuh"
#include "runtime.hpp"
#include "status.hpp"

namespace bjf {
namespace {

constexpr int kRgbaThreads = 256;
constexpr int kStatBlocks = 64;     // partials per stream and pass
constexpr int kMeanParts = 5;       // sum dR, dG, dB, d luma, per-pixel mean |delta|

struct Rgb {
  float r, g, b;
};

__device__ __forceinline__ Rgb load_rgb(const uint8_t* px) {
  // rgba[offset + c] as f32 / 255.0 (src/viewer.rs:1246-1252)
  const uchar4 v = *reinterpret_cast<const uchar4*>(px);
  return Rgb{__fdiv_rn((float)v.x, 255.0f), __fdiv_rn((float)v.y, 255.0f), __fdiv_rn((float)v.z, 255.0f)};
}

// rgb[0] * 0.2126 + rgb[1] * 0.7152 + rgb[2] * 0.0722 (:1254-1256)
__device__ __forceinline__ float luma(Rgb c) {
  return __fadd_rn(__fadd_rn(__fmul_rn(c.r, 0.2126f), __fmul_rn(c.g, 0.7152f)), __fmul_rn(c.b, 0.0722f));
}

// (sum of |chroma delta|) / 3 with chroma = rgb / max(r + g + b, 0.10) (:1258-1270)
__device__ __forceinline__ float chroma_diff(Rgb p, Rgb c) {
  const float dp = fmaxf(__fadd_rn(__fadd_rn(p.r, p.g), p.b), 0.10f);
  const float dc = fmaxf(__fadd_rn(__fadd_rn(c.r, c.g), c.b), 0.10f);
  const float a = fabsf(__fsub_rn(__fdiv_rn(c.r, dc), __fdiv_rn(p.r, dp)));
  const float b = fabsf(__fsub_rn(__fdiv_rn(c.g, dc), __fdiv_rn(p.g, dp)));
  const float d = fabsf(__fsub_rn(__fdiv_rn(c.b, dc), __fdiv_rn(p.b, dp)));
  return __fdiv_rn(__fadd_rn(__fadd_rn(a, b), d), 3.0f);
}

// Block-wide sum of a double (all threads get the result).
__device__ __forceinline__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < kRgbaThreads / 32; ++w) t += red[w];  // fixed order
  return t;
}

// Pass 1: per block, sums over its pixel range of the channel deltas, the luma delta and the
// per-pixel mean |delta| (src/viewer.rs:1079-1100).
__global__ void __launch_bounds__(kRgbaThreads)
    rgba_means_kernel(const uint8_t* __restrict__ prev, const uint8_t* __restrict__ cur, long long pixels,
                      double* __restrict__ partials) {
  __shared__ double red[kRgbaThreads / 32];
  const long long s = blockIdx.y;
  const uint8_t* p0 = prev + s * pixels * 4;
  const uint8_t* c0 = cur + s * pixels * 4;
  double acc[kMeanParts] = {0, 0, 0, 0, 0};
  for (long long i = (long long)blockIdx.x * kRgbaThreads + threadIdx.x; i < pixels;
       i += (long long)kStatBlocks * kRgbaThreads) {
    const Rgb a = load_rgb(p0 + i * 4), b = load_rgb(c0 + i * 4);
    const float dr = __fsub_rn(b.r, a.r), dg = __fsub_rn(b.g, a.g), db = __fsub_rn(b.b, a.b);
    acc[0] += dr;
    acc[1] += dg;
    acc[2] += db;
    acc[3] += __fsub_rn(luma(b), luma(a));
    acc[4] += __fdiv_rn(__fadd_rn(__fadd_rn(fabsf(dr), fabsf(dg)), fabsf(db)), 3.0f);
  }
  double* out = partials + (s * kStatBlocks + blockIdx.x) * kMeanParts;
#pragma unroll
  for (int k = 0; k < kMeanParts; ++k) {
    const double t = block_sum(acc[k], red);
    if (threadIdx.x == 0) out[k] = t;
  }
}

struct Means {
  float d[3];
  float luma;
  float raw;
  float residual;  // pass 3 only
};

// The stream's frame means from the block partials: thread k < kMeanParts (+1 for the
// residual) sums component k in a fixed order; the block shares them through `sh`.
// The reference divides its f32 sums by `pixels as f32` (:1097-1100, :1114).
__device__ __forceinline__ Means load_means(const double* mean_partials, const double* residual_partials,
                                            long long s, long long pixels, Means* sh) {
  const int k = threadIdx.x;
  const float n = (float)pixels;
  if (k < kMeanParts) {
    const double* part = mean_partials + s * kStatBlocks * kMeanParts;
    double t = 0.0;
    for (int i = 0; i < kStatBlocks; ++i) t += part[i * kMeanParts + k];
    const float v = __fdiv_rn((float)t, n);
    if (k < 3) sh->d[k] = v; else if (k == 3) sh->luma = v; else sh->raw = v;
  } else if (k == kMeanParts && residual_partials) {
    double t = 0.0;
    for (int i = 0; i < kStatBlocks; ++i) t += residual_partials[s * kStatBlocks + i];
    sh->residual = __fdiv_rn((float)t, n);
  }
  __syncthreads();
  return *sh;
}

// Pass 2: per block, sum of the per-pixel mean |delta - mean delta| (:1102-1113).
__global__ void __launch_bounds__(kRgbaThreads)
    rgba_residual_kernel(const uint8_t* __restrict__ prev, const uint8_t* __restrict__ cur, long long pixels,
                         const double* __restrict__ mean_partials, double* __restrict__ residual_partials) {
  __shared__ double red[kRgbaThreads / 32];
  __shared__ Means sh;
  const long long s = blockIdx.y;
  const Means m = load_means(mean_partials, nullptr, s, pixels, &sh);
  const uint8_t* p0 = prev + s * pixels * 4;
  const uint8_t* c0 = cur + s * pixels * 4;
  double acc = 0.0;
  for (long long i = (long long)blockIdx.x * kRgbaThreads + threadIdx.x; i < pixels;
       i += (long long)kStatBlocks * kRgbaThreads) {
    const Rgb a = load_rgb(p0 + i * 4), b = load_rgb(c0 + i * 4);
    const float er = fabsf(__fsub_rn(__fsub_rn(b.r, a.r), m.d[0]));
    const float eg = fabsf(__fsub_rn(__fsub_rn(b.g, a.g), m.d[1]));
    const float eb = fabsf(__fsub_rn(__fsub_rn(b.b, a.b), m.d[2]));
    acc += __fdiv_rn(__fadd_rn(__fadd_rn(er, eg), eb), 3.0f);
  }
  const double t = block_sum(acc, red);
  if (threadIdx.x == 0) residual_partials[s * kStatBlocks + blockIdx.x] = t;
}

// Pass 3: one warp per patch (:1199-1244).  Lane l takes pixels l, l + 32, ... of the patch
// in row-major order; the patch sum is reduced across the warp.
__global__ void __launch_bounds__(kRgbaThreads)
    rgba_scores_kernel(const uint8_t* __restrict__ prev, const uint8_t* __restrict__ cur, long long pixels,
                       int width, int patch, int gh, int gw, const double* __restrict__ mean_partials,
                       const double* __restrict__ residual_partials, float* __restrict__ scores,
                       bjf_rgba_frame_stats* __restrict__ stats_out) {
  __shared__ Means sh;
  const long long s = blockIdx.y;
  const Means m = load_means(mean_partials, residual_partials, s, pixels, &sh);
  const float residual = m.residual;
  const bool comp = m.raw > 1.0e-4f && residual <= __fmul_rn(m.raw, 0.35f);
  if (stats_out && blockIdx.x == 0 && threadIdx.x == 0) {
    bjf_rgba_frame_stats st;
    st.channel_delta[0] = m.d[0];
    st.channel_delta[1] = m.d[1];
    st.channel_delta[2] = m.d[2];
    st.luma_delta = m.luma;
    st.compensate_global_lighting = comp ? 1 : 0;
    st.raw_abs = m.raw;
    st.residual_abs = residual;
    stats_out[s] = st;
  }
  const int lane = threadIdx.x & 31;
  const long long patch_id = (long long)blockIdx.x * (kRgbaThreads / 32) + (threadIdx.x >> 5);
  const long long n_patches = (long long)gh * gw;
  if (patch_id >= n_patches) return;
  const int row = (int)(patch_id / gw), col = (int)(patch_id % gw);
  const uint8_t* p0 = prev + s * pixels * 4;
  const uint8_t* c0 = cur + s * pixels * 4;
  float acc = 0.0f;
  const int area = patch * patch;
  for (int k = lane; k < area; k += 32) {
    const int y = row * patch + k / patch, x = col * patch + k % patch;
    const long long off = ((long long)y * width + x) * 4;
    const Rgb a = load_rgb(p0 + off), b = load_rgb(c0 + off);
    float dr = __fsub_rn(b.r, a.r), dg = __fsub_rn(b.g, a.g), db = __fsub_rn(b.b, a.b);
    if (comp) {
      dr = __fsub_rn(dr, m.d[0]);
      dg = __fsub_rn(dg, m.d[1]);
      db = __fsub_rn(db, m.d[2]);
    }
    const float rgb_abs = __fdiv_rn(__fadd_rn(__fadd_rn(fabsf(dr), fabsf(dg)), fabsf(db)), 3.0f);
    const float pl = luma(a), cl = luma(b);
    float ld = __fsub_rn(cl, pl);
    if (comp) ld = __fsub_rn(ld, m.luma);
    const float luma_abs = fabsf(ld);
    const float rel = __fmul_rn(fminf(__fdiv_rn(luma_abs, fmaxf(fmaxf(pl, cl), 0.10f)), 1.0f), 0.25f);
    const float chroma = __fmul_rn(chroma_diff(a, b), 0.5f);
    acc += fmaxf(fmaxf(fmaxf(rgb_abs, luma_abs), rel), chroma);
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) scores[s * n_patches + patch_id] = __fdiv_rn(acc, (float)area);
}

size_t workspace_layout(int64_t streams, size_t* residual_off) {
  const size_t means = sizeof(double) * (size_t)streams * kStatBlocks * kMeanParts;
  *residual_off = (means + 255) & ~size_t(255);
  return *residual_off + sizeof(double) * (size_t)streams * kStatBlocks;
}

}  // namespace
}  // namespace bjf

using namespace bjf;

extern "C" size_t bjf_rgba_patch_diff_workspace_bytes(int64_t streams) {
  if (streams <= 0 || streams > 65535) return 0;
  size_t r;
  return workspace_layout(streams, &r);
}

extern "C" bjf_status bjf_rgba_patch_diff_scores(const uint8_t* prev, const uint8_t* current, int64_t streams,
                                                 int64_t width, int64_t height, int64_t patch_size,
                                                 const int64_t grid[3], float* scores,
                                                 bjf_rgba_frame_stats* stats_out, void* workspace,
                                                 size_t workspace_bytes, bjf_stream_t stream) {
  if (!grid) return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must not be null");
  // checks and messages of patch_diff_scores_from_rgba (src/viewer.rs:1133-1146)
  if (grid[0] != 1) return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff expects a single-frame grid");
  if (patch_size <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff patch size must be nonzero");
  if (grid[1] <= 0 || grid[2] <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must be non-empty");
  if (width != grid[2] * patch_size) return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff width must match the token grid");
  if (height < grid[1] * patch_size)
    return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff buffers are smaller than the token grid");
  if (streams <= 0 || streams > 65535) return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff supports 1..65535 streams");
  if (width > (1 << 20) || height > (1 << 20) || patch_size > 1024)
    return fail(BJF_ERR_UNSUPPORTED, "RGBA patch-diff frame exceeds the supported size");
  if (!prev || !current || !scores || !workspace)
    return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA patch-diff buffers must not be null");
  if ((reinterpret_cast<uintptr_t>(prev) | reinterpret_cast<uintptr_t>(current)) & 3)
    return fail(BJF_ERR_INVALID_ARGUMENT, "RGBA frames must be 4-byte aligned");
  size_t roff;
  const size_t need = workspace_layout(streams, &roff);
  if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "RGBA patch-diff workspace must be 256-byte aligned and hold " + std::to_string(need) + " bytes");
  const long long pixels = (long long)width * height;
  double* means = static_cast<double*>(workspace);
  double* resid = reinterpret_cast<double*>(static_cast<char*>(workspace) + roff);
  cudaStream_t st = as_cuda(stream);
  const dim3 sgrid(kStatBlocks, (unsigned)streams);
  rgba_means_kernel<<<sgrid, kRgbaThreads, 0, st>>>(prev, current, pixels, means);
  bjf_status rc = check_launch("RGBA lighting means launch");
  if (rc) return rc;
  rgba_residual_kernel<<<sgrid, kRgbaThreads, 0, st>>>(prev, current, pixels, means, resid);
  rc = check_launch("RGBA lighting residual launch");
  if (rc) return rc;
  const long long patches = grid[1] * grid[2];
  const dim3 pgrid((unsigned)ceil_div(patches, kRgbaThreads / 32), (unsigned)streams);
  rgba_scores_kernel<<<pgrid, kRgbaThreads, 0, st>>>(prev, current, pixels, (int)width, (int)patch_size,
                                                     (int)grid[1], (int)grid[2], means, resid, scores, stats_out);
  return check_launch("RGBA patch-diff scores launch");
}
