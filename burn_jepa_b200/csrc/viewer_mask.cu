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
// PatchDiffRefreshState (src/viewer.rs:275-528) of the launch's streams, in device memory, and
// the PatchDiffRefreshConfig (:186-270) values the kernel reads, resolved on the host.
struct RefreshParams {
  float* residual;                  // [S, n] subthreshold residuals; null: no refresh state
  uint32_t* age;                    // [S, n] frames since the token was last written
  unsigned long long* frame_index;  // [S]
  const float* scores;              // [S, n] the frame's patch-diff scores
  int augment;                      // can_add_tokens (:258-269)
  float threshold;                  // the sparsity threshold, compared as given (:515)
  float norm_threshold;             // threshold.max(1e-6) (:512)
  float decay, gain, trigger;       // decay.clamp(0, 1), gain.max(0), trigger.max(1e-6)
  int max_context;                  // context_tokens.max(1).min(n) (:388)
  int max_extra;                    // density_tokens(n, max_extra_density, Floor, 0)
  int stage_tokens[3];              // subthreshold / age / blue-noise budgets before `remaining`; 0: off
  uint32_t interval;                // age_refresh_interval_frames.min(u32::MAX)
  unsigned long long seed;          // blue_noise_seed
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

// ---- refresh stage (PatchDiffRefreshState::augment_mask and its bookkeeping) ----------------

__device__ __forceinline__ uint32_t sat_inc32(uint32_t v) { return v == 0xffffffffu ? v : v + 1; }

// mix64 (src/viewer.rs:530-536): the splitmix64 output function.
__device__ __forceinline__ unsigned long long refresh_mix64(unsigned long long v) {
  v ^= v >> 30;
  v *= 0xbf58476d1ce4e5b9ull;
  v ^= v >> 27;
  v *= 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

// A candidate's place in add_ranked_candidates' order (:505-511) as one 128-bit unsigned key,
// smaller first: priority descending, then the refresh rank, then the token index.  Every key is
// distinct because the index is in it.  -0.0 and 0.0 compare equal under partial_cmp, so both
// map to 0.0's key; no priority here is NaN (residual >= trigger, age as f32, or 0.0).
struct RefreshKey {
  unsigned long long hi, lo;
};
__device__ __forceinline__ RefreshKey refresh_key(float priority, unsigned long long rank, int index) {
  uint32_t b = __float_as_uint(priority == 0.0f ? 0.0f : priority);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // unsigned order = float order
  return {((unsigned long long)~b << 32) | (rank >> 32), (rank << 32) | (uint32_t)index};
}
__device__ __forceinline__ int key_digit(const RefreshKey& k, int d) {  // byte d, most significant first
  return d < 8 ? (int)((k.hi >> (56 - 8 * d)) & 0xff) : (int)((k.lo >> (56 - 8 * (d - 8))) & 0xff);
}
__device__ __forceinline__ bool key_prefix_is(const RefreshKey& k, int d, unsigned long long ph,
                                              unsigned long long pl) {  // top 8 d bits equal
  const unsigned long long mh = d == 0 ? 0ull : (d >= 8 ? ~0ull : ~0ull << (64 - 8 * d));
  const unsigned long long ml = d <= 8 ? 0ull : ~0ull << (64 - 8 * (d - 8));
  return (k.hi & mh) == ph && (k.lo & ml) == pl;
}

// Whether unselected token i is a candidate of `stage` (0 subthreshold, 1 age, 2 blue noise,
// the closures of :409-459) and its key.  Ages are read before this frame's increment.
__device__ __forceinline__ bool refresh_candidate(const RefreshParams& r, int stage, const float* res,
                                                  const uint32_t* age, int gw, unsigned long long frame, int i,
                                                  RefreshKey& key) {
  float priority = 0.0f;
  if (stage == 0) {
    priority = res[i];
    if (!(priority >= r.trigger)) return false;
  } else if (stage == 1) {
    const uint32_t a = sat_inc32(age[i]);
    if (a < r.interval) return false;
    priority = __uint2float_rn(a);  // `age as f32`
  }
  // refresh_rank (:520-528): the row and column of the flat index over the grid's width
  const unsigned long long row = (unsigned)i / (unsigned)gw, col = (unsigned)i % (unsigned)gw;
  const unsigned long long rank = refresh_mix64(r.seed ^ (row * 0x9e3779b97f4a7c15ull) ^
                                                (col * 0xbf58476d1ce4e5b9ull) ^ (frame * 0x94d049bb133111ebull));
  key = refresh_key(priority, rank, i);
  return true;
}

// add_ranked_candidates (:481-518): marks in keep (as 1) the `budget` smallest keys among the
// stage's candidates that keep does not hold, and returns how many it marked.  With more
// candidates than budget, a most-significant-byte-first radix select over the 128-bit key
// finds them: each pass takes every candidate below the byte holding the budget-th key, and
// stops when that byte's candidates are exactly the ones still needed.  Each token is owned by
// one thread (i = threadIdx.x + k blockDim.x) in every loop.
__device__ int refresh_add_ranked(const RefreshParams& r, int stage, int budget, int n, int gw, long long s,
                                  unsigned long long frame, unsigned char* keep, int* sums, int* hist, int* pick) {
  const float* res = r.residual + s * n;
  const uint32_t* age = r.age + s * n;
  RefreshKey k;
  int local = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    local += keep[i] == 0 && refresh_candidate(r, stage, res, age, gw, frame, i, k);
  int total;
  viewer_scan(local, sums, &total);
  if (total <= budget) {
    for (int i = threadIdx.x; i < n; i += blockDim.x)
      if (keep[i] == 0 && refresh_candidate(r, stage, res, age, gw, frame, i, k)) keep[i] = 1;
    __syncthreads();
    return total;
  }
  int need = budget;
  unsigned long long ph = 0, pl = 0;
  for (int d = 0; d < 16; ++d) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x)
      if (keep[i] == 0 && refresh_candidate(r, stage, res, age, gw, frame, i, k) && key_prefix_is(k, d, ph, pl))
        atomicAdd(&hist[key_digit(k, d)], 1);
    __syncthreads();
    if (threadIdx.x < 32) {  // the byte b with (candidates below b) < need <= (candidates up to b)
      const int lane = threadIdx.x;
      int c = 0;
      for (int j = 0; j < 8; ++j) c += hist[lane * 8 + j];
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      int before = inc - c;
      if (before < need && need <= inc) {
        for (int j = 0; j < 8; ++j) {
          const int h = hist[lane * 8 + j];
          if (before + h >= need) {
            pick[0] = lane * 8 + j;
            pick[1] = before;
            pick[2] = h;
            break;
          }
          before += h;
        }
      }
    }
    __syncthreads();
    const int b = pick[0];
    need -= pick[1];
    const bool whole = pick[2] == need;  // the byte's candidates are all still needed
    for (int i = threadIdx.x; i < n; i += blockDim.x)
      if (keep[i] == 0 && refresh_candidate(r, stage, res, age, gw, frame, i, k) && key_prefix_is(k, d, ph, pl)) {
        const int dg = key_digit(k, d);
        if (dg < b || (whole && dg == b)) keep[i] = 1;
      }
    __syncthreads();
    if (whole) break;  // reached by d = 15 at the latest: keys are distinct
    if (d < 8)
      ph |= (unsigned long long)b << (56 - 8 * d);
    else
      pl |= (unsigned long long)b << (56 - 8 * (d - 8));
  }
  return budget;
}

// One frame of the stream's refresh state around its write mask, held in keep as nonzero flags
// (count of n set): augment_mask (:377-458) when the config can add tokens and the mask is not
// every token, then begin_frame's increments and reset_selected over the final write mask
// (:352-375).  Residuals are updated before any ranking reads them; ages are read before the
// increment and written once at the end.
__device__ void refresh_stream(const RefreshParams& r, int n, int gw, long long s, int count, unsigned char* keep,
                               int* sums, int* hist, int* pick) {
  const unsigned long long f0 = r.frame_index[s];
  const unsigned long long frame = f0 == ~0ull ? f0 : f0 + 1;
  float* res = r.residual + s * n;
  uint32_t* age = r.age + s * n;
  if (r.augment && count < n) {
    int remaining = max(r.max_context - count, 0);
    remaining = min(remaining, r.max_extra);
    // update_subthreshold_residual (:461-479) against the base mask; Rust evaluates r * decay
    // and normalized * gain as separate f32 products and adds them, hence no contraction
    const float* scores = r.scores + s * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float sc = scores[i];
      float v = 0.0f;
      if (keep[i] == 0 && !(sc >= r.threshold)) {
        float norm = __fdiv_rn(sc, r.norm_threshold);
        norm = norm < 0.0f ? 0.0f : (norm > 1.0f ? 1.0f : norm);  // f32::clamp keeps a NaN
        v = __fadd_rn(__fmul_rn(res[i], r.decay), __fmul_rn(norm, r.gain));
      }
      res[i] = v;
    }
    __syncthreads();
    for (int stage = 0; stage < 3 && remaining > 0; ++stage) {
      if (r.stage_tokens[stage] == 0) continue;
      const int budget = min(remaining, r.stage_tokens[stage]);
      remaining -= refresh_add_ranked(r, stage, budget, n, gw, s, frame, keep, sums, hist, pick);
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (keep[i]) {
      res[i] = 0.0f;
      age[i] = 0;
    } else {
      age[i] = sat_inc32(age[i]);
    }
  }
  __syncthreads();  // every thread has read the old frame index
  if (threadIdx.x == 0) r.frame_index[s] = frame;
}

// observe_write_mask (:309-313) of a write mask that is every token.
__device__ __forceinline__ void refresh_all_written(const RefreshParams& r, int n, long long s) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    r.residual[s * n + i] = 0.0f;
    r.age[s * n + i] = 0;
  }
  if (threadIdx.x == 0) {
    const unsigned long long f0 = r.frame_index[s];
    r.frame_index[s] = f0 == ~0ull ? f0 : f0 + 1;
  }
}

// direct_idx / direct_cnt may alias write_idx / write_cnt: every direct index and count is
// read before the write mask is stored.
__global__ void __launch_bounds__(kViewerThreads)
    viewer_mask_kernel(const int32_t* direct_idx, const int32_t* direct_cnt, ViewerParams p, RefreshParams r,
                       int32_t* write_idx, int32_t* write_cnt, int32_t* __restrict__ enc_idx,
                       int32_t* __restrict__ enc_cnt) {
  extern __shared__ unsigned char keep[];
  __shared__ int sums[33];
  __shared__ int taken_sh;
  __shared__ int hist[256];
  __shared__ int pick[3];
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
    if (r.residual) refresh_all_written(r, n, s);
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
  if (r.residual) {
    // the refresh tokens join the write mask before the encode buckets (src/viewer.rs:343-346)
    int base = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) base += keep[i] != 0;
    viewer_scan(base, sums, &base);
    refresh_stream(r, n, p.gw, s, base, keep, sums, hist, pick);
  }
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
                               int32_t* enc_cnt, cudaStream_t st, const RefreshParams* refresh = nullptr) {
  const size_t smem = (size_t)p.n;
  cudaError_t e = cudaSuccess;
  if (smem > 48 * 1024 - 2048)  // the static arrays take the rest of the default 48 KB
    e = cudaFuncSetAttribute(viewer_mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "viewer mask attribute");
  RefreshParams r{};
  if (refresh) r = *refresh;
  viewer_mask_kernel<<<(unsigned)streams, kViewerThreads, smem, st>>>(direct_idx, direct_cnt, p, r, write_idx,
                                                                      write_cnt, enc_idx, enc_cnt);
  return check_launch("viewer mask launch");
}

// f32::clamp(lo, hi): a NaN stays NaN.
float rust_clamp(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// density_tokens(n, density, Floor, 0.0) (src/viewer.rs:739-752): f32 product, floor, a
// saturating `as usize`, then clamp(1, n).
int density_tokens_floor(int64_t n, float density) {
  const float x = std::floor((float)n * rust_clamp(density, 0.0f, 1.0f));
  const int64_t t = x > 0.0f ? (x >= (float)n ? n : (int64_t)x) : 0;  // NaN casts to 0
  return (int)std::min<int64_t>(std::max<int64_t>(t, 1), std::max<int64_t>(n, 1));
}

// The refresh state and config as the kernel reads them.  context_tokens is the sparsity
// config's (src/viewer.rs:388).
bjf_status refresh_params(const bjf_patch_diff_refresh_config* c, const bjf_patch_diff_refresh_state* state,
                          const float* scores, int64_t n, const bjf_patch_diff_config* sparsity, RefreshParams& r) {
  if (!c) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff refresh config must not be null");
  if (!state || !state->subthreshold_residual || !state->age_frames || !state->frame_index)
    return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff refresh state buffers must not be null");
  r = RefreshParams{};
  r.residual = state->subthreshold_residual;
  r.age = state->age_frames;
  r.frame_index = reinterpret_cast<unsigned long long*>(state->frame_index);
  r.scores = scores;
  const bool sub = c->subthreshold_enabled && c->subthreshold_max_density > 0.0f;
  const bool aged = c->age_refresh_enabled && c->age_refresh_interval_frames > 0 && c->age_refresh_max_density > 0.0f;
  const bool blue = c->blue_noise_enabled && c->blue_noise_refresh_density > 0.0f;
  // PatchDiffRefreshConfig::can_add_tokens (:258-269); without scores (the dense shortcuts of
  // the RGBA node) nothing is ranked
  r.augment = scores && c->enabled && c->max_extra_density > 0.0f && (sub || aged || blue);
  r.threshold = sparsity ? sparsity->threshold : 0.0f;
  r.norm_threshold = std::fmax(r.threshold, 1.0e-6f);  // f32::max returns the number for a NaN
  r.decay = rust_clamp(c->subthreshold_decay, 0.0f, 1.0f);
  r.gain = std::fmax(c->subthreshold_gain, 0.0f);
  r.trigger = std::fmax(c->subthreshold_trigger, 1.0e-6f);
  const int64_t ctx = sparsity ? sparsity->context_tokens : 1;
  r.max_context = (int)std::min<int64_t>(std::max<int64_t>(ctx, 1), n);
  r.max_extra = density_tokens_floor(n, c->max_extra_density);
  r.stage_tokens[0] = sub ? density_tokens_floor(n, c->subthreshold_max_density) : 0;
  r.stage_tokens[1] = aged ? density_tokens_floor(n, c->age_refresh_max_density) : 0;
  r.stage_tokens[2] = blue ? density_tokens_floor(n, c->blue_noise_refresh_density) : 0;
  r.interval = (uint32_t)std::min<uint64_t>(c->age_refresh_interval_frames, 0xffffffffull);
  r.seed = c->blue_noise_seed;
  return BJF_OK;
}

// observe_write_mask (src/viewer.rs:309-313) for one stream per CTA: every age advances, then
// the written tokens' residuals and ages return to zero.
__global__ void __launch_bounds__(kViewerThreads)
    refresh_observe_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ cnt, int n, RefreshParams r) {
  const long long s = blockIdx.x;
  for (int i = threadIdx.x; i < n; i += blockDim.x) r.age[s * n + i] = sat_inc32(r.age[s * n + i]);
  __syncthreads();  // the block's global writes are visible to it after the barrier
  const int m = min(max(cnt[s], 0), n);
  for (int j = threadIdx.x; j < m; j += blockDim.x) {
    const int i = idx[s * n + j];
    if (i < 0 || i >= n) continue;  // SparseTokenMask holds in-range indices; `get_mut` skips others
    r.residual[s * n + i] = 0.0f;
    r.age[s * n + i] = 0;
  }
  if (threadIdx.x == 0) {
    const unsigned long long f0 = r.frame_index[s];
    r.frame_index[s] = f0 == ~0ull ? f0 : f0 + 1;
  }
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

namespace {
bjf_status masks_from_scores(const float* scores, int64_t streams, const int64_t grid[3],
                             const bjf_patch_diff_config* config, const bjf_viewer_mask_policy* policy,
                             int32_t* write_indices, int32_t* write_counts, int32_t* encode_indices,
                             int32_t* encode_counts, bjf_stream_t stream,
                             const bjf_patch_diff_refresh_config* refresh,
                             const bjf_patch_diff_refresh_state* state) {
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
  RefreshParams rp{};
  if (state) {
    rc = refresh_params(refresh, state, scores, vp.n, config, rp);
    if (rc) return rc;
  }
  cudaStream_t st = as_cuda(stream);
  rc = launch_select(scores, streams, sp, write_indices, write_counts, st);
  if (rc) return rc;
  return launch_viewer_masks(write_indices, write_counts, streams, vp, write_indices, write_counts, encode_indices,
                             encode_counts, st, state ? &rp : nullptr);
}
}  // namespace

extern "C" bjf_status bjf_viewer_patch_diff_masks_from_scores(const float* scores, int64_t streams,
                                                              const int64_t grid[3],
                                                              const bjf_patch_diff_config* config,
                                                              const bjf_viewer_mask_policy* policy,
                                                              int32_t* write_indices, int32_t* write_counts,
                                                              int32_t* encode_indices, int32_t* encode_counts,
                                                              bjf_stream_t stream) {
  return masks_from_scores(scores, streams, grid, config, policy, write_indices, write_counts, encode_indices,
                           encode_counts, stream, nullptr, nullptr);
}

extern "C" bjf_status bjf_viewer_patch_diff_refresh_masks_from_scores(
    const float* scores, int64_t streams, const int64_t grid[3], const bjf_patch_diff_config* config,
    const bjf_viewer_mask_policy* policy, const bjf_patch_diff_refresh_config* refresh,
    const bjf_patch_diff_refresh_state* state, int32_t* write_indices, int32_t* write_counts,
    int32_t* encode_indices, int32_t* encode_counts, bjf_stream_t stream) {
  if (!state) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff refresh state buffers must not be null");
  return masks_from_scores(scores, streams, grid, config, policy, write_indices, write_counts, encode_indices,
                           encode_counts, stream, refresh, state);
}

extern "C" bjf_status bjf_viewer_patch_diff_refresh_observe(const int32_t* write_indices,
                                                            const int32_t* write_counts, int64_t streams,
                                                            const int64_t grid[3],
                                                            const bjf_patch_diff_refresh_state* state,
                                                            bjf_stream_t stream) {
  if (!grid || grid[0] <= 0 || grid[1] <= 0 || grid[2] <= 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must be non-empty");
  if (streams <= 0 || streams > (int64_t(1) << 31) - 1) return fail(BJF_ERR_INVALID_ARGUMENT, "stream count must be positive");
  const int64_t n = grid[0] * grid[1] * grid[2];
  if (n > kMaxViewerTokens) return fail(BJF_ERR_UNSUPPORTED, "viewer masks support grids up to 32768 tokens");
  if (!write_indices || !write_counts) return fail(BJF_ERR_INVALID_ARGUMENT, "viewer mask buffers must not be null");
  const bjf_patch_diff_refresh_config off{};
  RefreshParams r{};
  const bjf_status rc = refresh_params(&off, state, nullptr, n, nullptr, r);
  if (rc) return rc;
  refresh_observe_kernel<<<(unsigned)streams, kViewerThreads, 0, as_cuda(stream)>>>(write_indices, write_counts,
                                                                                    (int)n, r);
  return check_launch("refresh observe launch");
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

namespace {
bjf_status masks_from_rgba(const uint8_t* prev, const uint8_t* current, int64_t streams, int64_t width,
                           int64_t height, int64_t patch_size, const int64_t grid[3],
                           const bjf_patch_diff_config* config, const bjf_viewer_mask_policy* policy,
                           const bjf_patch_diff_refresh_config* refresh, const bjf_patch_diff_refresh_state* state,
                           int32_t* write_indices, int32_t* write_counts, int32_t* encode_indices,
                           int32_t* encode_counts, bjf_rgba_frame_stats* stats_out, void* workspace,
                           size_t workspace_bytes, bjf_stream_t stream) {
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
  RefreshParams rp{};
  if (state) {
    // PatchDiffRefreshState::masks_from_scores after the scores; a dense shortcut is
    // observe_write_mask of every token (crates/bevy_jepa/src/mask.rs:151-175)
    rc = refresh_params(refresh, state, scores, n, config, rp);
    if (rc) return rc;
  }
  cudaStream_t st = as_cuda(stream);
  rc = bjf_rgba_patch_diff_scores(prev, current, streams, width, height, patch_size, grid, scores, stats_out,
                                  workspace, workspace_bytes, stream);
  if (rc) return rc;
  rc = launch_select(scores, streams, sp, write_indices, write_counts, st);
  if (rc) return rc;
  return launch_viewer_masks(write_indices, write_counts, streams, vp, write_indices, write_counts, encode_indices,
                             encode_counts, st, state ? &rp : nullptr);
}
}  // namespace

extern "C" bjf_status bjf_viewer_patch_diff_masks_from_rgba(
    const uint8_t* prev, const uint8_t* current, int64_t streams, int64_t width, int64_t height, int64_t patch_size,
    const int64_t grid[3], const bjf_patch_diff_config* config, const bjf_viewer_mask_policy* policy,
    int32_t* write_indices, int32_t* write_counts, int32_t* encode_indices, int32_t* encode_counts,
    bjf_rgba_frame_stats* stats_out, void* workspace, size_t workspace_bytes, bjf_stream_t stream) {
  return masks_from_rgba(prev, current, streams, width, height, patch_size, grid, config, policy, nullptr, nullptr,
                         write_indices, write_counts, encode_indices, encode_counts, stats_out, workspace,
                         workspace_bytes, stream);
}

extern "C" bjf_status bjf_viewer_patch_diff_refresh_masks_from_rgba(
    const uint8_t* prev, const uint8_t* current, int64_t streams, int64_t width, int64_t height, int64_t patch_size,
    const int64_t grid[3], const bjf_patch_diff_config* config, const bjf_viewer_mask_policy* policy,
    const bjf_patch_diff_refresh_config* refresh, const bjf_patch_diff_refresh_state* state,
    int32_t* write_indices, int32_t* write_counts, int32_t* encode_indices, int32_t* encode_counts,
    bjf_rgba_frame_stats* stats_out, void* workspace, size_t workspace_bytes, bjf_stream_t stream) {
  if (!state) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff refresh state buffers must not be null");
  return masks_from_rgba(prev, current, streams, width, height, patch_size, grid, config, policy, refresh, state,
                         write_indices, write_counts, encode_indices, encode_counts, stats_out, workspace,
                         workspace_bytes, stream);
}
