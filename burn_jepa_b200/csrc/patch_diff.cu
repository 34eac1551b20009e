// patch_diff.cu -- step 1 of the sparse front end: patch-diff scores and the
// device-side mask selection.
//
// Scores restate `patch_diff_token_scores` (burn_jepa src/nodes.rs:565-631):
//   score[t, r, c] = sum_{pairs, b, ch, py, px} |x[f] - x[f-1]| / (pairs * B * C * P * P)
// with the frame pairs of `patch_diff_frame_pairs` (:621-631).  The reference runs
// a chain of tensor ops per tubelet and reads the clip about twice; here one
// memory-bound pass reads every byte once with 16-byte non-allocating loads, a
// group of P/VEC lanes owns one token column, and the partial sums meet through
// warp shuffles.
//
// Selection restates `patch_diff_context_mask_from_scores` (:458-537): sort by
// (score desc, index asc), keep while score >= threshold up to a cap, fill to a
// minimum, then SparseTokenMask::new (ascending, unique).  Without dilation the
// result is the top-n set for a count n fixed by the threshold count, so the
// kernel finds n, radix-selects the n-th largest key when n differs from the
// threshold count, and compacts the chosen indices in ascending order with block
// scans -- no sort, no host round trip.  With dilation the order of insertion
// matters when the cap binds, so that case sorts the keys in shared memory and
// replays the reference's walk exactly on one thread (push_dilated_sparse_index,
// :633-662); the common case (cap never binds) is the parallel union.
#include <algorithm>
#include <cmath>

#include <mutex>

#include "common.cuh"
#include "patch_diff.hpp"
#include "status.hpp"

namespace bjf {
namespace {

constexpr int kScoreThreads = 256;

// Frame pairs of tubelet t (nodes.rs:621-631): pairs are (f-1, f) for f in
// [first_next, first_next + npairs).
__device__ __forceinline__ void tubelet_pairs(int t, int kt, int frames, int& first_next, int& npairs) {
  int start = t * kt;
  int end = min((t + 1) * kt, frames);
  if (end > start + 1) {
    first_next = start + 1;
    npairs = end - start - 1;
  } else if (start > 0) {
    first_next = start;
    npairs = 1;
  } else {
    first_next = 0;
    npairs = 0;
  }
}

// The end of a scores pass.  Launched as a programmatic dependent, the pass may overlap the kernel
// before it (the previous frame's gather-GEMM, which none of its inputs depend on); it still does
// not complete before that kernel, so everything after it in the stream sees both finished.  Then
// the cache aging, now that the previous frame's GEMM (which writes observed / age) is done;
// blocks that finish their units early do it while others still stream.
__device__ __forceinline__ void finish_scores_pass(const ScoresAging& aging) {
  pdl_wait();
  if (aging.age) {
    const long long n4 = aging.len >> 2;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x, step = (long long)gridDim.x * blockDim.x;
    float4* a4 = reinterpret_cast<float4*>(aging.age);
    const float4* o4 = reinterpret_cast<const float4*>(aging.observed);
    for (long long i = tid; i < n4; i += step) {
      float4 a = a4[i];
      const float4 o = o4[i];
      a.x += o.x;
      a.y += o.y;
      a.z += o.z;
      a.w += o.w;
      a4[i] = a;
    }
    for (long long i = n4 * 4 + tid; i < aging.len; i += step) aging.age[i] += aging.observed[i];
  }
}

// Vectorised scores: a work unit is one (stream, tubelet, token row, chunk of token
// columns); warps stride over the units (a grid of 4 or 5 blocks of 8 warps per SM, 4 resident
// at <= 64 registers; the row loop unrolled eight deep so each lane keeps up to 16 loads in
// flight).  Consecutive warps of a block take adjacent column chunks of the same rows.
// Lane l covers VEC elements of token column (chunk*TPW + l/LPT).
template <typename T>
__global__ void __launch_bounds__(kScoreThreads, 4)
    patch_diff_scores_vec_kernel(const T* __restrict__ video, float* __restrict__ scores, int batch,
                                 int channels, int frames, int height, int width, int kt, int P,
                                 int depth, int gh, int gw, int chunks_per_row, long long total_warps,
                                 FrameRing ring, ScoresAging aging) {
  constexpr int VEC = 16 / sizeof(T);
  const int LPT = P / VEC;      // lanes per token column
  const int TPW = 32 / LPT;     // token columns per warp
  const int lane = threadIdx.x & 31;
  for (long long wid = (long long)blockIdx.x * (kScoreThreads / 32) + (threadIdx.x >> 5); wid < total_warps;
       wid += (long long)gridDim.x * (kScoreThreads / 32)) {
  const int chunk = (int)(wid % chunks_per_row);
  long long rest = wid / chunks_per_row;
  const int r = (int)(rest % gh);
  rest /= gh;
  const int t = (int)(rest % depth);
  const long long s = rest / depth;

  const int col = chunk * TPW + lane / LPT;
  const int part = lane % LPT;
  const bool valid = col < gw;
  const int x = col * P + part * VEC;

  int first_next, npairs;
  tubelet_pairs(t, kt, frames, first_next, npairs);
  const long long n_tokens = (long long)depth * gh * gw;
  float* out = scores + s * n_tokens + ((long long)t * gh + r) * gw;
  if (npairs == 0) {
    if (valid && part == 0) out[col] = 0.0f;
    continue;
  }

  const long long plane = (long long)height * width;
  float acc = 0.0f;
  if (valid) {
    for (int b = 0; b < batch; ++b) {
      for (int ch = 0; ch < channels; ++ch) {
        const T* vbase = video + (((s * batch + b) * channels + ch) * ring.storage_frames) * plane +
                         (long long)(r * P) * width + x;
        for (int p = 0; p < npairs; ++p) {
          const T* nxt = vbase + (long long)ring.frame(first_next + p) * plane;
          const T* prv = vbase + (long long)ring.frame(first_next + p - 1) * plane;
#pragma unroll 8
          for (int py = 0; py < P; ++py) {
            uint4 un = ld_nc_v4(nxt + (long long)py * width);
            uint4 up = ld_nc_v4(prv + (long long)py * width);
            const T* a = reinterpret_cast<const T*>(&un);
            const T* q = reinterpret_cast<const T*>(&up);
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc += fabsf(to_f32<T>(a[v]) - to_f32<T>(q[v]));
          }
        }
      }
    }
  }
  for (int o = LPT >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (valid && part == 0) {
    const double denom = (double)npairs * batch * channels * P * P;
    out[col] = acc * (float)(1.0 / denom);
  }
  }
  finish_scores_pass(aging);
}

// Scores of a small pass (a single clip, a few streams): one block per work unit (the 16 or so
// token columns one warp covers in the pass above), its warps splitting the unit's
// (batch, channel, frame pair, pixel row) iterations round-robin, so the pass spreads over the
// SMs instead of one warp per unit on a few of them.  Each warp's per-token partial sum (lanes of
// a token combined by shuffles) meets the others in shared memory, where warp 0 adds them in
// warp order: the same result whatever the timing.
template <typename T>
__global__ void __launch_bounds__(kScoreThreads)
    patch_diff_scores_split_kernel(const T* __restrict__ video, float* __restrict__ scores, int batch,
                                   int channels, int frames, int height, int width, int kt, int P, int depth,
                                   int gh, int gw, int chunks_per_row, long long units, FrameRing ring,
                                   ScoresAging aging) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int kWarps = kScoreThreads / 32;
  __shared__ float part[kWarps][32];
  const int LPT = P / VEC;   // lanes per token column
  const int TPW = 32 / LPT;  // token columns per unit
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long u = blockIdx.x; u < units; u += gridDim.x) {
    const int chunk = (int)(u % chunks_per_row);
    long long rest = u / chunks_per_row;
    const int r = (int)(rest % gh);
    rest /= gh;
    const int t = (int)(rest % depth);
    const long long s = rest / depth;
    const int col = chunk * TPW + lane / LPT;
    const int sub = lane % LPT;
    const bool valid = col < gw;
    const int x = col * P + sub * VEC;
    int first_next, npairs;
    tubelet_pairs(t, kt, frames, first_next, npairs);
    const long long plane = (long long)height * width;
    float acc = 0.0f;
    if (valid && npairs > 0) {
      const int iters = batch * channels * npairs * P;  // (b, ch, p, py), py fastest
#pragma unroll 4
      for (int it = warp; it < iters; it += kWarps) {
        const int py = it % P;
        int q = it / P;
        const int p = q % npairs;
        q /= npairs;
        const int ch = q % channels, b = q / channels;
        const T* vbase = video + (((s * batch + b) * channels + ch) * ring.storage_frames) * plane +
                         (long long)(r * P + py) * width + x;
        const uint4 un = ld_nc_v4(vbase + (long long)ring.frame(first_next + p) * plane);
        const uint4 up = ld_nc_v4(vbase + (long long)ring.frame(first_next + p - 1) * plane);
        const T* a = reinterpret_cast<const T*>(&un);
        const T* c = reinterpret_cast<const T*>(&up);
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc += fabsf(to_f32<T>(a[v]) - to_f32<T>(c[v]));
      }
    }
    for (int o = LPT >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    part[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && valid && sub == 0) {
      float* out = scores + s * ((long long)depth * gh * gw) + ((long long)t * gh + r) * gw;
      if (npairs == 0) {
        out[col] = 0.0f;
      } else {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += part[w][lane];
        const double denom = (double)npairs * batch * channels * P * P;
        out[col] = sum * (float)(1.0 / denom);
      }
    }
    __syncthreads();  // the partials are read before the next unit writes them
  }
  finish_scores_pass(aging);
}

// Generic scores (any patch size / alignment): one thread per token.
template <typename T>
__global__ void __launch_bounds__(kScoreThreads)
    patch_diff_scores_scalar_kernel(const T* __restrict__ video, float* __restrict__ scores,
                                    int batch, int channels, int frames, int height, int width,
                                    int kt, int P, int depth, int gh, int gw, long long total,
                                    FrameRing ring) {
  pdl_wait();
  long long i = (long long)blockIdx.x * kScoreThreads + threadIdx.x;
  if (i >= total) return;
  const long long n_tokens = (long long)depth * gh * gw;
  const long long s = i / n_tokens;
  const long long tok = i % n_tokens;
  const int t = (int)(tok / ((long long)gh * gw));
  const int r = (int)((tok / gw) % gh);
  const int c = (int)(tok % gw);
  int first_next, npairs;
  tubelet_pairs(t, kt, frames, first_next, npairs);
  if (npairs == 0) {
    scores[i] = 0.0f;
    return;
  }
  const long long plane = (long long)height * width;
  float acc = 0.0f;
  for (int b = 0; b < batch; ++b)
    for (int ch = 0; ch < channels; ++ch) {
      const T* vbase = video + (((s * batch + b) * channels + ch) * ring.storage_frames) * plane;
      for (int p = 0; p < npairs; ++p) {
        const T* nxt = vbase + (long long)ring.frame(first_next + p) * plane;
        const T* prv = vbase + (long long)ring.frame(first_next + p - 1) * plane;
        for (int py = 0; py < P; ++py)
          for (int px = 0; px < P; ++px) {
            long long off = (long long)(r * P + py) * width + c * P + px;
            acc += fabsf(to_f32<T>(nxt[off]) - to_f32<T>(prv[off]));
          }
      }
    }
  const double denom = (double)npairs * batch * channels * P * P;
  scores[i] = acc * (float)(1.0 / denom);
}

// ---------------------------------------------------------------------------
// Selection
// ---------------------------------------------------------------------------
constexpr int kSelectThreads = 1024;
constexpr int kMaxSelectTokens = 32768;
constexpr int kMaxDilatedTokens = 16384;

__device__ __forceinline__ void age_stream(const SelectParams& p, long long s) {
  if (!p.age) return;
  float* a = p.age + s * p.n;
  const float* o = p.observed + s * p.n;
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) a[i] += o[i];
}

// Order-preserving float -> uint32 key (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive scan of one int per thread.  Returns the exclusive prefix
// and writes the block total to *total.  `warp_sums` holds 32 ints of smem.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  __syncthreads();
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < (int)(blockDim.x >> 5)) ? warp_sums[lane] : 0;
    int winc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc += y;
    }
    warp_sums[lane] = winc - w;  // exclusive prefix of warp totals
    if (lane == 31) warp_sums[32] = winc;
  }
  __syncthreads();
  int result = warp_sums[warp] + inc - v;
  *total = warp_sums[32];
  __syncthreads();
  return result;
}

// Each thread owns the contiguous segment [seg_begin, seg_end) so that block
// scans over per-thread counts produce ascending-index order.
__device__ __forceinline__ void thread_segment(int n, int& b, int& e) {
  int per = (n + blockDim.x - 1) / blockDim.x;
  b = min(n, (int)threadIdx.x * per);
  e = min(n, b + per);
}

// Selection without dilation.  Shared memory: keys[n] (uint32).
__global__ void __launch_bounds__(kSelectThreads)
    patch_diff_select_kernel(const float* __restrict__ scores, SelectParams p,
                             int32_t* __restrict__ indices, int32_t* __restrict__ counts) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);
  __shared__ int warp_sums[33];
  __shared__ unsigned int hist[256];
  __shared__ uint32_t sel_prefix;
  __shared__ int sel_remaining;

  // The kernel after the selection (the GEMM of the fused step) may launch now and wait
  // for this one to complete; everything before the selection has completed by now.
  pdl_trigger();
  pdl_wait();
  const int n = p.n;
  const long long s = blockIdx.x;
  const float* sc = scores + s * n;
  int seg_b, seg_e;
  thread_segment(n, seg_b, seg_e);

  // a thread's segment is at most 32 tokens (n <= 32768, 1024 threads): one pass bit each
  int pass_local = 0;
  uint32_t pass_bits = 0;
  for (int i = seg_b; i < seg_e; ++i) {
    float v = sc[i];
    keys[i] = float_key(v);
    const bool pass = !(v < p.threshold);
    pass_local += pass;
    pass_bits |= (uint32_t)pass << (i - seg_b);
  }
  age_stream(p, s);  // independent of the scores: its loads overlap the scan below
  int n_pass;
  const int pass_pos = block_exclusive_scan(pass_local, warp_sums, &n_pass);
  const int n_sel = max(min(n_pass, p.cap), p.fill_target);

  int32_t* out = indices + s * n;
  if (n_sel == n_pass) {
    int pos = pass_pos;
    for (int i = seg_b; i < seg_e; ++i)
      if (pass_bits >> (i - seg_b) & 1u) out[pos++] = i;
    if (threadIdx.x == 0) counts[s] = n_sel;
    return;
  }

  // Radix-select the n_sel-th largest key, MSB digit first.
  if (threadIdx.x == 0) {
    sel_prefix = 0;
    sel_remaining = n_sel;
  }
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = sel_prefix;
    for (int i = seg_b; i < seg_e; ++i) {
      uint32_t k = keys[i];
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int remaining = sel_remaining;
      int bin = 255;
      for (; bin > 0; --bin) {
        int c = (int)hist[bin];
        if (c >= remaining) break;
        remaining -= c;
      }
      sel_prefix = prefix | ((uint32_t)bin << shift);
      sel_remaining = remaining;
    }
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  const uint32_t kth = sel_prefix;
  const int need_equal = sel_remaining;  // how many keys == kth to take, lowest index first

  int eq_local = 0;
  for (int i = seg_b; i < seg_e; ++i) eq_local += (keys[i] == kth);
  int eq_total;
  int eq_rank = block_exclusive_scan(eq_local, warp_sums, &eq_total);
  int local = 0;
  {
    int r = eq_rank;
    for (int i = seg_b; i < seg_e; ++i) {
      uint32_t k = keys[i];
      bool take = k > kth || (k == kth && r < need_equal);
      r += (k == kth);
      local += take;
    }
  }
  int total;
  int pos = block_exclusive_scan(local, warp_sums, &total);
  {
    int r = eq_rank;
    for (int i = seg_b; i < seg_e; ++i) {
      uint32_t k = keys[i];
      bool take = k > kth || (k == kth && r < need_equal);
      r += (k == kth);
      if (take) out[pos++] = i;
    }
  }
  if (threadIdx.x == 0) counts[s] = n_sel;
}

__device__ __forceinline__ bool push_dilated(int index, const SelectParams& p, unsigned char* keep,
                                             int& nsel, int target) {
  // Returns true when `target` is reached (push_dilated_sparse_index, nodes.rs:633-662).
  if (nsel >= target || index >= p.n) return nsel >= target;
  const int tpf = p.gh * p.gw;
  const int t = index / tpf, rem = index - t * tpf;
  const int row = rem / p.gw, col = rem - row * p.gw;
  const int r0 = max(row - p.dilation, 0), r1 = min(row + p.dilation, p.gh - 1);
  const int c0 = max(col - p.dilation, 0), c1 = min(col + p.dilation, p.gw - 1);
  for (int r = r0; r <= r1; ++r)
    for (int c = c0; c <= c1; ++c) {
      int idx = t * tpf + r * p.gw + c;
      if (keep[idx]) continue;
      keep[idx] = 1;
      if (++nsel >= target) return true;
    }
  return false;
}

// Selection with dilation.  Shared memory: comp[npow2] (uint64), keep[n] (bytes).
__global__ void __launch_bounds__(kSelectThreads)
    patch_diff_select_dilated_kernel(const float* __restrict__ scores, SelectParams p, int npow2,
                                     int32_t* __restrict__ indices, int32_t* __restrict__ counts) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned long long* comp = reinterpret_cast<unsigned long long*>(smem_raw);
  unsigned char* keep = smem_raw + sizeof(unsigned long long) * npow2;
  __shared__ int warp_sums[33];
  __shared__ int use_sequential;

  pdl_trigger();
  pdl_wait();
  const int n = p.n;
  const long long s = blockIdx.x;
  const float* sc = scores + s * n;
  int seg_b, seg_e;
  thread_segment(n, seg_b, seg_e);
  age_stream(p, s);

  for (int i = threadIdx.x; i < n; i += blockDim.x) keep[i] = 0;
  __syncthreads();
  // Parallel union of the dilated neighbourhoods of every token at or above the threshold.
  const int tpf = p.gh * p.gw;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (sc[i] < p.threshold) continue;
    const int t = i / tpf, rem = i - t * tpf;
    const int row = rem / p.gw, col = rem - row * p.gw;
    const int r0 = max(row - p.dilation, 0), r1 = min(row + p.dilation, p.gh - 1);
    const int c0 = max(col - p.dilation, 0), c1 = min(col + p.dilation, p.gw - 1);
    for (int r = r0; r <= r1; ++r)
      for (int c = c0; c <= c1; ++c) keep[t * tpf + r * p.gw + c] = 1;
  }
  __syncthreads();
  int local = 0;
  for (int i = seg_b; i < seg_e; ++i) local += keep[i];
  int n_union;
  block_exclusive_scan(local, warp_sums, &n_union);
  if (threadIdx.x == 0) use_sequential = !(n_union <= p.cap && n_union >= p.fill_target);
  __syncthreads();

  if (use_sequential) {
    // Exact replay: sort (score desc, index asc), then the reference's two loops.
    for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
      comp[i] = i < n ? ((unsigned long long)(~float_key(sc[i])) << 32) | (unsigned)i
                      : ~0ull;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) keep[i] = 0;
    __syncthreads();
    for (int k = 2; k <= npow2; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
          int ixj = i ^ j;
          if (ixj > i) {
            unsigned long long a = comp[i], b = comp[ixj];
            bool up = (i & k) == 0;
            if ((a > b) == up) {
              comp[i] = b;
              comp[ixj] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    if (threadIdx.x == 0) {
      int nsel = 0;
      for (int i = 0; i < n; ++i) {
        int idx = (int)(comp[i] & 0xFFFFFFFFu);
        if (sc[idx] < p.threshold) break;
        if (push_dilated(idx, p, keep, nsel, p.cap)) break;
      }
      if (nsel < p.fill_target) {
        for (int i = 0; i < n; ++i) {
          int idx = (int)(comp[i] & 0xFFFFFFFFu);
          if (push_dilated(idx, p, keep, nsel, p.fill_target)) break;
        }
      }
    }
    __syncthreads();
  }

  local = 0;
  for (int i = seg_b; i < seg_e; ++i) local += keep[i];
  int total;
  int pos = block_exclusive_scan(local, warp_sums, &total);
  int32_t* out = indices + s * n;
  for (int i = seg_b; i < seg_e; ++i)
    if (keep[i]) out[pos++] = i;
  if (threadIdx.x == 0) counts[s] = total;
}

bool grid_ok(const int64_t* g) { return g && g[0] > 0 && g[1] > 0 && g[2] > 0; }

}  // namespace

// Resolves the reference's budget arithmetic (nodes.rs:463-498, 516-520).
bjf_status resolve_select(const bjf_patch_diff_config* cfg, const int64_t* grid, SelectParams& p) {
  if (!cfg) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff config must not be null");
  if (!std::isfinite(cfg->threshold) || !(cfg->threshold >= 0.0f))
    return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff sparsity threshold must be finite and non-negative");
  const int64_t len = grid[0] * grid[1] * grid[2];
  if (cfg->dilation < 0) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff dilation must be non-negative");
  int64_t context;
  if (cfg->allow_full_context) {
    context = std::min(std::max<int64_t>(cfg->context_tokens, 1), len);
  } else {
    if (len <= 1) return fail(BJF_ERR_INVALID_ARGUMENT, "sparse JEPA mode requires at least two dense tokens");
    context = std::min(std::max<int64_t>(cfg->context_tokens, 1), len - 1);
  }
  const int64_t min_ctx = std::min(std::min(std::max<int64_t>(cfg->min_context_tokens, 1), context), len);
  p.threshold = cfg->threshold;
  p.cap = (int)(cfg->allow_full_context ? len : context);
  p.fill_target = (int)(cfg->fill_to_context_tokens ? context : min_ctx);
  p.dilation = (int)std::min<int64_t>(cfg->dilation, 1 << 20);
  p.depth = (int)grid[0];
  p.gh = (int)grid[1];
  p.gw = (int)grid[2];
  p.n = (int)len;
  p.age = nullptr;
  p.observed = nullptr;
  return BJF_OK;
}

bjf_status launch_select(const float* scores, int64_t streams, const SelectParams& p,
                         int32_t* indices, int32_t* counts, cudaStream_t st, bool pdl) {
  if (p.dilation == 0) {
    if (p.n > kMaxSelectTokens)
      return fail(BJF_ERR_UNSUPPORTED, "patch-diff selection supports grids up to 32768 tokens");
    size_t smem = sizeof(uint32_t) * (size_t)p.n;
    cudaError_t e = cudaFuncSetAttribute(patch_diff_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "patch-diff select attribute");
    e = launch_kernel(pdl, patch_diff_select_kernel, dim3((unsigned)streams), dim3(kSelectThreads), smem, st,
                      scores, p, indices, counts);
    return e == cudaSuccess ? BJF_OK : cuda_status(e, "patch-diff select launch");
  }
  if (p.n > kMaxDilatedTokens)
    return fail(BJF_ERR_UNSUPPORTED, "dilated patch-diff selection supports grids up to 16384 tokens");
  int npow2 = 1;
  while (npow2 < p.n) npow2 <<= 1;
  size_t smem = sizeof(unsigned long long) * (size_t)npow2 + (size_t)p.n;
  smem = (smem + 15) & ~size_t(15);
  cudaError_t e = cudaFuncSetAttribute(patch_diff_select_dilated_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "dilated select attribute");
  e = launch_kernel(pdl, patch_diff_select_dilated_kernel, dim3((unsigned)streams), dim3(kSelectThreads), smem,
                    st, scores, p, npow2, indices, counts);
  return e == cudaSuccess ? BJF_OK : cuda_status(e, "dilated patch-diff select launch");
}

namespace {
constexpr int kMaxDev = 64;
std::mutex g_scores_mu;
int g_sms[kMaxDev] = {};

// SM count of the current device by attribute query (nothing here allocates).
int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 148;
  std::lock_guard<std::mutex> lock(g_scores_mu);
  if (!g_sms[dev] && cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return g_sms[dev];
}
}  // namespace

bjf_status launch_scores(const void* video, int32_t dtype, const int64_t* vd, int64_t streams,
                         int64_t kt, int64_t P, float* scores, cudaStream_t st, bool pdl, const FrameRing* ring_in,
                         const ScoresAging* aging_in, bool* aged) {
  if (aged) *aged = false;
  const int64_t B = vd[0], C = vd[1], T = vd[2], H = vd[3], W = vd[4];
  const FrameRing ring = ring_in ? *ring_in : FrameRing::contiguous((int)T);
  const int64_t depth = T / kt, gh = H / P, gw = W / P;
  const int64_t n_tok = depth * gh * gw;
  if (n_tok == 0 || streams == 0) return BJF_OK;
  bjf_status rc = BJF_OK;
  bool ok = dispatch_float(dtype, [&](auto tag) {
    using T_ = decltype(tag);
    constexpr int VEC = 16 / sizeof(T_);
    const bool vec_ok = (P % VEC == 0) && (32 % (P / VEC) == 0) && (W % VEC == 0) &&
                        (reinterpret_cast<uintptr_t>(video) % 16 == 0);
    if (vec_ok) {
      const int LPT = (int)(P / VEC);
      const int TPW = 32 / LPT;
      const int chunks = (int)ceil_div(gw, TPW);
      long long warps = (long long)streams * depth * gh * chunks;
      // A grid-stride grid of one resident wave (4 blocks per SM), or of 5 blocks per SM for a
      // pass of at most 1.5 units a warp at that size.  In the fused step the pass starts beside
      // the previous frame's GEMM, where only two blocks an SM fit; measured on the live step
      // (32 streams, 8192 units) five blocks per SM gave 0.111 ms a step against 0.118 with four,
      // while at 64 streams (16 384 units) four were best, and five left the pass alone a tail
      // (0.90 vs 0.98 of HBM).
      const long long sms = sm_count();
      const long long per_sm = warps * 2 <= sms * 5 * (kScoreThreads / 32) * 3 ? 5 : 4;
      long long blocks = std::min<long long>(ceil_div(warps, kScoreThreads / 32), sms * per_sm);
      // 16-byte aligned metadata for the float4 aging loop
      ScoresAging aging{};
      if (aging_in && aging_in->age &&
          ((reinterpret_cast<uintptr_t>(aging_in->age) | reinterpret_cast<uintptr_t>(aging_in->observed)) & 15) == 0)
        aging = *aging_in;
      cudaError_t e;
      if (warps < sms * (kScoreThreads / 32)) {
        // too few units for a block of them on every SM (a single clip): a block per unit, its
        // warps splitting the unit's loop.  Measured: one ViT-L clip [3, 16, 256, 256] (128 units),
        // fused step 0.034 vs 0.046 ms; 8 live streams (2048 units) stay faster one warp a unit
        // (0.050 vs 0.057 ms split).
        e = launch_kernel(pdl, patch_diff_scores_split_kernel<T_>,
                          dim3((unsigned)std::min<long long>(warps, sms * (kScoreThreads / 32))),
                          dim3(kScoreThreads), 0, st, static_cast<const T_*>(video), scores, (int)B, (int)C, (int)T,
                          (int)H, (int)W, (int)kt, (int)P, (int)depth, (int)gh, (int)gw, chunks, warps, ring,
                          aging);
      } else {
        e = launch_kernel(pdl, patch_diff_scores_vec_kernel<T_>, dim3((unsigned)blocks), dim3(kScoreThreads), 0,
                          st, static_cast<const T_*>(video), scores, (int)B, (int)C, (int)T, (int)H, (int)W,
                          (int)kt, (int)P, (int)depth, (int)gh, (int)gw, chunks, warps, ring, aging);
      }
      rc = e == cudaSuccess ? BJF_OK : cuda_status(e, "patch-diff scores launch");
      if (!rc && aged) *aged = aging.age != nullptr;
      return;
    } else {
      long long total = (long long)streams * n_tok;
      patch_diff_scores_scalar_kernel<T_><<<(unsigned)ceil_div(total, kScoreThreads), kScoreThreads, 0, st>>>(
          static_cast<const T_*>(video), scores, (int)B, (int)C, (int)T, (int)H, (int)W, (int)kt,
          (int)P, (int)depth, (int)gh, (int)gw, total, ring);
    }
    rc = check_launch("patch-diff scores launch");
  });
  if (!ok) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff video dtype must be f32, f16 or bf16");
  return rc;
}

namespace {
bjf_status validate_video(const void* video, const int64_t* vd, int64_t streams, int64_t kt, int64_t P) {
  if (!vd) return fail(BJF_ERR_INVALID_ARGUMENT, "video dims must not be null");
  for (int i = 0; i < 5; ++i)
    if (vd[i] <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "video dims must be positive, got " + dims_str(vd, 5));
  if (streams <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "stream count must be positive");
  if (kt <= 0 || P <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "tubelet and patch sizes must be positive");
  if (!video) return fail(BJF_ERR_INVALID_ARGUMENT, "video pointer must not be null");
  const int64_t elems = streams * vd[0] * vd[1] * vd[2] * vd[3] * vd[4];
  if (elems / streams / vd[0] / vd[1] / vd[2] / vd[3] != vd[4] || elems > (int64_t(1) << 40))
    return fail(BJF_ERR_INVALID_ARGUMENT, "video element count overflow");
  if (vd[2] > (1 << 30) || vd[3] > (1 << 30) || vd[4] > (1 << 30))
    return fail(BJF_ERR_INVALID_ARGUMENT, "video dims exceed the supported range");
  return BJF_OK;
}

}  // namespace
}  // namespace bjf

using namespace bjf;

extern "C" {

bjf_status bjf_patch_diff_token_scores(const void* video, bjf_dtype video_dtype,
                                       const int64_t video_dims[5], int64_t streams,
                                       int64_t tubelet_size, int64_t patch_size, float* scores,
                                       bjf_stream_t stream) {
  bjf_status rc = validate_video(video, video_dims, streams, tubelet_size, patch_size);
  if (rc) return rc;
  if (!scores) return fail(BJF_ERR_INVALID_ARGUMENT, "scores pointer must not be null");
  return launch_scores(video, video_dtype, video_dims, streams, tubelet_size, patch_size, scores,
                       as_cuda(stream));
}

bjf_status bjf_patch_diff_context_mask_from_scores(const float* scores, int64_t streams,
                                                   const int64_t grid[3],
                                                   const bjf_patch_diff_config* config,
                                                   int32_t* indices, int32_t* counts,
                                                   bjf_stream_t stream) {
  if (!grid_ok(grid)) return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must be non-empty");
  if (streams <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "stream count must be positive");
  if (!scores || !indices || !counts) return fail(BJF_ERR_INVALID_ARGUMENT, "scores, indices and counts must not be null");
  if (grid[0] * grid[1] * grid[2] > (int64_t(1) << 30)) return fail(BJF_ERR_UNSUPPORTED, "token grid too large");
  SelectParams p;
  bjf_status rc = resolve_select(config, grid, p);
  if (rc) return rc;
  return launch_select(scores, streams, p, indices, counts, as_cuda(stream));
}

bjf_status bjf_patch_diff_context_mask(const void* video, bjf_dtype video_dtype,
                                       const int64_t video_dims[5], int64_t streams,
                                       int64_t tubelet_size, int64_t patch_size,
                                       const int64_t grid[3], const bjf_patch_diff_config* config,
                                       float* scores, int32_t* indices, int32_t* counts,
                                       bjf_stream_t stream) {
  // Check order follows patch_diff_context_mask (nodes.rs:417-441).
  if (!config) return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff config must not be null");
  if (!std::isfinite(config->threshold) || !(config->threshold >= 0.0f))
    return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff sparsity threshold must be finite and non-negative");
  bjf_status rc = validate_video(video, video_dims, streams, tubelet_size, patch_size);
  if (rc) return rc;
  if (!grid_ok(grid)) return fail(BJF_ERR_INVALID_ARGUMENT, "token grid must be non-empty");
  const int64_t T = video_dims[2], H = video_dims[3], W = video_dims[4];
  if (T % tubelet_size || H % patch_size || W % patch_size)
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "patch-diff sparsity requires frames/height/width divisible by tubelet and patch sizes");
  if (T / tubelet_size != grid[0] || H / patch_size != grid[1] || W / patch_size != grid[2])
    return fail(BJF_ERR_INVALID_ARGUMENT, "patch-diff sparsity grid must match the video shape");
  if (!scores || !indices || !counts) return fail(BJF_ERR_INVALID_ARGUMENT, "scores, indices and counts must not be null");
  if (grid[0] * grid[1] * grid[2] > (int64_t(1) << 30)) return fail(BJF_ERR_UNSUPPORTED, "token grid too large");
  SelectParams p;
  rc = resolve_select(config, grid, p);
  if (rc) return rc;
  cudaStream_t st = as_cuda(stream);
  rc = launch_scores(video, video_dtype, video_dims, streams, tubelet_size, patch_size, scores, st);
  if (rc) return rc;
  return launch_select(scores, streams, p, indices, counts, st);
}

}  // extern "C"
