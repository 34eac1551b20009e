// rgba.cu -- the live viewer's patch-diff scorer for RGBA u8 camera frames
// (burn_jepa src/viewer.rs:1069-1270: rgba_patch_diff_frame_stats, patch_diff_scores_from_rgba,
// rgba_patch_diff_pixel_score), batched over S independent streams.  Two passes over the frames:
//
//   1. lighting means   (rgba_means_kernel) per stream: mean RGB delta, mean luma delta, mean
//                       per-pixel |delta|
//   2. patches          (rgba_patch_kernel) one warp per patch: the patch score
//                       mean(max(|rgb delta| / 3, |luma delta|, relative luma / 4, chroma delta / 2))
//                       both as is and with the global lighting shift removed, and the lighting
//                       residual mean |delta - mean delta| (the shifted score's RGB term is that
//                       residual's per-pixel term, so one pass yields both)
//   3. finalize         (rgba_finalize_kernel, no frame reads) per stream: compensate when
//                       raw > 1e-4 and residual <= 0.35 raw, keep that score, write the stats
//
// When the means of pass 1 already rule the compensation out and no statistics are wanted,
// pass 2 computes the unshifted score alone and skips the pixels that did not change.
//
// The frame-wide sums are accumulated in f64 and reduced in a fixed order from per-block
// partials kept in the caller's workspace, so results do not depend on timing and no counters
// need resetting.  Every per-pixel operation is rounded as the reference's f32 code does (no
// contraction): u8 / 255 comes from a shared-memory table of the correctly rounded quotients,
// x / 3 from div3_rn below, the chroma quotients from a reciprocal and a correction step
// (div_by_rcp), every other quotient from an IEEE division.  The sums differ from
// the reference's sequential f32 loops in order and in precision: the channel-delta means are
// exact here (see accumulate_means), the luma and mean-|delta| sums nearly so, while the
// reference's f32 running sums round at every pixel.  The frame statistics therefore agree to
// within the reference's own f32 summation error, and a frame whose lighting residual sits
// within that error of 0.35 x the raw mean can take the other compensation decision.
#include <algorithm>
#include <string>

#include "../../include/bjf.h"
#include "common.cuh"
#include "runtime.hpp"
#include "status.hpp"

namespace bjf {
namespace {

constexpr int kRgbaThreads = 256;
constexpr int kPatchWarps = kRgbaThreads / 32;  // patches per block of the patch pass
constexpr int kStatBlocks = 64;                 // mean partials per stream
constexpr int kPatchBlocksTarget = 592;         // patch-pass blocks over all streams: 148 SMs x 4 resident
constexpr int kMeanParts = 5;                   // sum dR, dG, dB, d luma, per-pixel mean |delta|

struct Rgb {
  float r, g, b;
};

// Correctly rounded x / 3 for 0 <= x < 4: q = RN(x * RN(1/3)) is within one ulp of x / 3, the
// FMA residual x - 3q is exact and RN(q + r * RN(1/3)) is the correctly rounded quotient
// (Markstein's correction step).  Checked against IEEE division for every f32 in [0, 4).
__device__ __forceinline__ float div3_rn(float x) {
  constexpr float kThird = 0x1.555556p-2f;  // RN(1/3)
  const float q = __fmul_rn(x, kThird);
  const float r = __fmaf_rn(-q, 3.0f, x);
  return __fmaf_rn(r, kThird, q);
}

// inv[i] = RN(i / 255), the reference's `rgba[offset + c] as f32 / 255.0` (src/viewer.rs:1246-1252).
__device__ __forceinline__ void build_u8_table(float* inv) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) inv[i] = __fdiv_rn((float)i, 255.0f);
}

__device__ __forceinline__ Rgb rgb_of(uint32_t px, const float* inv) {
  return Rgb{inv[px & 255u], inv[(px >> 8) & 255u], inv[(px >> 16) & 255u]};
}

// rgb[0] * 0.2126 + rgb[1] * 0.7152 + rgb[2] * 0.0722 (:1254-1256)
__device__ __forceinline__ float luma(Rgb c) {
  return __fadd_rn(__fadd_rn(__fmul_rn(c.r, 0.2126f), __fmul_rn(c.g, 0.7152f)), __fmul_rn(c.b, 0.0722f));
}

// The chroma denominators max(r + g + b, 0.10) of the previous and current pixel.
struct ChromaDen {
  float dp, dc;
};

__device__ __forceinline__ ChromaDen chroma_den(Rgb p, Rgb c) {
  return ChromaDen{fmaxf(__fadd_rn(__fadd_rn(p.r, p.g), p.b), 0.10f),
                   fmaxf(__fadd_rn(__fadd_rn(c.r, c.g), c.b), 0.10f)};
}

// a / b correctly rounded from y = RN(1 / b): q = RN(a y), then Markstein's correction step
// RN(q + (a - b q) y) (the residual is exact with an FMA).  Used where a is a channel value
// i / 255 and b a chroma denominator max(r + g + b, 0.10) of such values: checked on the host
// against IEEE division for every one of those (a, b) pairs.
__device__ __forceinline__ float div_by_rcp(float a, float b, float y) {
  const float q = __fmul_rn(a, y);
  return __fmaf_rn(__fmaf_rn(-q, b, a), y, q);
}

// (sum of |chroma delta|) / 3 with chroma = rgb / max(r + g + b, 0.10) (:1258-1270): one
// reciprocal per pixel and denominator instead of six divisions
__device__ __forceinline__ float chroma_diff(Rgb p, Rgb c, ChromaDen d) {
  const float yc = __frcp_rn(d.dc), yp = __frcp_rn(d.dp);
  const float a = fabsf(__fsub_rn(div_by_rcp(c.r, d.dc, yc), div_by_rcp(p.r, d.dp, yp)));
  const float b = fabsf(__fsub_rn(div_by_rcp(c.g, d.dc, yc), div_by_rcp(p.g, d.dp, yp)));
  const float e = fabsf(__fsub_rn(div_by_rcp(c.b, d.dc, yc), div_by_rcp(p.b, d.dp, yp)));
  return div3_rn(__fadd_rn(__fadd_rn(a, b), e));
}

// A pixel's score is max(max(max(rgb, luma), rel), chroma) (:1238-1243).  The two tests below
// show without a division that a term is below m = max(rgb, luma), so the maximum is the same
// without it.  Both leave margins far above the rounding of the terms they bound (checked on
// the host against the rounded terms for pixel pairs of several distributions).
//
// rel = min(RN(luma / den), 1) / 4 <= (luma / den)(1 + 2^-24) / 4: below m when
// luma / 4 (1 + 1e-5) <= m den, up to the roundings of this test.
__device__ __forceinline__ bool rel_below(float luma_abs, float den, float m) {
  return __fmul_rn(__fmul_rn(luma_abs, 0.25f), 1.00001f) <= __fmul_rn(m, den);
}

// chroma / 2 with Q_i = c_i / dc - p_i / dp is at most (sum |Q_i| + 4e-7) / 6 (1 + 1e-6) after
// its roundings (each quotient is at most 1), and sum |Q_i| = w / (dc dp) with
// w = sum |c_i dp - p_i dc| computed here within 3e-6: below m when w + 7e-6 < 5.999 m dc dp.
__device__ __forceinline__ bool chroma_below(Rgb p, Rgb c, ChromaDen d, float m) {
  const float w = __fadd_rn(__fadd_rn(fabsf(__fmaf_rn(c.r, d.dp, -__fmul_rn(p.r, d.dc))),
                                      fabsf(__fmaf_rn(c.g, d.dp, -__fmul_rn(p.g, d.dc)))),
                            fabsf(__fmaf_rn(c.b, d.dp, -__fmul_rn(p.b, d.dc))));
  return __fadd_rn(w, 7.0e-6f) < __fmul_rn(__fmul_rn(__fmul_rn(5.999f, m), d.dc), d.dp);
}

__device__ __forceinline__ float rel_term(float luma_abs, float den) {
  return __fmul_rn(fminf(__fdiv_rn(luma_abs, den), 1.0f), 0.25f);
}

// Block-wide sum of a double in a fixed order (all threads get the result).
__device__ __forceinline__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < kRgbaThreads / 32; ++w) t += red[w];
  return t;
}

// True when the two pixels' RGB bytes are equal (alpha is not read).
__device__ __forceinline__ bool same_rgb(uint32_t pp, uint32_t cp) { return ((pp ^ cp) & 0x00ffffffu) == 0; }

// One pixel's contribution to the frame means (src/viewer.rs:1079-1100).  The channel deltas are
// multiples of 2^-31 below 1 in magnitude, so their f64 sums are exact in any order; the luma
// delta and the mean |delta| have finer steps, so their f64 sums round (far below the f32
// rounding of the reference's running sums).  An unchanged pixel adds exact zeros, so it is
// skipped.
__device__ __forceinline__ void accumulate_means(uint32_t pp, uint32_t cp, const float* inv, double (&acc)[5]) {
  if (same_rgb(pp, cp)) return;
  const Rgb a = rgb_of(pp, inv), b = rgb_of(cp, inv);
  const float dr = __fsub_rn(b.r, a.r), dg = __fsub_rn(b.g, a.g), db = __fsub_rn(b.b, a.b);
  acc[0] += dr;
  acc[1] += dg;
  acc[2] += db;
  acc[3] += __fsub_rn(luma(b), luma(a));
  acc[4] += div3_rn(__fadd_rn(__fadd_rn(fabsf(dr), fabsf(dg)), fabsf(db)));
}

// Pass 1: per block, sums over its pixel range of the channel deltas, the luma delta and the
// per-pixel mean |delta|.  vec: both frames 16-byte aligned with a multiple of 4 pixels, read
// four pixels per load.
__global__ void __launch_bounds__(kRgbaThreads)
    rgba_means_kernel(const uint8_t* __restrict__ prev, const uint8_t* __restrict__ cur, long long pixels, int vec,
                      double* __restrict__ partials) {
  __shared__ float inv[256];
  __shared__ double red[kRgbaThreads / 32];
  build_u8_table(inv);
  __syncthreads();
  const long long s = blockIdx.y;
  const uint8_t* p0 = prev + s * pixels * 4;
  const uint8_t* c0 = cur + s * pixels * 4;
  double acc[kMeanParts] = {0, 0, 0, 0, 0};
  const long long first = (long long)blockIdx.x * kRgbaThreads + threadIdx.x;
  const long long step = (long long)kStatBlocks * kRgbaThreads;
  if (vec) {
    // two iterations' loads in flight per thread, consumed in the same order as one at a time
    const uint4* p4 = reinterpret_cast<const uint4*>(p0);
    const uint4* c4 = reinterpret_cast<const uint4*>(c0);
    const long long nq = pixels / 4;
    for (long long i = first; i < nq; i += 2 * step) {
      const bool second = i + step < nq;
      const uint4 a0 = __ldg(p4 + i), b0 = __ldg(c4 + i);
      uint4 a1 = a0, b1 = b0;
      if (second) {
        a1 = __ldg(p4 + i + step);
        b1 = __ldg(c4 + i + step);
      }
      accumulate_means(a0.x, b0.x, inv, acc);
      accumulate_means(a0.y, b0.y, inv, acc);
      accumulate_means(a0.z, b0.z, inv, acc);
      accumulate_means(a0.w, b0.w, inv, acc);
      if (second) {
        accumulate_means(a1.x, b1.x, inv, acc);
        accumulate_means(a1.y, b1.y, inv, acc);
        accumulate_means(a1.z, b1.z, inv, acc);
        accumulate_means(a1.w, b1.w, inv, acc);
      }
    }
  } else {
    const uint32_t* p1 = reinterpret_cast<const uint32_t*>(p0);
    const uint32_t* c1 = reinterpret_cast<const uint32_t*>(c0);
    for (long long i = first; i < pixels; i += step) accumulate_means(__ldg(p1 + i), __ldg(c1 + i), inv, acc);
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
  // an unchanged pixel's terms with the global shift removed: |0 - d| summed and / 3, |0 - luma|
  float rgb_still;
  float luma_still;
};

// The stream's frame means from the block partials: warp 0 sums them (lane l takes partials
// l, l + 32, ...; a fixed xor tree combines the lanes) and shares them through `sh` (the
// caller synchronises).  The reference divides its f32 sums by `pixels as f32` (:1097-1100).
__device__ __forceinline__ void load_means(const double* mean_partials, long long s, long long pixels, Means* sh) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const double* part = mean_partials + s * kStatBlocks * kMeanParts;
  double t[kMeanParts] = {0, 0, 0, 0, 0};
  for (int i = lane; i < kStatBlocks; i += 32)
#pragma unroll
    for (int k = 0; k < kMeanParts; ++k) t[k] += part[i * kMeanParts + k];
#pragma unroll
  for (int k = 0; k < kMeanParts; ++k)
    for (int o = 16; o > 0; o >>= 1) t[k] += __shfl_xor_sync(0xffffffffu, t[k], o);
  if (lane == 0) {
    const float n = (float)pixels;
    sh->d[0] = __fdiv_rn((float)t[0], n);
    sh->d[1] = __fdiv_rn((float)t[1], n);
    sh->d[2] = __fdiv_rn((float)t[2], n);
    sh->luma = __fdiv_rn((float)t[3], n);
    sh->raw = __fdiv_rn((float)t[4], n);
  }
}

// One pixel of the patch pass: the score term without (raw) and with (comp) the global shift
// removed (:1199-1244), and the lighting-residual term (:1102-1113), which is comp's RGB term.
// For an unchanged pixel every delta, the chroma difference and the raw term are exact zeros,
// so the terms reduce to the stream's constants and one quotient (the same values the full
// computation gives).
__device__ __forceinline__ void accumulate_patch(uint32_t pp, uint32_t cp, const float* inv, const Means& m,
                                                 float& acc_raw, float& acc_comp, double& res) {
  if (same_rgb(pp, cp)) {
    const Rgb a = rgb_of(pp, inv);
    const float den = fmaxf(luma(a), 0.10f);
    const float still = fmaxf(m.rgb_still, m.luma_still);
    res += m.rgb_still;
    acc_comp += rel_below(m.luma_still, den, still) ? still : fmaxf(still, rel_term(m.luma_still, den));
    return;
  }
  const Rgb a = rgb_of(pp, inv), b = rgb_of(cp, inv);
  const float dr = __fsub_rn(b.r, a.r), dg = __fsub_rn(b.g, a.g), db = __fsub_rn(b.b, a.b);
  const float rgb_raw = div3_rn(__fadd_rn(__fadd_rn(fabsf(dr), fabsf(dg)), fabsf(db)));
  const float er = fabsf(__fsub_rn(dr, m.d[0])), eg = fabsf(__fsub_rn(dg, m.d[1])), eb = fabsf(__fsub_rn(db, m.d[2]));
  const float rgb_comp = div3_rn(__fadd_rn(__fadd_rn(er, eg), eb));
  res += rgb_comp;
  const float pl = luma(a), cl = luma(b);
  const float ld = __fsub_rn(cl, pl);
  const float luma_raw = fabsf(ld), luma_comp = fabsf(__fsub_rn(ld, m.luma));
  const float den = fmaxf(fmaxf(pl, cl), 0.10f);
  const float m_raw = fmaxf(rgb_raw, luma_raw), m_comp = fmaxf(rgb_comp, luma_comp);
  float s_raw = rel_below(luma_raw, den, m_raw) ? m_raw : fmaxf(m_raw, rel_term(luma_raw, den));
  float s_comp = rel_below(luma_comp, den, m_comp) ? m_comp : fmaxf(m_comp, rel_term(luma_comp, den));
  const ChromaDen cd = chroma_den(a, b);
  if (!chroma_below(a, b, cd, fminf(m_raw, m_comp))) {
    const float chroma = __fmul_rn(chroma_diff(a, b, cd), 0.5f);
    s_raw = fmaxf(s_raw, chroma);
    s_comp = fmaxf(s_comp, chroma);
  }
  acc_raw += s_raw;
  acc_comp += s_comp;
}

// The patch score without the shift alone (:1199-1244), for streams that cannot compensate;
// an unchanged pixel's term is an exact zero.
__device__ __forceinline__ void accumulate_raw(uint32_t pp, uint32_t cp, const float* inv, float& acc_raw) {
  if (same_rgb(pp, cp)) return;
  const Rgb a = rgb_of(pp, inv), b = rgb_of(cp, inv);
  const float dr = __fsub_rn(b.r, a.r), dg = __fsub_rn(b.g, a.g), db = __fsub_rn(b.b, a.b);
  const float rgb_raw = div3_rn(__fadd_rn(__fadd_rn(fabsf(dr), fabsf(dg)), fabsf(db)));
  const float pl = luma(a), cl = luma(b);
  const float luma_raw = fabsf(__fsub_rn(cl, pl));
  const float den = fmaxf(fmaxf(pl, cl), 0.10f);
  const float m_raw = fmaxf(rgb_raw, luma_raw);
  float s_raw = rel_below(luma_raw, den, m_raw) ? m_raw : fmaxf(m_raw, rel_term(luma_raw, den));
  const ChromaDen cd = chroma_den(a, b);
  if (!chroma_below(a, b, cd, m_raw)) s_raw = fmaxf(s_raw, __fmul_rn(chroma_diff(a, b, cd), 0.5f));
  acc_raw += s_raw;
}

// True when the frame means alone rule out the compensation (:1114-1123): it needs raw > 1e-4
// and residual <= 0.35 raw, while every pixel's residual term is at least its raw term minus
// the shift term s = (|dR| + |dG| + |dB|) / 3 of the means, so residual >= raw - s up to a few
// ulps; s < 0.6 raw therefore leaves the residual above 0.35 raw with a wide margin.  Only used
// when the caller does not ask for the frame statistics (which report the residual).
__device__ __forceinline__ bool no_compensation(const Means& m, float shift) {
  return m.raw <= 1.0e-4f || shift < __fmul_rn(0.6f, m.raw);
}

// Pass 2: one warp per patch, the blocks of a stream striding over its patches.  Writes both
// scores of each patch (raw into `scores`, comp into `scores_comp`) and the block's partial of
// the lighting residual over its patches' pixels (:1102-1113; together the partials cover the
// pixel rows of the grid, `rest_rows` more rows below it are added by the last block).  vec:
// 16-byte aligned rows and a patch width that is a multiple of 4, four pixels per load.  A
// stream the means rule out from compensating (and no stats wanted) gets the raw scores only.
__global__ void __launch_bounds__(kRgbaThreads)
    rgba_patch_kernel(const uint8_t* __restrict__ prev, const uint8_t* __restrict__ cur, long long pixels,
                      int width, int patch, int gh, int gw, int vec, int rest_rows, int want_stats,
                      const double* __restrict__ mean_partials, float* __restrict__ scores,
                      float* __restrict__ scores_comp, double* __restrict__ residual_partials) {
  __shared__ float inv[256];
  __shared__ double red[kRgbaThreads / 32];
  __shared__ Means sh;
  build_u8_table(inv);
  const long long s = blockIdx.y;
  load_means(mean_partials, s, pixels, &sh);
  __syncthreads();
  Means m = sh;
  m.rgb_still = div3_rn(__fadd_rn(__fadd_rn(fabsf(m.d[0]), fabsf(m.d[1])), fabsf(m.d[2])));
  m.luma_still = fabsf(m.luma);
  const bool raw_only = !want_stats && no_compensation(m, m.rgb_still);  // the same for the block
  const int lane = threadIdx.x & 31;
  const long long n_patches = (long long)gh * gw;
  const uint8_t* p0 = prev + s * pixels * 4;
  const uint8_t* c0 = cur + s * pixels * 4;
  double res = 0.0;
  for (long long patch_id = (long long)blockIdx.x * kPatchWarps + (threadIdx.x >> 5); patch_id < n_patches;
       patch_id += (long long)gridDim.x * kPatchWarps) {
    const int row = (int)(patch_id / gw), col = (int)(patch_id % gw);
    float acc_raw = 0.0f, acc_comp = 0.0f;
    if (vec) {
      // quads q and q + 32 of the lane loaded together (a 16x16 patch has 64 quads), then
      // consumed in the order q, q + 32 as one at a time would
      const int qpr = patch >> 2;  // 4-pixel groups per patch row
      const int nq = patch * qpr;
      for (int q = lane; q < nq; q += 64) {
        const bool second = q + 32 < nq;
        const int y0 = row * patch + q / qpr, x0 = col * patch + 4 * (q % qpr);
        const long long off0 = ((long long)y0 * width + x0) * 4;
        const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(p0 + off0));
        const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(c0 + off0));
        uint4 a1 = a0, b1 = b0;
        if (second) {
          const int y1 = row * patch + (q + 32) / qpr, x1 = col * patch + 4 * ((q + 32) % qpr);
          const long long off1 = ((long long)y1 * width + x1) * 4;
          a1 = __ldg(reinterpret_cast<const uint4*>(p0 + off1));
          b1 = __ldg(reinterpret_cast<const uint4*>(c0 + off1));
        }
        if (raw_only) {
          accumulate_raw(a0.x, b0.x, inv, acc_raw);
          accumulate_raw(a0.y, b0.y, inv, acc_raw);
          accumulate_raw(a0.z, b0.z, inv, acc_raw);
          accumulate_raw(a0.w, b0.w, inv, acc_raw);
          if (second) {
            accumulate_raw(a1.x, b1.x, inv, acc_raw);
            accumulate_raw(a1.y, b1.y, inv, acc_raw);
            accumulate_raw(a1.z, b1.z, inv, acc_raw);
            accumulate_raw(a1.w, b1.w, inv, acc_raw);
          }
        } else {
          accumulate_patch(a0.x, b0.x, inv, m, acc_raw, acc_comp, res);
          accumulate_patch(a0.y, b0.y, inv, m, acc_raw, acc_comp, res);
          accumulate_patch(a0.z, b0.z, inv, m, acc_raw, acc_comp, res);
          accumulate_patch(a0.w, b0.w, inv, m, acc_raw, acc_comp, res);
          if (second) {
            accumulate_patch(a1.x, b1.x, inv, m, acc_raw, acc_comp, res);
            accumulate_patch(a1.y, b1.y, inv, m, acc_raw, acc_comp, res);
            accumulate_patch(a1.z, b1.z, inv, m, acc_raw, acc_comp, res);
            accumulate_patch(a1.w, b1.w, inv, m, acc_raw, acc_comp, res);
          }
        }
      }
    } else {
      for (int k = lane; k < patch * patch; k += 32) {
        const int y = row * patch + k / patch, x = col * patch + k % patch;
        const long long off = ((long long)y * width + x) * 4;
        const uint32_t a = __ldg(reinterpret_cast<const uint32_t*>(p0 + off));
        const uint32_t b = __ldg(reinterpret_cast<const uint32_t*>(c0 + off));
        if (raw_only)
          accumulate_raw(a, b, inv, acc_raw);
        else
          accumulate_patch(a, b, inv, m, acc_raw, acc_comp, res);
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      acc_raw += __shfl_xor_sync(0xffffffffu, acc_raw, o);
      acc_comp += __shfl_xor_sync(0xffffffffu, acc_comp, o);
    }
    if (lane == 0) {
      const float area = (float)(patch * patch);
      scores[s * n_patches + patch_id] = __fdiv_rn(acc_raw, area);
      if (!raw_only) scores_comp[s * n_patches + patch_id] = __fdiv_rn(acc_comp, area);
    }
  }
  if (raw_only) return;
  // pixel rows below the grid (a frame taller than gh * patch) count toward the residual only
  if (rest_rows > 0 && blockIdx.x == gridDim.x - 1) {
    const uint32_t* p1 = reinterpret_cast<const uint32_t*>(p0) + (long long)gh * patch * width;
    const uint32_t* c1 = reinterpret_cast<const uint32_t*>(c0) + (long long)gh * patch * width;
    for (long long i = threadIdx.x; i < (long long)rest_rows * width; i += kRgbaThreads) {
      const Rgb a = rgb_of(__ldg(p1 + i), inv), b = rgb_of(__ldg(c1 + i), inv);
      const float er = fabsf(__fsub_rn(__fsub_rn(b.r, a.r), m.d[0]));
      const float eg = fabsf(__fsub_rn(__fsub_rn(b.g, a.g), m.d[1]));
      const float eb = fabsf(__fsub_rn(__fsub_rn(b.b, a.b), m.d[2]));
      res += div3_rn(__fadd_rn(__fadd_rn(er, eg), eb));
    }
  }
  const double t = block_sum(res, red);
  if (threadIdx.x == 0) residual_partials[s * gridDim.x + blockIdx.x] = t;
}

// Pass 3: per stream, the lighting residual from the patch blocks' partials (fixed order), the
// compensation decision (:1114-1123), the stats, and the compensated scores where it applies.
__global__ void __launch_bounds__(kRgbaThreads)
    rgba_finalize_kernel(long long pixels, long long n_patches, int patch_blocks,
                         const double* __restrict__ mean_partials, const double* __restrict__ residual_partials,
                         const float* __restrict__ scores_comp, float* __restrict__ scores,
                         bjf_rgba_frame_stats* __restrict__ stats_out) {
  __shared__ double red[kRgbaThreads / 32];
  __shared__ Means sh;
  const long long s = blockIdx.y;
  load_means(mean_partials, s, pixels, &sh);
  __syncthreads();
  const Means m = sh;
  const float shift = div3_rn(__fadd_rn(__fadd_rn(fabsf(m.d[0]), fabsf(m.d[1])), fabsf(m.d[2])));
  if (!stats_out && no_compensation(m, shift)) return;  // the patch pass wrote the raw scores only
  double part = 0.0;
  for (int i = threadIdx.x; i < patch_blocks; i += kRgbaThreads) part += residual_partials[s * patch_blocks + i];
  const double total = block_sum(part, red);
  const float residual = __fdiv_rn((float)total, (float)pixels);
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
  if (!comp) return;
  for (long long i = (long long)blockIdx.x * kRgbaThreads + threadIdx.x; i < n_patches;
       i += (long long)gridDim.x * kRgbaThreads)
    scores[s * n_patches + i] = scores_comp[s * n_patches + i];
}

struct Workspace {
  size_t residual, comp, bytes;
  int64_t patch_blocks;  // patch-pass blocks per stream
};

// [S, 64, 5] f64 mean partials | [S, patch blocks] f64 residual partials | [S, patches] f32
// compensated scores, each 256-byte aligned.  The patch-pass grid is a function of the sizes
// only, so the residual's summation order is too.
Workspace workspace_layout(int64_t streams, int64_t n_patches) {
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  Workspace w;
  // at most one wave of kPatchBlocksTarget blocks over all streams (rounding up left a second
  // wave of a few blocks)
  w.patch_blocks = std::max<int64_t>(
      1, std::min<int64_t>(ceil_div(n_patches, kPatchWarps), kPatchBlocksTarget / streams));
  w.residual = up(sizeof(double) * (size_t)streams * kStatBlocks * kMeanParts);
  w.comp = up(w.residual + sizeof(double) * (size_t)streams * (size_t)w.patch_blocks);
  w.bytes = w.comp + sizeof(float) * (size_t)streams * (size_t)n_patches;
  return w;
}

bool grid_ok(int64_t streams, const int64_t grid[3]) {
  return streams > 0 && streams <= 65535 && grid && grid[1] > 0 && grid[2] > 0 && grid[1] <= (1 << 20) &&
         grid[2] <= (1 << 20) && grid[1] * grid[2] <= (int64_t(1) << 30);
}

}  // namespace
}  // namespace bjf

using namespace bjf;

extern "C" size_t bjf_rgba_patch_diff_workspace_bytes(int64_t streams, const int64_t grid[3]) {
  if (!grid_ok(streams, grid)) return 0;
  return workspace_layout(streams, grid[1] * grid[2]).bytes;
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
  const int64_t n_patches = grid[1] * grid[2];
  if (n_patches > (int64_t(1) << 30)) return fail(BJF_ERR_UNSUPPORTED, "RGBA patch-diff grid exceeds the supported size");
  const Workspace w = workspace_layout(streams, n_patches);
  if (workspace_bytes < w.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "RGBA patch-diff workspace must be 256-byte aligned and hold " + std::to_string(w.bytes) + " bytes");
  const long long pixels = (long long)width * height;
  char* ws = static_cast<char*>(workspace);
  double* means = reinterpret_cast<double*>(ws);
  double* resid = reinterpret_cast<double*>(ws + w.residual);
  float* comp = reinterpret_cast<float*>(ws + w.comp);
  const bool aligned = ((reinterpret_cast<uintptr_t>(prev) | reinterpret_cast<uintptr_t>(current)) & 15) == 0;
  cudaStream_t st = as_cuda(stream);
  rgba_means_kernel<<<dim3(kStatBlocks, (unsigned)streams), kRgbaThreads, 0, st>>>(
      prev, current, pixels, aligned && pixels % 4 == 0 ? 1 : 0, means);
  bjf_status rc = check_launch("RGBA lighting means launch");
  if (rc) return rc;
  const int rest_rows = (int)(height - grid[1] * patch_size);
  rgba_patch_kernel<<<dim3((unsigned)w.patch_blocks, (unsigned)streams), kRgbaThreads, 0, st>>>(
      prev, current, pixels, (int)width, (int)patch_size, (int)grid[1], (int)grid[2],
      aligned && width % 4 == 0 && patch_size % 4 == 0 ? 1 : 0, rest_rows, stats_out ? 1 : 0, means, scores,
      comp, resid);
  rc = check_launch("RGBA patch-diff scores launch");
  if (rc) return rc;
  const unsigned fin_blocks = (unsigned)std::min<int64_t>(64, ceil_div(n_patches, 4 * kRgbaThreads));
  rgba_finalize_kernel<<<dim3(fin_blocks, (unsigned)streams), kRgbaThreads, 0, st>>>(
      pixels, n_patches, (int)w.patch_blocks, means, resid, comp, scores, stats_out);
  return check_launch("RGBA patch-diff finalize launch");
}
