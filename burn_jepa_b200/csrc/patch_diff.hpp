// patch_diff.hpp -- internal interface of the patch-diff mask kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bjf.h"

namespace bjf {

struct SelectParams {
  float threshold;
  int cap;          // threshold-phase cap (grid.len() with allow_full_context)
  int fill_target;  // context_tokens (fill_to_context_tokens) or min_context_tokens
  int dilation;
  int depth, gh, gw, n;
  // Optional token-cache aging fused into the selection launch (one CTA per stream):
  // age[s, :] += observed[s, :] (the first half of the AssignLatest update,
  // src/sparse_feature_memory.rs:46-52).  Null when not requested.
  float* age;
  const float* observed;
};

// Resolves the reference's context budget arithmetic (src/nodes.rs:463-498, 516-520).
bjf_status resolve_select(const bjf_patch_diff_config* cfg, const int64_t* grid, SelectParams& p);

// One CTA per stream: selection (and optional aging) -> indices [streams, n], counts [streams].
bjf_status launch_select(const float* scores, int64_t streams, const SelectParams& p, int32_t* indices,
                         int32_t* counts, cudaStream_t st, bool pdl = false);

// Where the frames of a clip live: contiguous [.., T, H, W] (storage_frames = T, frame(f) = f), or
// a frame ring [.., R, H, W] holding R frames per channel of which a two-frame clip uses slots
// (slot0, slot1) in that order (storage_frames = R).
struct FrameRing {
  int storage_frames;
  int ring;  // 0: contiguous
  int slot0, slot1;
  __host__ __device__ __forceinline__ int frame(int f) const { return ring ? (f == 0 ? slot0 : slot1) : f; }
  static FrameRing contiguous(int frames) { return FrameRing{frames, 0, 0, 1}; }
};

// Per-tubelet mean |delta| scores for `streams` videos [B, C, T, H, W] -> [streams, N]; with a
// ring (T = 2 only), the frames are read from its slots.
// With `aging` (age[i] += observed[i] over `aging_len` floats, the first half of the AssignLatest
// update), the vector pass does the aging after its closing wait for the kernel before it (the
// previous frame's GEMM, which writes those arrays) and sets *aged; otherwise *aged = false and
// the caller ages elsewhere.
struct ScoresAging {
  float* age;
  const float* observed;
  long long len;
};
bjf_status launch_scores(const void* video, int32_t dtype, const int64_t* video_dims, int64_t streams,
                         int64_t tubelet_size, int64_t patch_size, float* scores, cudaStream_t st,
                         bool pdl = false, const FrameRing* ring = nullptr, const ScoresAging* aging = nullptr,
                         bool* aged = nullptr);

// Device plan (coords rows) from per-stream mask indices; see bjf_sparse_patchify_plan_coords.
bjf_status launch_plan(const int32_t* indices, int64_t index_stride, const int32_t* counts, int64_t mask_rows,
                       int64_t batch, const int64_t grid[3], int32_t* coords, int64_t coords_capacity,
                       int32_t* total_rows, cudaStream_t st, bool pdl = false);

}  // namespace bjf
