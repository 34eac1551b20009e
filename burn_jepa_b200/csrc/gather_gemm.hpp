// gather_gemm.hpp -- internal interface of the sparse-patchify gather-GEMM.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bjf.h"
#include "runtime.hpp"

namespace bjf {

// Input video and token-grid geometry of one sparse patchify call.
struct GatherGeometry {
  int C, T, H, W;      // channels, frames, height, width of each batch element
  int kt, ph, pw;      // tubelet and patch sizes
  int batch;           // batch elements in the input
  int depth, gh, gw;   // token grid
  int K, D;            // C*kt*ph*pw and output channels
  int num_kb;          // K / 64 (tensor-core path)
  int is_bf16;
  uint64_t wait_ns;    // limit of every bounded pipeline wait (bjf_set_bounded_wait)
  int stall;           // 1: the single-CTA kernel's MMA thread waits on a barrier nothing completes
  // Frame ring (a two-frame clip of depth 1 read from slots slot0, slot1 of Ts stored frames);
  // ring = 0: contiguous frames, Ts = T (set by launch_gather_gemm)
  int ring, Ts, slot0, slot1;
  // Split K (pair kernel, plain epilogue): each 256 x bn tile is ksplit units of num_kb / ksplit
  // K blocks whose f32 partial sums go to ep.out + unit's split x ep.split_stride bytes, summed
  // by a reduce launch.  0 or 1: none.
  int ksplit;
};

enum { kEpiloguePlain = 0, kEpilogueScatter = 1 };

// Where the projected rows go.
//  plain:   out[m, :] with row stride ldo elements
//  scatter: out[(b * dense_tokens + token_index(t, r, col)), :] with row stride ldo, plus
//           observed[slot] = 1, age[slot] = 0 (a fused token-cache write)
struct EpilogueArgs {
  void* out;
  int32_t out_dtype;
  int out_elem_bytes;
  int64_t ldo;
  int mode;
  int64_t dense_tokens;
  float* observed;
  float* age;
  const float* bias;
  // Encoder input (plain mode): out += position_table[token index of the row, :] (row stride
  // pos_ld), then += modality_embed[:], after the bias and in that order.  Null when unused.
  const float* position_table;
  int64_t pos_ld;
  const float* modality_embed;
  int64_t split_stride;  // bytes between the split-K partial outputs (GatherGeometry::ksplit)
};

// Where the gathered rows come from: either explicit coords rows (b, t, r, col), or the
// per-stream token indices of a selection with the first row of each stream (the plan the
// coords form describes, without materialising it): row m belongs to the stream s with
// offsets[s] <= m < offsets[s + 1] and is its token indices[s, m - offsets[s]].
constexpr int kMaxRowStreams = 4096;
struct RowSource {
  const int4* coords;      // [rows] or null
  const int32_t* indices;  // [streams, index_stride] when coords is null
  const int32_t* counts;   // [streams] rows of each stream (clamped to 0..index_stride); the
                           // kernel scans them into the stream row offsets
  int index_stride;
  int streams;             // <= kMaxRowStreams
};

inline RowSource coords_rows(const int4* coords) { return RowSource{coords, nullptr, nullptr, 0, 0}; }

// Enqueues out = gather(input, rows) x weight^T + bias.  `rows_dev` (device, nullable)
// caps the row count at run time; `rows_cap` bounds the grid.
bjf_status launch_gather_gemm(const DeviceInfo& dev, const void* input, int32_t in_dt,
                              const void* weight, int32_t w_dt, const GatherGeometry& g,
                              const RowSource& rows, const int32_t* rows_dev, int64_t rows_cap,
                              const EpilogueArgs& ep, cudaStream_t st, bool pdl = false,
                              bool may_allocate = true);

bool sm100_path_supported(const DeviceInfo& dev, const GatherGeometry& g, int32_t in_dt,
                          int32_t w_dt, const void* input, const void* weight);

}  // namespace bjf
