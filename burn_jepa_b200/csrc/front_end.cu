// front_end.cu -- one step of the sparse front end for S independent streams,
// fully on the device:
//
//   1. patch-diff scores          [S, N] f32                  (memory-bound pass over the clips)
//   2. selection + cache aging    indices [S, N], counts [S]  (one CTA per stream; the
//                                 AssignLatest aging age += observed runs in the same launch)
//   3. gather-GEMM                tcgen05 tiles over the concatenated active rows: each CTA
//                                 scans the counts into the first row of every stream (the
//                                 plan) and reads each row's token from the indices; the
//                                 epilogue adds the bias and writes each row straight into
//                                 its stream's token cache slot, setting observed = 1, age = 0
//
// The three kernels are chained with programmatic dependent launch: each waits for its
// predecessor only where it reads that predecessor's output, and the patch-diff pass of the
// next frame runs alongside this frame's GEMM (HBM-bound next to tensor-bound work).
//
// This is the composition the reference pipeline performs per stream and per frame
// (patch_diff_context_mask -> SparsePatchifyPlan::new -> sparse_patchify3d_forward_cuda ->
// update_tokens_tiled_assign_cuda_raw, src/nodes.rs:411-456, src/sparse_patchify.rs:236-269,
// src/model.rs:1273-1328, src/feature_memory.rs:616-645), with no host round trip: the
// mask never leaves the device and the features never exist outside the cache.  Row
// counts are only known on the device, so the GEMM grid is sized for the capacity and
// surplus tiles exit at once.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "gather_gemm.hpp"
#include "patch_diff.hpp"
#include "runtime.hpp"
#include "status.hpp"

namespace bjf {
namespace {

struct Workspace {
  size_t scores, indices, counts, bytes;
};

Workspace layout(int64_t S, int64_t N) {
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  Workspace w{};
  size_t off = 0;
  w.scores = off;
  off = up(off + sizeof(float) * S * N);
  w.indices = off;
  off = up(off + sizeof(int32_t) * S * N);
  w.counts = off;
  off = up(off + sizeof(int32_t) * S);
  w.bytes = off;
  return w;
}

bjf_status validate(const bjf_front_end_desc* d, int64_t& N) {
  if (!d) return fail(BJF_ERR_INVALID_ARGUMENT, "front-end descriptor must not be null");
  const int64_t v[9] = {d->streams, d->channels, d->frames, d->height, d->width,
                        d->tubelet_size, d->patch_size, d->embed_dim, 1};
  for (int64_t x : v)
    if (x <= 0 || x > (1 << 30)) return fail(BJF_ERR_INVALID_ARGUMENT, "front-end sizes must be positive");
  if (d->frames % d->tubelet_size || d->height % d->patch_size || d->width % d->patch_size)
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "patch-diff sparsity requires frames/height/width divisible by tubelet and patch sizes");
  N = (d->frames / d->tubelet_size) * (d->height / d->patch_size) * (d->width / d->patch_size);
  if (d->streams > 4096) return fail(BJF_ERR_UNSUPPORTED, "the front end supports up to 4096 streams per call");
  if (d->streams * N > INT32_MAX) return fail(BJF_ERR_UNSUPPORTED, "streams x tokens exceeds 2^31-1");
  if (dtype_size(d->cache_dtype) == 0 || d->cache_dtype == BJF_DTYPE_I32)
    return fail(BJF_ERR_INVALID_ARGUMENT, "cache dtype must be f32, f16 or bf16");
  return BJF_OK;
}

}  // namespace
}  // namespace bjf

using namespace bjf;

extern "C" size_t bjf_front_end_workspace_bytes(const bjf_front_end_desc* d) {
  int64_t N = 0;
  if (validate(d, N)) return 0;
  return layout(d->streams, N).bytes;
}

namespace {

// One step over S streams whose clips are `video` (contiguous [S, C, T, H, W]) or, with `ring`,
// the two slots of a frame ring [S, C, R, H, W].
bjf_status front_end_step(const bjf_front_end_desc* d, const void* video, const FrameRing* ring, const void* weight,
                          const float* bias, void* caches, float* observed, float* age_frames, int32_t age_observed,
                          void* workspace, size_t workspace_bytes, int32_t* counts_out, bjf_stream_t stream) {
  int64_t N = 0;
  bjf_status rc = validate(d, N);
  if (rc) return rc;
  const int64_t S = d->streams;
  const Workspace w = layout(S, N);
  if (!workspace || workspace_bytes < w.bytes)
    return fail(BJF_ERR_INVALID_ARGUMENT, "front-end workspace too small: need " + std::to_string(w.bytes) + " bytes");
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(BJF_ERR_INVALID_ARGUMENT, "front-end workspace must be 256-byte aligned");
  if (!video || !weight || !caches || !observed || !age_frames)
    return fail(BJF_ERR_INVALID_ARGUMENT, "front-end buffers must not be null");
  const int64_t grid[3] = {d->frames / d->tubelet_size, d->height / d->patch_size, d->width / d->patch_size};
  SelectParams sel;
  rc = resolve_select(&d->mask, grid, sel);
  if (rc) return rc;
  const DeviceInfo* dev = nullptr;
  rc = current_device(&dev);
  if (rc) return rc;

  char* ws = static_cast<char*>(workspace);
  float* scores = reinterpret_cast<float*>(ws + w.scores);
  int32_t* indices = reinterpret_cast<int32_t*>(ws + w.indices);
  int32_t* counts = counts_out ? counts_out : reinterpret_cast<int32_t*>(ws + w.counts);
  cudaStream_t st = as_cuda(stream);

  const int64_t vd[5] = {1, d->channels, d->frames, d->height, d->width};
  // the cache aging rides at the end of the scores pass when it can, else in the selection
  const ScoresAging aging{age_frames, observed, (long long)(S * N)};
  bool aged = false;
  rc = launch_scores(video, d->video_dtype, vd, S, d->tubelet_size, d->patch_size, scores, st, true, ring,
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
  if (ring) {
    g.ring = 1;
    g.Ts = ring->storage_frames;
    g.slot0 = ring->slot0;
    g.slot1 = ring->slot1;
  }
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
  // the GEMM scans the per-stream counts into its row offsets
  const RowSource rows{nullptr, indices, counts, (int)N, (int)S};
  return launch_gather_gemm(*dev, video, d->video_dtype, weight, d->weight_dtype, g, rows, nullptr, S * N, ep, st,
                            true);
}

}  // namespace

extern "C" bjf_status bjf_front_end_step(const bjf_front_end_desc* d, const void* video, const void* weight,
                                         const float* bias, void* caches, float* observed, float* age_frames,
                                         int32_t age_observed, void* workspace, size_t workspace_bytes,
                                         int32_t* counts_out, bjf_stream_t stream) {
  return front_end_step(d, video, nullptr, weight, bias, caches, observed, age_frames, age_observed, workspace,
                        workspace_bytes, counts_out, stream);
}

extern "C" bjf_status bjf_front_end_step_ring(const bjf_front_end_desc* d, const void* frame_ring, int32_t ring_slots,
                                              int32_t prev_slot, int32_t cur_slot, const void* weight,
                                              const float* bias, void* caches, float* observed, float* age_frames,
                                              int32_t age_observed, void* workspace, size_t workspace_bytes,
                                              int32_t* counts_out, bjf_stream_t stream) {
  if (!d) return fail(BJF_ERR_INVALID_ARGUMENT, "front-end descriptor must not be null");
  if (d->frames != 2 || d->tubelet_size != 2)
    return fail(BJF_ERR_INVALID_ARGUMENT, "the frame-ring step needs frames = 2 and tubelet_size = 2");
  if (ring_slots < 2 || ring_slots > 64)
    return fail(BJF_ERR_INVALID_ARGUMENT, "frame ring must hold 2 to 64 frames per stream");
  if (prev_slot < 0 || prev_slot >= ring_slots || cur_slot < 0 || cur_slot >= ring_slots || prev_slot == cur_slot)
    return fail(BJF_ERR_INVALID_ARGUMENT, "frame ring slots must be distinct and inside the ring");
  const FrameRing ring{ring_slots, 1, prev_slot, cur_slot};
  return front_end_step(d, frame_ring, &ring, weight, bias, caches, observed, age_frames, age_observed, workspace,
                        workspace_bytes, counts_out, stream);
}

extern "C" bjf_status bjf_frame_ring_upload(const bjf_front_end_desc* d, const void* host_frame, void* frame_ring,
                                            int32_t ring_slots, int32_t slot, int64_t stream_begin,
                                            int64_t stream_end, bjf_stream_t stream) {
  if (!d) return fail(BJF_ERR_INVALID_ARGUMENT, "front-end descriptor must not be null");
  if (ring_slots < 2 || ring_slots > 64)
    return fail(BJF_ERR_INVALID_ARGUMENT, "frame ring must hold 2 to 64 frames per stream");
  if (slot < 0 || slot >= ring_slots) return fail(BJF_ERR_INVALID_ARGUMENT, "frame ring slot outside the ring");
  if (stream_begin < 0 || stream_end > d->streams || stream_begin > stream_end)
    return fail(BJF_ERR_INVALID_ARGUMENT, "frame ring upload streams outside the descriptor's");
  const size_t esz = dtype_size(d->video_dtype);
  if (esz == 0 || d->video_dtype == BJF_DTYPE_I32) return fail(BJF_ERR_INVALID_ARGUMENT, "video dtype must be f32, f16 or bf16");
  if (d->channels <= 0 || d->height <= 0 || d->width <= 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "front-end descriptor dims must be positive");
  if (!host_frame || !frame_ring) return fail(BJF_ERR_INVALID_ARGUMENT, "buffers must not be null");
  if (stream_begin == stream_end) return BJF_OK;
  // one [H, W] plane per (stream, channel): a 2-D copy of S C rows, one plane each, from a
  // dense source to the ring's slot (row pitch ring_slots planes)
  const size_t plane = (size_t)d->height * (size_t)d->width * esz;
  const size_t rows = (size_t)(stream_end - stream_begin) * (size_t)d->channels;
  const char* src = static_cast<const char*>(host_frame) + (size_t)stream_begin * d->channels * plane;
  char* dst = static_cast<char*>(frame_ring) + ((size_t)stream_begin * d->channels * ring_slots + slot) * plane;
  const cudaError_t e = cudaMemcpy2DAsync(dst, plane * ring_slots, src, plane, plane, rows, cudaMemcpyHostToDevice,
                                          as_cuda(stream));
  return e == cudaSuccess ? BJF_OK : cuda_status(e, "frame ring upload");
}
