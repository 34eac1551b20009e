/*
 * bjf.h -- C ABI of the B200 (sm_100a) sparse front end for burn_jepa.
 *
 * The three steps of burn_jepa's sparse video front end, as stateless C entry
 * points over caller-owned device memory:
 *
 *   1. patch-diff mask   per-tubelet mean |frame delta| -> threshold policy ->
 *                        ascending active token indices
 *   2. sparse patchify   gather the active kt x ph x pw tubelets and project them
 *                        through the Conv3d patch-embed weight (+ bias)
 *   3. token-cache write scatter the new token features into the persistent
 *                        [B, N, D] token cache and update observed / age metadata
 *
 * Each entry point names the reference (mosure/burn_jepa 0.21.0) interface it
 * replaces.  Conventions shared by every function:
 *   - All pointers are device pointers unless the parameter says "host".
 *   - Work is enqueued on `stream` (NULL = legacy default stream); nothing
 *     synchronises the host.  Inputs must stay valid until the work completes.
 *   - Return value: 0 = success; negative = invalid argument (nothing was
 *     launched; the message is available from bjf_get_last_error_string on the
 *     calling thread); positive = CUDA launch/runtime error.
 *   - Shapes are passed as the tensor dims the caller already holds (Rust:
 *     `tensor.dims()`), so the library can return the reference's own shape
 *     error messages.  Tensors are contiguous row-major.
 *   - Token indices and coordinates are int32 (the reference's Int element on
 *     the Cuda<f32, i32> backend).
 *   - Functions are thread-safe; per-device state is created lazily.
 */
#ifndef BJF_H
#define BJF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 2: bjf_rgba_patch_diff_workspace_bytes takes the token grid.
 * 3: bjf_set_bounded_wait, bjf_front_end_step_ring.
 * 4: the patch-diff refresh state on the device (bjf_viewer_patch_diff_refresh_*),
 *    bjf_frame_ring_upload. */
#define BJF_ABI_VERSION 4

#if defined(__GNUC__)
#define BJF_API __attribute__((visibility("default")))
#else
#define BJF_API
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* bjf_stream_t;

typedef int32_t bjf_status;
enum {
  BJF_OK = 0,
  BJF_ERR_INVALID_ARGUMENT = -1, /* shape / value error (message set) */
  BJF_ERR_UNSUPPORTED = -2,      /* valid request this build does not serve (message set) */
  BJF_ERR_CUDA = 1               /* CUDA error (message set) */
};

typedef enum bjf_dtype {
  BJF_DTYPE_F32 = 0,
  BJF_DTYPE_F16 = 1,
  BJF_DTYPE_BF16 = 2,
  BJF_DTYPE_I32 = 3
} bjf_dtype;

/* burn_flex_gmm::SparsePatchify3dConfig (fields as the reference fills them,
 * src/model.rs:1297-1306).  All fields must be positive. */
typedef struct bjf_patchify_config {
  int64_t in_channels;
  int64_t out_channels;
  int64_t frames;
  int64_t height;
  int64_t width;
  int64_t tubelet_size;
  int64_t patch_h;
  int64_t patch_w;
} bjf_patchify_config;

/* SparseJepaPatchDiffSparsityConfig (src/nodes.rs:97-157). */
typedef struct bjf_patch_diff_config {
  float threshold;            /* finite, >= 0 */
  int64_t context_tokens;     /* cap (or budget) on selected tokens */
  int64_t target_tokens;      /* carried for parity; the mask does not use it */
  int64_t dilation;           /* spatial dilation radius in tokens */
  int64_t min_context_tokens; /* adaptive fill target */
  int32_t fill_to_context_tokens;
  int32_t allow_full_context;
} bjf_patch_diff_config;

/* ABI version of the loaded library (BJF_ABI_VERSION it was built with). */
BJF_API int32_t bjf_abi_version(void);

/* Copies the message of the last failing call made on this thread into `buf`
 * (NUL-terminated, truncated to `len`).  Returns the length of the full message. */
BJF_API size_t bjf_get_last_error_string(char* buf, size_t len);

/* Synchronises `stream` and reports whether any kernel of this library on the
 * current device gave up on a bounded wait since the last check (*flag_out = 1;
 * the flag is then cleared).  Kernels never spin forever: a pipeline wait that
 * exceeds its time limit records this flag, releases its resources and returns.
 * Covers the workspace entry points and bjf_front_end_step_no_alloc alike; the
 * check itself allocates nothing. */
BJF_API bjf_status bjf_device_error_check(bjf_stream_t stream, int32_t* flag_out);

/* No counterpart in the reference (its failure handling is host-side): sets the time limit of
 * every bounded pipeline wait in the gather-GEMM kernels for launches enqueued after the call
 * (limit_ns; 0 restores the default of 2 s).  stall = 1 is a test hook for the give-up path:
 * the MMA thread of the single-CTA tensor-core kernel (launches of at most 128 rows) first
 * waits on a barrier that nothing completes, so that wait runs out after limit_ns, the kernel
 * drains its copies, frees its TMEM, returns and sets the flag bjf_device_error_check reports;
 * stall = 0 turns it off.  Process-wide; not meant to change while launches are being
 * enqueued on other threads. */
BJF_API bjf_status bjf_set_bounded_wait(uint64_t limit_ns, int32_t stall);

/* ------------------------------------------------------------------------
 * Step 1: patch-diff mask
 * ---------------------------------------------------------------------- */

/* Replaces `patch_diff_token_scores` (src/nodes.rs:565-619, frame pairs :621-631).
 * video: `streams` independent videos, each [B, C, T, H, W] (dims in video_dims),
 * stored back to back.  scores: [streams, N] f32, N = T/kt * H/P * W/P.  Within a
 * video the batch is summed into one score map, as in the reference. */
BJF_API bjf_status bjf_patch_diff_token_scores(const void* video, bjf_dtype video_dtype,
                                       const int64_t video_dims[5], int64_t streams,
                                       int64_t tubelet_size, int64_t patch_size, float* scores,
                                       bjf_stream_t stream);

/* Replaces `patch_diff_context_mask_from_scores` (src/nodes.rs:458-537) and the
 * top-k fast path `patch_diff_topk_context_mask` (:548-563): the selection runs on
 * the device, with no host sort.  scores: [streams, N] for grid (depth, height,
 * width).  Writes each stream's mask as ascending unique int32 token indices into
 * indices[s * N ...] and its length into counts[s] (device).  Grids up to 32768
 * tokens (16384 with dilation > 0). */
BJF_API bjf_status bjf_patch_diff_context_mask_from_scores(const float* scores, int64_t streams,
                                                   const int64_t grid[3],
                                                   const bjf_patch_diff_config* config,
                                                   int32_t* indices, int32_t* counts,
                                                   bjf_stream_t stream);

/* Replaces `patch_diff_context_mask_from_video` (src/nodes.rs:539-546 -> 411-456):
 * scores then selection.  `grid` must equal the grid of the video shape.  scores
 * ([streams, N] f32) is required: it holds the per-tubelet scores on return. */
BJF_API bjf_status bjf_patch_diff_context_mask(const void* video, bjf_dtype video_dtype,
                                       const int64_t video_dims[5], int64_t streams,
                                       int64_t tubelet_size, int64_t patch_size,
                                       const int64_t grid[3], const bjf_patch_diff_config* config,
                                       float* scores, int32_t* indices, int32_t* counts,
                                       bjf_stream_t stream);

/* ------------------------------------------------------------------------
 * Plans
 * ---------------------------------------------------------------------- */

/* Device-resident `SparsePatchifyPlan::new` / `SparsePatchifyBatchPlan::new`
 * (src/sparse_patchify.rs:236-269, 290-330): token indices -> coords rows
 * (batch, tubelet, row, col), batch-major then mask order.
 * indices: [mask_rows, index_stride] int32; counts: [mask_rows] int32 device
 * lengths, or NULL when every row holds exactly `index_stride` indices.
 * mask_rows == 1: the one mask is repeated for every batch element (uniform plan);
 * mask_rows == batch: row b uses mask row b (batch plan; rows may differ in length,
 * they are concatenated).  coords: [coords_capacity, 4] int32.
 * total_rows (device, nullable) receives the number of rows written. */
BJF_API bjf_status bjf_sparse_patchify_plan_coords(const int32_t* indices, int64_t index_stride,
                                           const int32_t* counts, int64_t mask_rows,
                                           int64_t batch, const int64_t grid[3], int32_t* coords,
                                           int64_t coords_capacity, int32_t* total_rows,
                                           bjf_stream_t stream);

/* ------------------------------------------------------------------------
 * Step 2: sparse patchify (gather-GEMM)
 * ---------------------------------------------------------------------- */

/* Replaces `burn_flex_gmm::cuda::sparse_patchify3d_forward_cuda` (burn_flex_gmm
 * 0.21.2, called at src/model.rs:1140, 1197, 1319 and src/sparse_patchify.rs:184):
 *   out[m, d] = bias[d] + sum_k W[d, k] * x[b, c, t*kt+dt, r*ph+dy, col*pw+dx]
 * with (b, t, r, col) = coords[m], k = ((c*kt + dt)*ph + dy)*pw + dx: Conv3d with
 * stride = kernel evaluated at the selected tubelets.
 * input: [B, C, T, H, W] (dims in input_dims); weight: [D, C, kt, ph, pw];
 * bias: [D] f32 or NULL (zeros, as the reference substitutes at src/model.rs:1307-1318);
 * out: [rows, D].  f16/bf16 input and weight (same dtype) run on the tcgen05 tensor
 * cores with f32 accumulation.  f32 input and weight run there too, each operand split into
 * bf16 high and low parts and three bf16 products per term (a_hi w_hi + a_hi w_lo + a_lo w_hi,
 * dropped terms below 3 * 2^-16 |a w|), when pw and W are multiples of 8, K <= 2730 and both
 * buffers are 16-byte aligned; else on a SIMT f32 kernel.  The split's bf16 copies (1.5x the
 * input's f32 bytes and 1.5x the weight's) come from the library's stream-ordered memory pool
 * and return to it when the call's kernels finish.  Rows whose coords lie outside the input
 * are written as zeros. */
BJF_API bjf_status bjf_sparse_patchify3d_forward(const bjf_patchify_config* config, const void* input,
                                         bjf_dtype input_dtype, const int64_t input_dims[5],
                                         const int32_t* coords, int64_t rows, const void* weight,
                                         bjf_dtype weight_dtype, const int64_t weight_dims[5],
                                         const float* bias, void* out, bjf_dtype out_dtype,
                                         bjf_stream_t stream);

/* bjf_sparse_patchify3d_forward producing the encoder's input tokens: after the bias each row
 * adds its token's position embedding, then the modality embedding, in that order
 * (VJepaEncoder::forward_sparse_plan, src/model.rs:690-703, with SparseEncoderPlan's
 * position_embed, :296-319).  position_table: [T/kt * H/ph * W/pw, D] f32 indexed by the row's
 * token index (t * gh * gw + r * gw + col), e.g. get_3d_sincos_pos_embed (src/positional.rs:42-85),
 * or NULL (RoPE models); modality_embed: [D] f32 or NULL.  Rows with out-of-range coords stay
 * zero. */
BJF_API bjf_status bjf_sparse_patchify3d_forward_encoder_input(
    const bjf_patchify_config* config, const void* input, bjf_dtype input_dtype, const int64_t input_dims[5],
    const int32_t* coords, int64_t rows, const void* weight, bjf_dtype weight_dtype, const int64_t weight_dims[5],
    const float* bias, const float* position_table, const float* modality_embed, void* out, bjf_dtype out_dtype,
    bjf_stream_t stream);

/* ------------------------------------------------------------------------
 * Step 3: token-cache write
 * ---------------------------------------------------------------------- */

/* Replaces `sparse_feature_memory_assign_latest_cuda_raw`
 * (src/sparse_feature_memory.rs:296-313 -> 110-267), the kernels behind
 * `InterframeJepaFeatureMemory::update_tokens_tiled_assign_cuda(_raw)`
 * (src/feature_memory.rs:586-645).  In place:
 *   if age_observed: age_frames += observed          (every slot)
 *   features[b, idx[b,s], :] = tokens[b, s, :]; observed = 1; age_frames = 0
 * Indices < 0 or >= N are skipped.  features: [B, N, D] (f32/f16/bf16);
 * observed, age_frames: [B, N] f32; tokens: [B, S, D]; token_indices: [B, S] int32.
 * Shape errors return the reference's messages (:127-178).  Duplicate indices in a
 * row race (as in the reference's kernel); masks from SparseTokenMask are unique. */
BJF_API bjf_status bjf_feature_memory_assign_latest(void* features, bjf_dtype features_dtype,
                                            const int64_t features_dims[3], float* observed,
                                            const int64_t observed_dims[2], float* age_frames,
                                            const int64_t age_dims[2], const void* tokens,
                                            bjf_dtype tokens_dtype, const int64_t tokens_dims[3],
                                            const int32_t* token_indices,
                                            const int64_t indices_dims[2], int32_t age_observed,
                                            bjf_stream_t stream);

/* Replaces the EMA mode of `InterframeJepaFeatureMemory::update_tokens`
 * (InterframeJepaFeatureUpdateMode::Ema, src/feature_memory.rs:227-290), which the
 * reference runs on its portable tensor path (update_tokens_tiled_assign_cuda falls back to
 * it, :624-626).  In place, same shapes and errors as bjf_feature_memory_assign_latest:
 *   if age_observed: age_frames += observed
 *   features[b, idx, :] += (prev (1 - alpha) + tok alpha) observed[b, idx] + tok (1 - observed[b, idx]) - prev
 *   observed = 1; age_frames = 0
 * in the reference's f32 operation order; alpha is clamped to [0, 1] as the config's
 * normalisation does.  Duplicate indices in a row race (the reference adds their deltas). */
BJF_API bjf_status bjf_feature_memory_update_ema(void* features, bjf_dtype features_dtype,
                                                 const int64_t features_dims[3], float* observed,
                                                 const int64_t observed_dims[2], float* age_frames,
                                                 const int64_t age_dims[2], const void* tokens,
                                                 bjf_dtype tokens_dtype, const int64_t tokens_dims[3],
                                                 const int32_t* token_indices, const int64_t indices_dims[2],
                                                 float alpha, int32_t age_observed, bjf_stream_t stream);

/* Replaces `InterframeJepaFeatureMemory::reset_rows` (src/feature_memory.rs:348-375): zeroes
 * features[r], observed[r] and age_frames[r] for each of the `row_count` batch rows listed in
 * `rows` (device int32).  Rows outside [0, B) are skipped (the host-list form,
 * reset_row_indices :377-386, rejects them first in the C++ layer).  row_count 0 is a
 * no-op; at most 65535 rows per call. */
BJF_API bjf_status bjf_feature_memory_reset_rows(void* features, bjf_dtype features_dtype,
                                                 const int64_t features_dims[3], float* observed,
                                                 float* age_frames, const int32_t* rows, int64_t row_count,
                                                 bjf_stream_t stream);

/* ------------------------------------------------------------------------
 * Live viewer scorer (RGBA u8 camera frames)
 * ---------------------------------------------------------------------- */

/* RgbaPatchDiffFrameStats (src/viewer.rs:1067-1076) plus the two means the compensation
 * decision compares. */
typedef struct bjf_rgba_frame_stats {
  float channel_delta[3]; /* mean RGB delta in [0, 1] units */
  float luma_delta;       /* mean luma delta */
  int32_t compensate_global_lighting;
  float raw_abs;          /* mean per-pixel |delta| */
  float residual_abs;     /* mean per-pixel |delta - channel_delta| */
} bjf_rgba_frame_stats;

/* Bytes of device workspace bjf_rgba_patch_diff_scores needs for `streams` frame pairs on
 * `grid` (0 for a stream count outside 1..65535 or an empty grid). */
BJF_API size_t bjf_rgba_patch_diff_workspace_bytes(int64_t streams, const int64_t grid[3]);

/* Replaces `patch_diff_scores_from_rgba` (src/viewer.rs:1126-1157) with its frame statistics
 * `rgba_patch_diff_frame_stats` (:1079-1124), for S frame pairs at once.  prev / current:
 * [S, height, width, 4] u8 RGBA (4-byte aligned); grid = {1, height / P, width / P};
 * scores: [S, grid[1] * grid[2]] f32 (device); stats_out: [S] (device, nullable).  The
 * lighting statistics cover all height x width pixels of each frame, as the reference's cover
 * its whole buffers.  Errors use the reference's messages (:1133-1146). */
BJF_API bjf_status bjf_rgba_patch_diff_scores(const uint8_t* prev, const uint8_t* current, int64_t streams,
                                              int64_t width, int64_t height, int64_t patch_size,
                                              const int64_t grid[3], float* scores,
                                              bjf_rgba_frame_stats* stats_out, void* workspace,
                                              size_t workspace_bytes, bjf_stream_t stream);

/* The live viewer's mask policy after the threshold selection: the mask fields of
 * FeatureFrameViewerConfig (src/viewer.rs:566-579).  The encode bucket widths are derived on
 * the device as sparse_mask_bucket_widths (:887-925) derives them. */
typedef struct bjf_viewer_mask_policy {
  float dense_fallback_density; /* patch_diff_dense_fallback_density */
  int64_t dilation;             /* patch_diff_dilation_tiles (bjf_viewer_patch_diff_masks) */
  int32_t bucketed_encode;      /* sparse_encode_mode: 0 Exact, 1 BucketedContext */
  int64_t bucket_tokens;        /* sparse_mask_bucket_tokens (used with no densities) */
  int32_t bucket_density_count; /* entries of bucket_densities in use, 0..32 */
  float bucket_densities[32];   /* sparse_mask_bucket_densities */
} bjf_viewer_mask_policy;

/* Replaces patch_diff_dense_fallback -> dilate_sparse_patch_mask -> finalize_patch_diff_encode_masks
 * (src/viewer.rs:780-816, 946-961) for S streams: direct_indices [S, N] / direct_counts [S]
 * (a selection without dilation) -> write mask and encode mask, [S, N] / [S] each, ascending.
 * The direct buffers may be the write buffers.  Grids up to 32768 tokens.  Errors: a null
 * buffer or policy, an empty grid, more than 32 bucket densities. */
BJF_API bjf_status bjf_viewer_patch_diff_masks(const int32_t* direct_indices, const int32_t* direct_counts,
                                               int64_t streams, const int64_t grid[3],
                                               const bjf_viewer_mask_policy* policy, int32_t* write_indices,
                                               int32_t* write_counts, int32_t* encode_indices,
                                               int32_t* encode_counts, bjf_stream_t stream);

/* patch_diff_masks_from_scores (src/viewer.rs:831-841): the selection of `config` without its
 * dilation (patch_diff_base_mask_from_scores, :819-829), then bjf_viewer_patch_diff_masks with
 * config->dilation in place of the policy's (the reference dilates by the sparsity config).
 * scores [S, N] f32 (device). */
BJF_API bjf_status bjf_viewer_patch_diff_masks_from_scores(const float* scores, int64_t streams,
                                                           const int64_t grid[3], const bjf_patch_diff_config* config,
                                                           const bjf_viewer_mask_policy* policy,
                                                           int32_t* write_indices, int32_t* write_counts,
                                                           int32_t* encode_indices, int32_t* encode_counts,
                                                           bjf_stream_t stream);

/* Bytes of device workspace bjf_viewer_patch_diff_masks_from_rgba needs (0 for a stream count
 * outside 1..65535 or a grid that is not single-frame with at most 32768 tokens). */
BJF_API size_t bjf_viewer_rgba_masks_workspace_bytes(int64_t streams, const int64_t grid[3]);

/* Replaces the RGBA branch of the Bevy mask node, patch_diff_mask_from_rgba
 * (crates/bevy_jepa/src/mask.rs:126-175) without its refresh state, for S camera frame pairs:
 * the dense fast path (patch_diff_can_use_dense_fast_path, src/viewer.rs:1031-1036), the
 * sampled dense fast path (patch_diff_sampled_dense_fast_path_from_rgba, :1160-1195), else the
 * RGBA scores and patch_diff_masks_from_scores.  A dense shortcut gives every token in both
 * masks.  prev / current: [S, height, width, 4] u8; height = grid[1] * P, width = grid[2] * P;
 * outputs as bjf_viewer_patch_diff_masks_from_scores; stats_out as bjf_rgba_patch_diff_scores. */
BJF_API bjf_status bjf_viewer_patch_diff_masks_from_rgba(
    const uint8_t* prev, const uint8_t* current, int64_t streams, int64_t width, int64_t height, int64_t patch_size,
    const int64_t grid[3], const bjf_patch_diff_config* config, const bjf_viewer_mask_policy* policy,
    int32_t* write_indices, int32_t* write_counts, int32_t* encode_indices, int32_t* encode_counts,
    bjf_rgba_frame_stats* stats_out, void* workspace, size_t workspace_bytes, bjf_stream_t stream);

/* PatchDiffRefreshConfig (src/viewer.rs:186-270): bounded extra cache writes for tokens whose
 * motion stays below the threshold (subthreshold), tokens unwritten for a number of frames
 * (age) and a seeded scatter (blue noise).  Flags are 0 or 1; the reference's defaults are
 * enabled 0, decay 0.92, gain 1, trigger 1, subthreshold 0.04, interval 90, age 0.01, blue
 * noise 0.005 with seed 0x9e3779b97f4a7c15, max extra 0.05 (src/viewer.rs:35-49). */
typedef struct bjf_patch_diff_refresh_config {
  int32_t enabled;
  int32_t subthreshold_enabled;
  float subthreshold_decay;
  float subthreshold_gain;
  float subthreshold_trigger;
  float subthreshold_max_density;
  int32_t age_refresh_enabled;
  uint64_t age_refresh_interval_frames;
  float age_refresh_max_density;
  int32_t blue_noise_enabled;
  float blue_noise_refresh_density;
  uint64_t blue_noise_seed;
  float max_extra_density;
} bjf_patch_diff_refresh_config;

/* PatchDiffRefreshState (src/viewer.rs:275-283) of S streams, in device memory the caller owns:
 * per stream and token the decayed below-threshold residual and the frames since the token was
 * last written, per stream the frame index.  All zeros is the state before a stream's first
 * frame.  The reference starts a state over when the grid's token count changes; a caller that
 * changes grids zeroes the buffers (sized for the new grid) itself. */
typedef struct bjf_patch_diff_refresh_state {
  float* subthreshold_residual; /* [S, N] f32 */
  uint32_t* age_frames;         /* [S, N] */
  uint64_t* frame_index;        /* [S] */
} bjf_patch_diff_refresh_state;

/* PatchDiffRefreshState::masks_from_scores (src/viewer.rs:312-356) for S streams, each with
 * its own state: bjf_viewer_patch_diff_masks_from_scores with the refresh tokens of
 * augment_mask (:377-458) added to the write mask before the encode buckets, and every stream's
 * state advanced one frame, inside the same launch after the selection.  Inputs and outputs as
 * bjf_viewer_patch_diff_masks_from_scores.  Errors: those, and a null config or state buffer. */
BJF_API bjf_status bjf_viewer_patch_diff_refresh_masks_from_scores(
    const float* scores, int64_t streams, const int64_t grid[3], const bjf_patch_diff_config* config,
    const bjf_viewer_mask_policy* policy, const bjf_patch_diff_refresh_config* refresh,
    const bjf_patch_diff_refresh_state* state, int32_t* write_indices, int32_t* write_counts,
    int32_t* encode_indices, int32_t* encode_counts, bjf_stream_t stream);

/* The RGBA mask node with its refresh state (crates/bevy_jepa/src/mask.rs:126-185):
 * bjf_viewer_patch_diff_masks_from_rgba, where a dense shortcut is observe_write_mask of every
 * token and the scored path is PatchDiffRefreshState::masks_from_scores. */
BJF_API bjf_status bjf_viewer_patch_diff_refresh_masks_from_rgba(
    const uint8_t* prev, const uint8_t* current, int64_t streams, int64_t width, int64_t height, int64_t patch_size,
    const int64_t grid[3], const bjf_patch_diff_config* config, const bjf_viewer_mask_policy* policy,
    const bjf_patch_diff_refresh_config* refresh, const bjf_patch_diff_refresh_state* state,
    int32_t* write_indices, int32_t* write_counts, int32_t* encode_indices, int32_t* encode_counts,
    bjf_rgba_frame_stats* stats_out, void* workspace, size_t workspace_bytes, bjf_stream_t stream);

/* PatchDiffRefreshState::observe_write_mask (src/viewer.rs:309-313) for S streams: each stream
 * advances one frame with write_indices [S, N] / write_counts [S] (ascending, as the mask
 * entries write them) as its written tokens; indices outside the grid are skipped. */
BJF_API bjf_status bjf_viewer_patch_diff_refresh_observe(const int32_t* write_indices, const int32_t* write_counts,
                                                         int64_t streams, const int64_t grid[3],
                                                         const bjf_patch_diff_refresh_state* state,
                                                         bjf_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused step: mask -> plan -> patchify -> cache write, for S independent streams
 * ---------------------------------------------------------------------- */

/* One video stream per index s: video [S, C, T, H, W] (batch 1 each), token caches
 * [S, N, D], observed / age [S, N] f32, N = T/kt * H/P * W/P. */
typedef struct bjf_front_end_desc {
  int64_t streams;
  int64_t channels;
  int64_t frames;
  int64_t height;
  int64_t width;
  int64_t tubelet_size;
  int64_t patch_size;
  int64_t embed_dim;
  bjf_dtype video_dtype;  /* f16 / bf16 / f32 (f32 as bjf_sparse_patchify3d_forward runs it) */
  bjf_dtype weight_dtype; /* same as video_dtype for the tensor-core path */
  bjf_dtype cache_dtype;  /* f32 / f16 / bf16 */
  bjf_patch_diff_config mask;
} bjf_front_end_desc;

/* Bytes of device workspace bjf_front_end_step needs (0 for an invalid descriptor). */
BJF_API size_t bjf_front_end_workspace_bytes(const bjf_front_end_desc* desc);

/* One frame step of the front end for every stream, the per-stream composition of
 * patch_diff_context_mask (src/nodes.rs:411-456) -> SparsePatchifyPlan::new
 * (src/sparse_patchify.rs:236-269) -> sparse_patchify3d_forward_cuda (src/model.rs:1273-1328)
 * -> InterframeJepaFeatureMemory::update_tokens_tiled_assign_cuda_raw
 * (src/feature_memory.rs:616-645), with the patch-embed features written straight into
 * each stream's token cache.  age_observed: the memory has stepped before (step > 0).
 * weight [D, C, kt, P, P]; bias [D] f32 or NULL.  workspace: 256-byte aligned device
 * memory of bjf_front_end_workspace_bytes(desc) bytes.  counts_out (device, nullable):
 * [S] int32 active tubelets per stream.  Consecutive steps on one stream may overlap on the
 * device (a step's patch-diff pass starts beside the previous step's GEMM); results are as
 * if they ran one after another. */
BJF_API bjf_status bjf_front_end_step(const bjf_front_end_desc* desc, const void* video,
                                      const void* weight, const float* bias, void* caches,
                                      float* observed, float* age_frames, int32_t age_observed,
                                      void* workspace, size_t workspace_bytes, int32_t* counts_out,
                                      bjf_stream_t stream);

/* bjf_front_end_step for a live stream whose previous frame is already on the device: the step
 * that src/highres_pipeline.rs:1999-2052 runs per camera frame, which takes one new image per
 * step.  frame_ring: [S, C, ring_slots, H, W] -- ring_slots frames per stream and channel; the
 * step's clip is (ring[prev_slot], ring[cur_slot]), in that order, so a caller copies only each
 * new frame into the next slot (and, with three or more slots, may copy the next frame while
 * this step runs).  desc->frames and desc->tubelet_size must be 2; other arguments, workspace
 * (bjf_front_end_workspace_bytes(desc)) and results as bjf_front_end_step on the clip
 * [S, C, 2, H, W] = (prev, cur), bit for bit. */
BJF_API bjf_status bjf_front_end_step_ring(const bjf_front_end_desc* desc, const void* frame_ring,
                                           int32_t ring_slots, int32_t prev_slot, int32_t cur_slot,
                                           const void* weight, const float* bias, void* caches,
                                           float* observed, float* age_frames, int32_t age_observed,
                                           void* workspace, size_t workspace_bytes, int32_t* counts_out,
                                           bjf_stream_t stream);

/* The upload half of a live stream's step (src/highres_pipeline.rs:1999-2052 receives one new
 * image per step): copies streams [stream_begin, stream_end) of one new frame, host_frame
 * [S, C, H, W] (pinned host memory for an asynchronous copy), into slot `slot` of the frame
 * ring [S, C, ring_slots, H, W] that bjf_front_end_step_ring reads, as one 2-D copy (one
 * H x W plane per stream and channel).  Dims and dtype are desc's.  The copy is ordered on
 * `stream`; issue it on a copy stream to overlap the step that reads the other slots. */
BJF_API bjf_status bjf_frame_ring_upload(const bjf_front_end_desc* desc, const void* host_frame, void* frame_ring,
                                         int32_t ring_slots, int32_t slot, int64_t stream_begin, int64_t stream_end,
                                         bjf_stream_t stream);

/* No counterpart in the reference: bjf_front_end_step for callers that cannot
 * allocate device memory (a host whose device memory belongs to its framework's caching
 * allocator, or a real-time loop that forbids allocation after start-up because an
 * allocation can stall the device).  Same arguments and results as bjf_front_end_step,
 * minus the workspace: the step's scratch lives in a fixed 4 MiB __device__ array that
 * every GPU loading the library holds until exit, so streams x tokens is limited to about
 * 520k (the bench's 32 streams x 4096 tokens fit); larger steps return
 * BJF_ERR_UNSUPPORTED.  All calls on a device share that array: calls that overlap on the
 * GPU race, so issue them in order on one stream.  The first call on each device looks up
 * the array's address and clears its timeout flag; make it before any stream capture
 * begins.  The address is kept for the life of the process: resetting the device
 * (cudaDeviceReset) while the library is loaded is not supported.  A bounded-wait timeout
 * is reported by bjf_device_error_check, as for the workspace step.  A call allocates
 * nothing, so f32 operands run on the SIMT kernel here. */
BJF_API bjf_status bjf_front_end_step_no_alloc(const bjf_front_end_desc* desc, const void* video,
                                               const void* weight, const float* bias, void* caches,
                                               float* observed, float* age_frames,
                                               int32_t age_observed, int32_t* counts_out,
                                               bjf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BJF_H */
