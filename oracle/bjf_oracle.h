/*
 * bjf_oracle.h -- CPU oracle for the burn_jepa sparse front end.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * algorithm (mosure/burn_jepa 0.21.0, Rust) used as the parity checker for the
 * CUDA library and as the timed CPU baseline.  Nothing in the product links
 * or calls it.  Every function cites the reference file:line it restates.
 *
 * Parity pin: the restatement is checked against the known-answer vectors the
 * reference's own tests assert (tests/feature_memory.rs, tests/sparse_pipeline.rs,
 * tests/highres_anyup_pca_pipeline.rs, src/sparse_patchify.rs tests,
 * src/positional.rs tests, src/tokens.rs tests) and, for the Conv3d patch-embed
 * arithmetic that lives in the un-vendored crate burn_flex_gmm 0.21.2, against
 * torch F.conv3d (the op the reference's own fixture
 * tests/fixtures/vjepa_tiny_parity.py:130-133 uses) on seeded inputs.
 *
 * Conventions: sizes are int64_t; token indices are int64_t on the host side
 * (Rust usize) and int32_t where the reference stores them in an Int tensor on
 * the Cuda<f32,i32> backend (coords, token_indices).  All float arithmetic is
 * f32 as on the reference's NdArray<f32> backend; reductions accumulate in
 * double and round once, which is at least as accurate as the reference.
 *
 * Return codes: 0 = ok, negative = the reference's `ensure!`/`Err` branch
 * (the code names which one; see BJO_E_* below).
 */
#ifndef BJF_ORACLE_H
#define BJF_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  BJO_OK = 0,
  BJO_E_DENSE_LEN_ZERO = -1,        /* tokens.rs:44 */
  BJO_E_INDEX_OUT_OF_RANGE = -2,    /* tokens.rs:45-48 */
  BJO_E_THRESHOLD = -3,             /* nodes.rs:417-420, 467-470 */
  BJO_E_SCORE_LEN = -4,             /* nodes.rs:463-466 */
  BJO_E_GRID_TOO_SMALL = -5,        /* nodes.rs:379-385 */
  BJO_E_NOT_DIVISIBLE = -6,         /* nodes.rs:427-432 */
  BJO_E_GRID_MISMATCH = -7,         /* nodes.rs:433-436 */
  BJO_E_BATCH_ZERO = -8,            /* sparse_patchify.rs:243 */
  BJO_E_SPARSE_LEN_ZERO = -9,       /* sparse_feature_memory.rs:148-150 */
  BJO_E_BAD_ARG = -10
};

/* src/positional.rs:10-17 */
void bjo_token_index_to_coords(int64_t index, int64_t depth, int64_t height, int64_t width,
                               int64_t* frame, int64_t* row, int64_t* col);
/* src/positional.rs:19-21 */
int64_t bjo_coords_to_token_index(int64_t frame, int64_t row, int64_t col, int64_t depth,
                                  int64_t height, int64_t width);

/* src/tokens.rs:41-50  SparseTokenMask::new (sort_unstable + dedup + range check).
 * Sorts `indices` in place; returns the deduplicated length (>= 0) or an error. */
int64_t bjo_sparse_token_mask_new(int64_t* indices, int64_t n, int64_t dense_len);
/* src/tokens.rs:52-59  SparseTokenMask::from_keep_ratio; writes the indices, returns count */
int64_t bjo_from_keep_ratio(int64_t dense_len, float keep_ratio, int64_t* out);
/* src/tokens.rs:66-75  SparseTokenMask::evenly_spaced_indices; returns count */
int64_t bjo_evenly_spaced_indices(int64_t dense_len, int64_t keep, int64_t* out);
/* src/tokens.rs:143-157  SparseTokenMask::complement; returns count */
int64_t bjo_complement(const int64_t* indices, int64_t n, int64_t dense_len, int64_t* out);
/* src/tokens.rs:94-128  SparseTokenMask::padded_to_len; `indices` sorted unique; returns count */
int64_t bjo_padded_to_len(const int64_t* indices, int64_t n, int64_t dense_len, int64_t target_len,
                          int64_t* out);
/* src/tokens.rs:497-528  target_mask_from_context; returns count */
int64_t bjo_target_mask_from_context(const int64_t* context, int64_t n, int64_t dense_len,
                                     int64_t target_tokens, int64_t* out);

/* src/nodes.rs:565-631  patch_diff_token_scores (+ patch_diff_frame_pairs).
 * video [B,C,T,H,W] f32 contiguous -> scores [T/kt * H/P * W/P].  The batch is
 * summed into one shared score map. */
int bjo_patch_diff_token_scores(const float* video, int64_t batch, int64_t channels, int64_t frames,
                                int64_t height, int64_t width, int64_t tubelet_size,
                                int64_t patch_size, float* scores);

/* Mirrors SparseJepaPatchDiffSparsityConfig (src/nodes.rs:97-157). */
typedef struct bjo_patch_diff_config {
  float threshold;
  int64_t context_tokens;
  int64_t target_tokens;
  int64_t dilation;
  int64_t min_context_tokens;
  int32_t fill_to_context_tokens;
  int32_t allow_full_context;
} bjo_patch_diff_config;

/* src/nodes.rs:458-537 (+ push_dilated_sparse_index 633-662, SparseTokenMask::new).
 * Writes the ascending unique mask into out_indices (capacity depth*height*width)
 * and its length into *out_count. */
int bjo_patch_diff_context_mask_from_scores(const float* scores, int64_t n_scores, int64_t depth,
                                            int64_t height, int64_t width,
                                            const bjo_patch_diff_config* config,
                                            int64_t* out_indices, int64_t* out_count);

/* src/nodes.rs:411-456  patch_diff_context_mask (video -> mask), including the
 * top-k fast path (nodes.rs:443-449, 548-563). */
int bjo_patch_diff_context_mask(const float* video, int64_t batch, int64_t channels, int64_t frames,
                                int64_t height, int64_t width, int64_t tubelet_size,
                                int64_t patch_size, int64_t depth, int64_t grid_h, int64_t grid_w,
                                const bjo_patch_diff_config* config, int64_t* out_indices,
                                int64_t* out_count);

/* src/sparse_patchify.rs:236-269  SparsePatchifyPlan::new -> coords [batch*n, 4] =
 * (batch, tubelet, row, col), batch-major then mask order. */
int bjo_sparse_patchify_plan(const int64_t* mask_indices, int64_t n, int64_t depth, int64_t height,
                             int64_t width, int64_t batch, int32_t* coords);

/* Mirrors burn_flex_gmm::SparsePatchify3dConfig (fields as built at src/model.rs:1297-1306). */
typedef struct bjo_patchify_config {
  int64_t in_channels;
  int64_t out_channels;
  int64_t frames;
  int64_t height;
  int64_t width;
  int64_t tubelet_size;
  int64_t patch_h;
  int64_t patch_w;
} bjo_patchify_config;

/* burn_flex_gmm::cuda::sparse_patchify3d_forward_cuda semantics, pinned by
 * tests/sparse_patchify_cuda.rs:45-82 to Conv3d (stride = kernel) evaluated at
 * the selected tubelets (PatchEmbed3d::forward src/model.rs:88-93 + apply_token_mask
 * src/tokens.rs:541-548).
 *   out[row, d] = bias[d] + sum_{c,dt,dy,dx} W[d,c,dt,dy,dx] * x[b,c,t*kt+dt,r*ph+dy,col*pw+dx]
 * input [batch,C,T,H,W], coords [rows,4], weight [D,C,kt,ph,pw], bias [D] or NULL.
 * Rows whose coords fall outside the input are written as zeros. */
int bjo_sparse_patchify3d_forward(const bjo_patchify_config* config, int64_t batch,
                                  const float* input, const int32_t* coords, int64_t rows,
                                  const float* weight, const float* bias, float* out);

/* PatchEmbed3d::forward (src/model.rs:88-93): dense Conv3d -> [B, N, D]. */
int bjo_patch_embed3d_dense(const bjo_patchify_config* config, int64_t batch, const float* input,
                            const float* weight, const float* bias, float* out);

/* src/sparse_feature_memory.rs:22-108 (copy_feature_memory_kernel followed by
 * sparse_assign_feature_memory_kernel), applied in place:
 *   if age_observed: age += observed (every slot)
 *   for (b,s): features[b, idx[b,s], :] = tokens[b,s,:]; observed = 1; age = 0
 * Indices < 0 or >= dense_tokens are skipped (:79-85, :98-104). */
int bjo_feature_memory_assign_latest(float* features, float* observed, float* age_frames,
                                     const float* tokens, const int32_t* token_indices,
                                     int64_t batch, int64_t dense_tokens, int64_t embed_dim,
                                     int64_t sparse_len, int32_t age_observed);

/* src/feature_memory.rs:227-290, EMA update mode (portable path, in place, f32; duplicates
 * add their deltas as the reference's scatter-add does). */
int bjo_feature_memory_update_ema(float* features, float* observed, float* age_frames, const float* tokens,
                                  const int32_t* token_indices, int64_t batch, int64_t dense_tokens,
                                  int64_t embed_dim, int64_t sparse_len, float alpha, int32_t age_observed);

/* src/feature_memory.rs:348-375 reset_rows (rows outside [0, batch) skipped). */
int bjo_feature_memory_reset_rows(float* features, float* observed, float* age_frames, int64_t batch,
                                  int64_t dense_tokens, int64_t embed_dim, const int32_t* rows, int64_t row_count);

/* One front-end step over S independent streams, the per-stream composition the
 * reference pipeline runs (src/highres_pipeline.rs:2021-2040 with the patch-diff
 * driver of src/nodes.rs:411-456): patch_diff_context_mask -> SparsePatchifyPlan
 * (batch 1) -> sparse_patchify3d_forward -> feature-memory assign.  f32 throughout.
 * video [S,C,T,H,W]; caches [S,N,D]; observed/age [S,N]; counts[s] = active tubelets.
 * Streams run one after another; the inner loops use every OpenMP thread. */
int bjo_front_end_streams(const float* video, int64_t streams, const bjo_patchify_config* config,
                          const bjo_patch_diff_config* mask_config, const float* weight,
                          const float* bias, float* caches, float* observed, float* age_frames,
                          int32_t age_observed, int64_t* counts);

/* src/positional.rs:46-87 sparse_3d_sincos_pos_embed -> out [n, embed_dim]. */
void bjo_sparse_3d_sincos_pos_embed(int64_t embed_dim, int64_t depth, int64_t gh, int64_t gw,
                                    const int64_t* indices, int64_t n, float* out);
/* Patch embed + position table + modality embedding (src/model.rs:690-703), f32. */
int bjo_patchify_encoder_input(const bjo_patchify_config* config, int64_t batch, const float* input,
                               const int32_t* coords, int64_t rows, const float* weight, const float* bias,
                               const float* position_table, const float* modality_embed, float* out);

/* ---- live viewer policy (src/viewer.rs) ---- */
typedef struct bjo_rgba_frame_stats {
  float channel_delta[3];
  float luma_delta;
  int32_t compensate_global_lighting;
  float raw_abs;
  float residual_abs;
} bjo_rgba_frame_stats;

/* src/viewer.rs:1079-1124 rgba_patch_diff_frame_stats (sequential f32, as the reference). */
void bjo_rgba_patch_diff_frame_stats(const uint8_t* prev, int64_t prev_len, const uint8_t* cur, int64_t cur_len,
                                     bjo_rgba_frame_stats* out);
/* src/viewer.rs:1126-1244 patch_diff_scores_from_rgba (scores [gh * gw]). */
int bjo_patch_diff_scores_from_rgba(const uint8_t* prev, int64_t prev_len, const uint8_t* cur, int64_t cur_len,
                                    int64_t width, int64_t patch_size, int64_t depth, int64_t gh, int64_t gw,
                                    float* scores, bjo_rgba_frame_stats* stats_out);
/* src/viewer.rs:780-793 patch_diff_dense_fallback (returns the new length). */
int64_t bjo_patch_diff_dense_fallback(const int64_t* idx, int64_t n, int64_t dense_len, float density, int64_t* out);
/* src/viewer.rs:796-816, 844-869 dilate_sparse_patch_mask (returns the new length, -1 on error). */
int64_t bjo_dilate_sparse_patch_mask(const int64_t* idx, int64_t n, int64_t depth, int64_t gh, int64_t gw,
                                     int64_t dilation, int64_t* out);
/* src/viewer.rs:873-885 bucket_sparse_mask (returns the new length). */
int64_t bjo_bucket_sparse_mask(const int64_t* idx, int64_t n, int64_t dense_len, int64_t bucket_tokens, int64_t* out);

/* training/mask.rs:557-563 splitmix64 (the reference's own mixer; used for seeded inputs) */
uint64_t bjo_splitmix64(uint64_t value);

/* Number of OpenMP threads the oracle will use (1 when built without OpenMP). */
int bjo_num_threads(void);

#ifdef __cplusplus
}
#endif

#endif /* BJF_ORACLE_H */
