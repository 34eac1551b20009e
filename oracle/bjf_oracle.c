/*
 * bjf_oracle.c -- CPU oracle (TEST INFRASTRUCTURE ONLY) for the burn_jepa sparse
 * front end.  A restatement of the reference's algorithm in plain C; see
 * bjf_oracle.h for the contract and the pinning strategy.  It is the checker for
 * the CUDA library in tests/ and the timed CPU baseline in bench.py, nothing else.
 */
#include "bjf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

int bjo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static int64_t max_i64(int64_t a, int64_t b) { return a > b ? a : b; }
static int64_t min_i64(int64_t a, int64_t b) { return a < b ? a : b; }

/* ------------------------------------------------------------------------- */
/* src/positional.rs:10-21                                                    */
/* ------------------------------------------------------------------------- */
void bjo_token_index_to_coords(int64_t index, int64_t depth, int64_t height, int64_t width,
                               int64_t* frame, int64_t* row, int64_t* col) {
  (void)depth;
  int64_t tpf = max_i64(height * width, 1);
  int64_t f = index / tpf;
  int64_t rem = index - f * tpf;
  int64_t w = max_i64(width, 1);
  int64_t r = rem / w;
  *frame = f;
  *row = r;
  *col = rem - r * w;
}

int64_t bjo_coords_to_token_index(int64_t frame, int64_t row, int64_t col, int64_t depth,
                                  int64_t height, int64_t width) {
  (void)depth;
  return frame * (height * width) + row * width + col;
}

/* ------------------------------------------------------------------------- */
/* src/tokens.rs                                                              */
/* ------------------------------------------------------------------------- */
static int cmp_i64(const void* a, const void* b) {
  int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
  return (x > y) - (x < y);
}

/* tokens.rs:41-50: sort_unstable, dedup, then the two ensure! checks in order. */
int64_t bjo_sparse_token_mask_new(int64_t* indices, int64_t n, int64_t dense_len) {
  if (n > 0) qsort(indices, (size_t)n, sizeof(int64_t), cmp_i64);
  int64_t m = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (m == 0 || indices[m - 1] != indices[i]) indices[m++] = indices[i];
  }
  if (dense_len <= 0) return BJO_E_DENSE_LEN_ZERO;
  for (int64_t i = 0; i < m; ++i) {
    if (indices[i] < 0 || indices[i] >= dense_len) return BJO_E_INDEX_OUT_OF_RANGE;
  }
  return m;
}

/* tokens.rs:52-59 */
int64_t bjo_from_keep_ratio(int64_t dense_len, float keep_ratio, int64_t* out) {
  float r = keep_ratio < 0.0f ? 0.0f : (keep_ratio > 1.0f ? 1.0f : keep_ratio);
  int64_t keep = (int64_t)ceilf((float)dense_len * r);
  keep = min_i64(max_i64(keep, 1), max_i64(dense_len, 1));
  for (int64_t i = 0; i < keep; ++i) out[i] = i;
  return keep;
}

/* tokens.rs:66-75 */
int64_t bjo_evenly_spaced_indices(int64_t dense_len, int64_t keep, int64_t* out) {
  keep = min_i64(max_i64(keep, 1), max_i64(dense_len, 1));
  if (keep == dense_len) {
    for (int64_t i = 0; i < dense_len; ++i) out[i] = i;
    return dense_len;
  }
  int64_t last = dense_len > 0 ? dense_len - 1 : 0;
  int64_t denom = max_i64(keep, 1);
  for (int64_t i = 0; i < keep; ++i) out[i] = (i * last + keep / 2) / denom;
  return keep;
}

/* tokens.rs:143-157 */
int64_t bjo_complement(const int64_t* indices, int64_t n, int64_t dense_len, int64_t* out) {
  unsigned char* keep = (unsigned char*)calloc((size_t)max_i64(dense_len, 1), 1);
  for (int64_t i = 0; i < n; ++i) keep[indices[i]] = 1;
  int64_t m = 0;
  for (int64_t i = 0; i < dense_len; ++i)
    if (!keep[i]) out[m++] = i;
  free(keep);
  return m;
}

/* tokens.rs:94-128 */
int64_t bjo_padded_to_len(const int64_t* indices, int64_t n, int64_t dense_len, int64_t target_len,
                          int64_t* out) {
  if (target_len <= n) {
    memcpy(out, indices, (size_t)n * sizeof(int64_t));
    return n;
  }
  if (target_len >= dense_len) {
    for (int64_t i = 0; i < dense_len; ++i) out[i] = i;
    return dense_len;
  }
  unsigned char* keep = (unsigned char*)calloc((size_t)dense_len, 1);
  int64_t* even = (int64_t*)malloc((size_t)dense_len * sizeof(int64_t));
  int64_t m = 0;
  for (int64_t i = 0; i < n; ++i) {
    keep[indices[i]] = 1;
    out[m++] = indices[i];
  }
  int64_t ne = bjo_evenly_spaced_indices(dense_len, target_len, even);
  for (int64_t i = 0; i < ne && m < target_len; ++i) {
    if (!keep[even[i]]) {
      keep[even[i]] = 1;
      out[m++] = even[i];
    }
  }
  for (int64_t i = 0; i < dense_len && m < target_len; ++i) {
    if (!keep[i]) {
      keep[i] = 1;
      out[m++] = i;
    }
  }
  free(even);
  free(keep);
  return bjo_sparse_token_mask_new(out, m, dense_len);
}

/* tokens.rs:497-528 */
int64_t bjo_target_mask_from_context(const int64_t* context, int64_t n, int64_t dense_len,
                                     int64_t target_tokens, int64_t* out) {
  int64_t avail = dense_len > n ? dense_len - n : 0;
  target_tokens = min_i64(max_i64(target_tokens, 1), max_i64(avail, 1));
  unsigned char* blocked = (unsigned char*)calloc((size_t)max_i64(dense_len, 1), 1);
  int64_t* even = (int64_t*)malloc((size_t)max_i64(dense_len, 1) * sizeof(int64_t));
  for (int64_t i = 0; i < n; ++i) blocked[context[i]] = 1;
  int64_t ne = bjo_evenly_spaced_indices(dense_len, target_tokens, even);
  int64_t m = 0;
  for (int64_t i = 0; i < ne; ++i)
    if (!blocked[even[i]]) out[m++] = even[i];
  for (int64_t i = 0; i < m; ++i) blocked[out[i]] = 1;
  if (m < target_tokens) {
    for (int64_t i = 0; i < dense_len; ++i) {
      if (!blocked[i]) {
        out[m++] = i;
        blocked[i] = 1;
        if (m >= target_tokens) break;
      }
    }
  }
  free(even);
  free(blocked);
  return bjo_sparse_token_mask_new(out, m, dense_len);
}

/* ------------------------------------------------------------------------- */
/* src/nodes.rs:565-631  patch_diff_token_scores                              */
/* ------------------------------------------------------------------------- */
int bjo_patch_diff_token_scores(const float* video, int64_t batch, int64_t channels, int64_t frames,
                                int64_t height, int64_t width, int64_t tubelet_size,
                                int64_t patch_size, float* scores) {
  int64_t P = max_i64(patch_size, 1);
  int64_t kt = max_i64(tubelet_size, 1);
  int64_t depth = frames / kt, gh = height / P, gw = width / P;
  int64_t tpf = gh * gw;
  const int64_t plane = height * width;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t tr = 0; tr < depth * gh; ++tr) {
    int64_t tubelet = tr / gh, r = tr % gh;
    int64_t start = tubelet * kt;
    int64_t end = min_i64((tubelet + 1) * kt, frames);
    /* patch_diff_frame_pairs nodes.rs:621-631 */
    int64_t pair_next[64];
    int64_t npairs = 0;
    if (end > start + 1) {
      for (int64_t f = start + 1; f < end && npairs < 64; ++f) pair_next[npairs++] = f;
    } else if (start > 0) {
      pair_next[npairs++] = start;
    }
    float* out = scores + tubelet * tpf + r * gw;
    if (npairs == 0) {
      for (int64_t c = 0; c < gw; ++c) out[c] = 0.0f;
      continue;
    }
    const double denom = (double)(npairs * batch * channels * P * P);
    const float inv = (float)(1.0 / denom); /* mul_scalar(1/denom) on an f32 tensor */
    for (int64_t c = 0; c < gw; ++c) {
      double acc = 0.0;
      for (int64_t b = 0; b < batch; ++b)
        for (int64_t ch = 0; ch < channels; ++ch) {
          const float* base = video + ((b * channels + ch) * frames) * plane;
          for (int64_t py = 0; py < P; ++py)
            for (int64_t px = 0; px < P; ++px) {
              int64_t off = (r * P + py) * width + c * P + px;
              /* diff_sum accumulates |next - prev| over the pairs in f32 (nodes.rs:586-600) */
              float d = 0.0f;
              for (int64_t p = 0; p < npairs; ++p) {
                int64_t f = pair_next[p];
                float v = fabsf(base[f * plane + off] - base[(f - 1) * plane + off]);
                d = (p == 0) ? v : d + v;
              }
              acc += (double)d;
            }
        }
      out[c] = (float)acc * inv;
    }
  }
  return BJO_OK;
}

/* ------------------------------------------------------------------------- */
/* src/nodes.rs:458-537, 633-662  selection from scores                       */
/* ------------------------------------------------------------------------- */
typedef struct {
  int64_t index;
  float score;
} scored_t;

/* sort_by(score desc via partial_cmp, NaN -> Equal, then index asc) nodes.rs:485-491 */
static int cmp_scored(const void* a, const void* b) {
  const scored_t* l = (const scored_t*)a;
  const scored_t* r = (const scored_t*)b;
  if (!isnan(l->score) && !isnan(r->score)) {
    if (r->score < l->score) return -1;
    if (r->score > l->score) return 1;
  }
  return (l->index > r->index) - (l->index < r->index);
}

/* nodes.rs:633-662 push_dilated_sparse_index */
static void push_dilated(int64_t index, int64_t depth, int64_t gh, int64_t gw, int64_t dilation,
                         unsigned char* keep, int64_t* selected, int64_t* nsel, int64_t target) {
  int64_t len = depth * gh * gw;
  if (*nsel >= target || index >= len) return;
  int64_t t, row, col;
  bjo_token_index_to_coords(index, depth, gh, gw, &t, &row, &col);
  int64_t r0 = row > dilation ? row - dilation : 0;
  int64_t r1 = min_i64(row + dilation, gh > 0 ? gh - 1 : 0);
  int64_t c0 = col > dilation ? col - dilation : 0;
  int64_t c1 = min_i64(col + dilation, gw > 0 ? gw - 1 : 0);
  for (int64_t r = r0; r <= r1; ++r)
    for (int64_t c = c0; c <= c1; ++c) {
      int64_t idx = bjo_coords_to_token_index(t, r, c, depth, gh, gw);
      if (keep[idx]) continue;
      keep[idx] = 1;
      selected[(*nsel)++] = idx;
      if (*nsel >= target) return;
    }
}

int bjo_patch_diff_context_mask_from_scores(const float* scores, int64_t n_scores, int64_t depth,
                                            int64_t height, int64_t width,
                                            const bjo_patch_diff_config* cfg,
                                            int64_t* out_indices, int64_t* out_count) {
  const int64_t len = depth * height * width;
  if (n_scores != len) return BJO_E_SCORE_LEN;
  if (!isfinite(cfg->threshold) || !(cfg->threshold >= 0.0f)) return BJO_E_THRESHOLD;
  int64_t context_tokens;
  if (cfg->allow_full_context) {
    context_tokens = min_i64(max_i64(cfg->context_tokens, 1), len);
  } else {
    if (len <= 1) return BJO_E_GRID_TOO_SMALL; /* context_budget nodes.rs:379-385 */
    context_tokens = min_i64(max_i64(cfg->context_tokens, 1), len - 1);
  }
  int64_t min_context = min_i64(min_i64(max_i64(cfg->min_context_tokens, 1), context_tokens), len);
  scored_t* sorted = (scored_t*)malloc((size_t)max_i64(len, 1) * sizeof(scored_t));
  for (int64_t i = 0; i < len; ++i) {
    sorted[i].index = i;
    sorted[i].score = scores[i];
  }
  qsort(sorted, (size_t)len, sizeof(scored_t), cmp_scored);
  unsigned char* keep = (unsigned char*)calloc((size_t)max_i64(len, 1), 1);
  int64_t threshold_cap = cfg->allow_full_context ? len : context_tokens;
  int64_t nsel = 0;
  for (int64_t i = 0; i < len; ++i) {
    if (sorted[i].score < cfg->threshold) break;
    push_dilated(sorted[i].index, depth, height, width, cfg->dilation, keep, out_indices, &nsel,
                 threshold_cap);
    if (nsel >= threshold_cap) break;
  }
  int64_t fill_target = cfg->fill_to_context_tokens ? context_tokens : min_context;
  if (nsel < fill_target) {
    for (int64_t i = 0; i < len; ++i) {
      push_dilated(sorted[i].index, depth, height, width, cfg->dilation, keep, out_indices, &nsel,
                   fill_target);
      if (nsel >= fill_target) break;
    }
  }
  free(keep);
  free(sorted);
  int64_t m = bjo_sparse_token_mask_new(out_indices, nsel, len);
  if (m < 0) return (int)m;
  *out_count = m;
  return BJO_OK;
}

/* nodes.rs:411-456 (+ top-k fast path 548-563) */
int bjo_patch_diff_context_mask(const float* video, int64_t batch, int64_t channels, int64_t frames,
                                int64_t height, int64_t width, int64_t tubelet_size,
                                int64_t patch_size, int64_t depth, int64_t grid_h, int64_t grid_w,
                                const bjo_patch_diff_config* cfg, int64_t* out_indices,
                                int64_t* out_count) {
  if (!isfinite(cfg->threshold) || !(cfg->threshold >= 0.0f)) return BJO_E_THRESHOLD;
  int64_t kt = max_i64(tubelet_size, 1), P = max_i64(patch_size, 1);
  if (frames % kt != 0 || height % P != 0 || width % P != 0) return BJO_E_NOT_DIVISIBLE;
  if (frames / kt != depth || height / P != grid_h || width / P != grid_w) return BJO_E_GRID_MISMATCH;
  const int64_t len = depth * grid_h * grid_w;
  int64_t context_tokens;
  if (cfg->allow_full_context) {
    context_tokens = min_i64(max_i64(cfg->context_tokens, 1), len);
  } else {
    if (len <= 1) return BJO_E_GRID_TOO_SMALL;
    context_tokens = min_i64(max_i64(cfg->context_tokens, 1), len - 1);
  }
  float* scores = (float*)malloc((size_t)max_i64(len, 1) * sizeof(float));
  int rc = bjo_patch_diff_token_scores(video, batch, channels, frames, height, width, tubelet_size,
                                       patch_size, scores);
  if (rc == BJO_OK && cfg->threshold <= 0.0f && cfg->dilation == 0 && !cfg->allow_full_context &&
      cfg->fill_to_context_tokens) {
    /* topk_with_indices(context_tokens): the k largest scores; ties broken by
     * ascending index (a stable descending sort). */
    scored_t* sorted = (scored_t*)malloc((size_t)len * sizeof(scored_t));
    for (int64_t i = 0; i < len; ++i) {
      sorted[i].index = i;
      sorted[i].score = scores[i];
    }
    qsort(sorted, (size_t)len, sizeof(scored_t), cmp_scored);
    for (int64_t i = 0; i < context_tokens; ++i) out_indices[i] = sorted[i].index;
    free(sorted);
    int64_t m = bjo_sparse_token_mask_new(out_indices, context_tokens, len);
    free(scores);
    if (m < 0) return (int)m;
    *out_count = m;
    return BJO_OK;
  }
  if (rc == BJO_OK)
    rc = bjo_patch_diff_context_mask_from_scores(scores, len, depth, grid_h, grid_w, cfg,
                                                 out_indices, out_count);
  free(scores);
  return rc;
}

/* ------------------------------------------------------------------------- */
/* src/sparse_patchify.rs:236-269  SparsePatchifyPlan::new                    */
/* ------------------------------------------------------------------------- */
int bjo_sparse_patchify_plan(const int64_t* mask_indices, int64_t n, int64_t depth, int64_t height,
                             int64_t width, int64_t batch, int32_t* coords) {
  if (batch <= 0) return BJO_E_BATCH_ZERO;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t i = 0; i < n; ++i) {
      int64_t t, r, c;
      bjo_token_index_to_coords(mask_indices[i], depth, height, width, &t, &r, &c);
      int32_t* out = coords + (b * n + i) * 4;
      out[0] = (int32_t)b;
      out[1] = (int32_t)t;
      out[2] = (int32_t)r;
      out[3] = (int32_t)c;
    }
  return BJO_OK;
}

/* ------------------------------------------------------------------------- */
/* Conv3d at selected tubelets (flex-gmm semantics; model.rs:88-93)           */
/* ------------------------------------------------------------------------- */
static void gather_tubelet(const bjo_patchify_config* cfg, const float* input, int64_t b, int64_t t,
                           int64_t r, int64_t col, float* a) {
  const int64_t C = cfg->in_channels, T = cfg->frames, H = cfg->height, W = cfg->width;
  const int64_t kt = cfg->tubelet_size, ph = cfg->patch_h, pw = cfg->patch_w;
  int64_t k = 0;
  for (int64_t ch = 0; ch < C; ++ch)
    for (int64_t dt = 0; dt < kt; ++dt)
      for (int64_t dy = 0; dy < ph; ++dy) {
        const float* src =
            input + (((b * C + ch) * T + t * kt + dt) * H + r * ph + dy) * W + col * pw;
        for (int64_t dx = 0; dx < pw; ++dx) a[k++] = src[dx];
      }
}

static void project_row(const float* a, int64_t K, int64_t D, const float* weight, const float* bias,
                        float* out) {
  for (int64_t d = 0; d < D; ++d) {
    const float* w = weight + d * K;
    double acc = 0.0;
#pragma omp simd reduction(+ : acc)
    for (int64_t k = 0; k < K; ++k) acc += (double)w[k] * (double)a[k];
    out[d] = (float)acc + (bias ? bias[d] : 0.0f);
  }
}

int bjo_sparse_patchify3d_forward(const bjo_patchify_config* cfg, int64_t batch, const float* input,
                                  const int32_t* coords, int64_t rows, const float* weight,
                                  const float* bias, float* out) {
  const int64_t C = cfg->in_channels, D = cfg->out_channels;
  const int64_t kt = cfg->tubelet_size, ph = cfg->patch_h, pw = cfg->patch_w;
  if (C <= 0 || D <= 0 || kt <= 0 || ph <= 0 || pw <= 0 || batch <= 0) return BJO_E_BAD_ARG;
  const int64_t K = C * kt * ph * pw;
  const int64_t depth = cfg->frames / kt, gh = cfg->height / ph, gw = cfg->width / pw;
#pragma omp parallel
  {
    float* a = (float*)malloc((size_t)K * sizeof(float));
#pragma omp for schedule(dynamic, 4)
    for (int64_t m = 0; m < rows; ++m) {
      const int32_t* cd = coords + m * 4;
      if (cd[0] < 0 || cd[0] >= batch || cd[1] < 0 || cd[1] >= depth || cd[2] < 0 || cd[2] >= gh ||
          cd[3] < 0 || cd[3] >= gw) {
        for (int64_t d = 0; d < D; ++d) out[m * D + d] = 0.0f;
        continue;
      }
      gather_tubelet(cfg, input, cd[0], cd[1], cd[2], cd[3], a);
      project_row(a, K, D, weight, bias, out + m * D);
    }
    free(a);
  }
  return BJO_OK;
}

int bjo_patch_embed3d_dense(const bjo_patchify_config* cfg, int64_t batch, const float* input,
                            const float* weight, const float* bias, float* out) {
  const int64_t kt = cfg->tubelet_size, ph = cfg->patch_h, pw = cfg->patch_w;
  if (kt <= 0 || ph <= 0 || pw <= 0 || batch <= 0) return BJO_E_BAD_ARG;
  const int64_t depth = cfg->frames / kt, gh = cfg->height / ph, gw = cfg->width / pw;
  const int64_t n = depth * gh * gw;
  int32_t* coords = (int32_t*)malloc((size_t)(batch * n * 4) * sizeof(int32_t));
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t i = 0; i < n; ++i) {
      int64_t t, r, c;
      bjo_token_index_to_coords(i, depth, gh, gw, &t, &r, &c);
      int32_t* cd = coords + (b * n + i) * 4;
      cd[0] = (int32_t)b;
      cd[1] = (int32_t)t;
      cd[2] = (int32_t)r;
      cd[3] = (int32_t)c;
    }
  int rc = bjo_sparse_patchify3d_forward(cfg, batch, input, coords, batch * n, weight, bias, out);
  free(coords);
  return rc;
}

/* ------------------------------------------------------------------------- */
/* src/sparse_feature_memory.rs:22-108  tiled AssignLatest                    */
/* ------------------------------------------------------------------------- */
int bjo_feature_memory_assign_latest(float* features, float* observed, float* age_frames,
                                     const float* tokens, const int32_t* token_indices,
                                     int64_t batch, int64_t dense_tokens, int64_t embed_dim,
                                     int64_t sparse_len, int32_t age_observed) {
  if (sparse_len == 0) return BJO_E_SPARSE_LEN_ZERO;
  if (age_observed) {
    for (int64_t i = 0; i < batch * dense_tokens; ++i) age_frames[i] += observed[i];
  }
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t s = 0; s < sparse_len; ++s) {
      int32_t idx = token_indices[b * sparse_len + s];
      if (idx < 0 || idx >= dense_tokens) continue;
      memcpy(features + (b * dense_tokens + idx) * embed_dim,
             tokens + (b * sparse_len + s) * embed_dim, (size_t)embed_dim * sizeof(float));
      observed[b * dense_tokens + idx] = 1.0f;
      age_frames[b * dense_tokens + idx] = 0.0f;
    }
  return BJO_OK;
}

/* src/feature_memory.rs:227-290, InterframeJepaFeatureUpdateMode::Ema { alpha } (the
 * portable update_tokens path, with the config's clamp of alpha, :40-48):
 *   if age_observed: age += observed
 *   previous = features[b, idx]; obs = observed[b, idx]            (gathered before any write)
 *   blended = previous * (1 - alpha) + tokens * alpha
 *   delta = (blended * obs + tokens * (-obs + 1)) - previous
 *   features = features.scatter(idx, delta, Add)                   (duplicates add their deltas)
 *   observed += 1 - observed[b, idx];  age += 0 - age[b, idx]      (scatter-add likewise)
 * f32 arithmetic, one operation at a time (the build does not contract). */
int bjo_feature_memory_update_ema(float* features, float* observed, float* age_frames, const float* tokens,
                                  const int32_t* token_indices, int64_t batch, int64_t dense_tokens,
                                  int64_t embed_dim, int64_t sparse_len, float alpha, int32_t age_observed) {
  if (sparse_len == 0) return BJO_E_SPARSE_LEN_ZERO;
  if (alpha < 0.0f) alpha = 0.0f;
  if (alpha > 1.0f) alpha = 1.0f;
  const float one_minus_alpha = 1.0f - alpha;
  if (age_observed) {
    for (int64_t i = 0; i < batch * dense_tokens; ++i) age_frames[i] += observed[i];
  }
  const int64_t rows = batch * sparse_len;
  float* delta = (float*)malloc(sizeof(float) * (size_t)(rows * embed_dim + 2 * rows));
  if (!delta) return BJO_E_BAD_ARG;
  float* dobs = delta + rows * embed_dim;
  float* dage = dobs + rows;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t s = 0; s < sparse_len; ++s) {
      const int64_t r = b * sparse_len + s;
      const int32_t idx = token_indices[r];
      if (idx < 0 || idx >= dense_tokens) continue;
      const int64_t slot = b * dense_tokens + idx;
      const float obs = observed[slot];
      const float first = -obs + 1.0f;
      for (int64_t d = 0; d < embed_dim; ++d) {
        const float prev = features[slot * embed_dim + d];
        const float tok = tokens[r * embed_dim + d];
        const float blended = prev * one_minus_alpha + tok * alpha;
        delta[r * embed_dim + d] = (blended * obs + tok * first) - prev;
      }
      dobs[r] = 1.0f - obs;
      dage[r] = 0.0f - age_frames[slot];
    }
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t s = 0; s < sparse_len; ++s) {
      const int64_t r = b * sparse_len + s;
      const int32_t idx = token_indices[r];
      if (idx < 0 || idx >= dense_tokens) continue;
      const int64_t slot = b * dense_tokens + idx;
      for (int64_t d = 0; d < embed_dim; ++d) features[slot * embed_dim + d] += delta[r * embed_dim + d];
      observed[slot] += dobs[r];
      age_frames[slot] += dage[r];
    }
  free(delta);
  return BJO_OK;
}

/* src/feature_memory.rs:348-375 reset_rows: zero features / observed / age of the listed rows
 * (rows outside [0, batch) are skipped here; the reference's host form rejects them). */
int bjo_feature_memory_reset_rows(float* features, float* observed, float* age_frames, int64_t batch,
                                  int64_t dense_tokens, int64_t embed_dim, const int32_t* rows, int64_t row_count) {
  for (int64_t i = 0; i < row_count; ++i) {
    const int32_t r = rows[i];
    if (r < 0 || r >= batch) continue;
    memset(features + (int64_t)r * dense_tokens * embed_dim, 0, sizeof(float) * (size_t)(dense_tokens * embed_dim));
    memset(observed + (int64_t)r * dense_tokens, 0, sizeof(float) * (size_t)dense_tokens);
    memset(age_frames + (int64_t)r * dense_tokens, 0, sizeof(float) * (size_t)dense_tokens);
  }
  return BJO_OK;
}

int bjo_front_end_streams(const float* video, int64_t streams, const bjo_patchify_config* cfg,
                          const bjo_patch_diff_config* mask_cfg, const float* weight,
                          const float* bias, float* caches, float* observed, float* age_frames,
                          int32_t age_observed, int64_t* counts) {
  const int64_t C = cfg->in_channels, T = cfg->frames, H = cfg->height, W = cfg->width;
  const int64_t kt = cfg->tubelet_size, P = cfg->patch_h, D = cfg->out_channels;
  if (kt <= 0 || P <= 0 || cfg->patch_w != P) return BJO_E_BAD_ARG;
  const int64_t depth = T / kt, gh = H / P, gw = W / P, n = depth * gh * gw;
  int64_t* idx = (int64_t*)malloc((size_t)n * sizeof(int64_t));
  int32_t* coords = (int32_t*)malloc((size_t)n * 4 * sizeof(int32_t));
  int32_t* idx32 = (int32_t*)malloc((size_t)n * sizeof(int32_t));
  float* feats = (float*)malloc((size_t)(n * D) * sizeof(float));
  int rc = BJO_OK;
  for (int64_t s = 0; s < streams && rc == BJO_OK; ++s) {
    const float* v = video + s * C * T * H * W;
    int64_t m = 0;
    rc = bjo_patch_diff_context_mask(v, 1, C, T, H, W, kt, P, depth, gh, gw, mask_cfg, idx, &m);
    if (rc != BJO_OK) break;
    rc = bjo_sparse_patchify_plan(idx, m, depth, gh, gw, 1, coords);
    if (rc != BJO_OK) break;
    rc = bjo_sparse_patchify3d_forward(cfg, 1, v, coords, m, weight, bias, feats);
    if (rc != BJO_OK) break;
    for (int64_t i = 0; i < m; ++i) idx32[i] = (int32_t)idx[i];
    rc = bjo_feature_memory_assign_latest(caches + s * n * D, observed + s * n, age_frames + s * n,
                                          feats, idx32, 1, n, D, m, age_observed);
    counts[s] = m;
  }
  free(feats);
  free(idx32);
  free(coords);
  free(idx);
  return rc;
}

/* ---- encoder input (src/positional.rs, src/model.rs) ---- */

static int64_t even_dim(int64_t d) { return d - (d % 2); }

/* src/positional.rs:69-87 one_position_sincos: sin(pos * omega_i) then cos(pos * omega_i),
 * omega_i = 1 / 10000^(i / half) in f32; a trailing 0 for an odd dim. */
static float* one_position_sincos(int64_t dim, float pos, float* out) {
  if (dim == 0) return out;
  const int64_t half = dim / 2;
  const float h = (float)(half > 1 ? half : 1);
  for (int64_t i = 0; i < half; ++i) *out++ = sinf(pos * (1.0f / powf(10000.0f, (float)i / h)));
  for (int64_t i = 0; i < half; ++i) *out++ = cosf(pos * (1.0f / powf(10000.0f, (float)i / h)));
  if (dim % 2 == 1) *out++ = 0.0f;
  return out;
}

/* src/positional.rs:46-67 sparse_3d_sincos_pos_embed: per token index, the frame, row and
 * column sin-cos blocks of dims even(D/2), even(D/4), even(D - both), zero-padded to D. */
void bjo_sparse_3d_sincos_pos_embed(int64_t embed_dim, int64_t depth, int64_t gh, int64_t gw,
                                    const int64_t* indices, int64_t n, float* out) {
  const int64_t d_dim = even_dim(embed_dim / 2), h_dim = even_dim(embed_dim / 4);
  int64_t w_dim = embed_dim - (d_dim + h_dim);
  if (w_dim < 0) w_dim = 0;
  w_dim = even_dim(w_dim);
  int64_t rem = embed_dim - (d_dim + h_dim + w_dim);
  if (rem < 0) rem = 0;
  const int64_t tpf = gh * gw > 0 ? gh * gw : 1, w = gw > 0 ? gw : 1;
  (void)depth;
  for (int64_t k = 0; k < n; ++k) {
    const int64_t index = indices[k];
    const int64_t frame = index / tpf, local = index - frame * tpf, row = local / w, col = local - row * w;
    float* o = out + k * embed_dim;
    o = one_position_sincos(d_dim, (float)frame, o);
    o = one_position_sincos(h_dim, (float)row, o);
    o = one_position_sincos(w_dim, (float)col, o);
    for (int64_t i = 0; i < rem; ++i) *o++ = 0.0f;
  }
}

/* Encoder input tokens (src/model.rs:690-703 after the patch embed): ((conv + bias) + pos) +
 * modality per row, pos = table[token index of the row]; f32, in that order.  Rows whose
 * coords fall outside the input stay zero, as in bjo_sparse_patchify3d_forward. */
int bjo_patchify_encoder_input(const bjo_patchify_config* config, int64_t batch, const float* input,
                               const int32_t* coords, int64_t rows, const float* weight, const float* bias,
                               const float* position_table, const float* modality_embed, float* out) {
  int rc = bjo_sparse_patchify3d_forward(config, batch, input, coords, rows, weight, bias, out);
  if (rc) return rc;
  const int64_t D = config->out_channels, gh = config->height / config->patch_h, gw = config->width / config->patch_w;
  const int64_t depth = config->frames / config->tubelet_size;
  for (int64_t r = 0; r < rows; ++r) {
    const int32_t* c = coords + r * 4;
    if (c[0] < 0 || c[0] >= batch || c[1] < 0 || c[1] >= depth || c[2] < 0 || c[2] >= gh || c[3] < 0 || c[3] >= gw)
      continue;
    const int64_t token = ((int64_t)c[1] * gh + c[2]) * gw + c[3];
    for (int64_t d = 0; d < D; ++d) {
      float v = out[r * D + d];
      if (position_table) v = v + position_table[token * D + d];
      if (modality_embed) v = v + modality_embed[d];
      out[r * D + d] = v;
    }
  }
  return BJO_OK;
}

/* ---- live viewer policy (src/viewer.rs) ---- */

static void rgba_rgb(const uint8_t* rgba, int64_t offset, float out[3]) {
  /* :1246-1252 */
  out[0] = (float)rgba[offset] / 255.0f;
  out[1] = (float)rgba[offset + 1] / 255.0f;
  out[2] = (float)rgba[offset + 2] / 255.0f;
}

static float rgb_luma(const float rgb[3]) { return rgb[0] * 0.2126f + rgb[1] * 0.7152f + rgb[2] * 0.0722f; }

static void rgb_chroma(const float rgb[3], float out[3]) {
  /* :1267-1270 */
  float denom = rgb[0] + rgb[1] + rgb[2];
  if (denom < 0.10f) denom = 0.10f;
  out[0] = rgb[0] / denom;
  out[1] = rgb[1] / denom;
  out[2] = rgb[2] / denom;
}

static float rgb_chroma_diff(const float prev[3], const float cur[3]) {
  /* :1258-1265 */
  float p[3], c[3];
  rgb_chroma(prev, p);
  rgb_chroma(cur, c);
  return (fabsf(c[0] - p[0]) + fabsf(c[1] - p[1]) + fabsf(c[2] - p[2])) / 3.0f;
}

static float fmax_rust(float a, float b) { return a > b ? a : b; } /* finite inputs */

/* :1079-1124  rgba_patch_diff_frame_stats: sequential f32 sums over min(len) / 4 pixels. */
void bjo_rgba_patch_diff_frame_stats(const uint8_t* prev, int64_t prev_len, const uint8_t* cur, int64_t cur_len,
                                     bjo_rgba_frame_stats* out) {
  int64_t pixels = (prev_len < cur_len ? prev_len : cur_len) / 4;
  if (pixels < 1) pixels = 1;
  float channel_delta[3] = {0.0f, 0.0f, 0.0f};
  float luma_delta = 0.0f, raw_abs = 0.0f;
  for (int64_t i = 0; i < pixels; ++i) {
    float p[3], c[3];
    rgba_rgb(prev, i * 4, p);
    rgba_rgb(cur, i * 4, c);
    float pixel_abs = 0.0f;
    for (int ch = 0; ch < 3; ++ch) {
      const float d = c[ch] - p[ch];
      channel_delta[ch] += d;
      pixel_abs += fabsf(d);
    }
    raw_abs += pixel_abs / 3.0f;
    luma_delta += rgb_luma(c) - rgb_luma(p);
  }
  for (int ch = 0; ch < 3; ++ch) channel_delta[ch] /= (float)pixels;
  luma_delta /= (float)pixels;
  float residual_abs = 0.0f;
  for (int64_t i = 0; i < pixels; ++i) {
    float p[3], c[3];
    rgba_rgb(prev, i * 4, p);
    rgba_rgb(cur, i * 4, c);
    float pixel_abs = 0.0f;
    for (int ch = 0; ch < 3; ++ch) pixel_abs += fabsf(c[ch] - p[ch] - channel_delta[ch]);
    residual_abs += pixel_abs / 3.0f;
  }
  raw_abs = raw_abs / (float)pixels;
  residual_abs = residual_abs / (float)pixels;
  out->channel_delta[0] = channel_delta[0];
  out->channel_delta[1] = channel_delta[1];
  out->channel_delta[2] = channel_delta[2];
  out->luma_delta = luma_delta;
  out->compensate_global_lighting = raw_abs > 1.0e-4f && residual_abs <= raw_abs * 0.35f;
  out->raw_abs = raw_abs;
  out->residual_abs = residual_abs;
}

/* :1216-1244  rgba_patch_diff_pixel_score */
static float rgba_pixel_score(const uint8_t* prev, const uint8_t* cur, int64_t offset, const bjo_rgba_frame_stats* st) {
  float p[3], c[3];
  rgba_rgb(prev, offset, p);
  rgba_rgb(cur, offset, c);
  float rgb_abs = 0.0f;
  for (int ch = 0; ch < 3; ++ch) {
    float d = c[ch] - p[ch];
    if (st->compensate_global_lighting) d -= st->channel_delta[ch];
    rgb_abs += fabsf(d);
  }
  rgb_abs = rgb_abs / 3.0f;
  const float pl = rgb_luma(p), cl = rgb_luma(c);
  float ld = cl - pl;
  if (st->compensate_global_lighting) ld -= st->luma_delta;
  const float luma_abs = fabsf(ld);
  float rel = luma_abs / fmax_rust(fmax_rust(pl, cl), 0.10f);
  if (rel > 1.0f) rel = 1.0f;
  rel = rel * 0.25f;
  const float chroma = rgb_chroma_diff(p, c) * 0.5f;
  return fmax_rust(fmax_rust(fmax_rust(rgb_abs, luma_abs), rel), chroma);
}

/* :1126-1157 and :1199-1214  patch_diff_scores_from_rgba */
int bjo_patch_diff_scores_from_rgba(const uint8_t* prev, int64_t prev_len, const uint8_t* cur, int64_t cur_len,
                                    int64_t width, int64_t patch_size, int64_t depth, int64_t gh, int64_t gw,
                                    float* scores, bjo_rgba_frame_stats* stats_out) {
  if (depth != 1) return BJO_E_BAD_ARG;
  if (patch_size <= 0) return BJO_E_BAD_ARG;
  if (width != gw * patch_size) return BJO_E_BAD_ARG;
  const int64_t expected = width * gh * patch_size * 4;
  if (prev_len < expected || cur_len < expected) return BJO_E_BAD_ARG;
  bjo_rgba_frame_stats st;
  bjo_rgba_patch_diff_frame_stats(prev, prev_len, cur, cur_len, &st);
  if (stats_out) *stats_out = st;
  for (int64_t row = 0; row < gh; ++row)
    for (int64_t col = 0; col < gw; ++col) {
      float sum = 0.0f;
      for (int64_t y = row * patch_size; y < (row + 1) * patch_size; ++y)
        for (int64_t x = col * patch_size; x < (col + 1) * patch_size; ++x)
          sum += rgba_pixel_score(prev, cur, (y * width + x) * 4, &st);
      scores[row * gw + col] = sum / (float)(patch_size * patch_size);
    }
  return BJO_OK;
}

/* :780-793  patch_diff_dense_fallback: the mask, or every token when it is already at least
 * ceil(len * density) long (and that is below the grid). Returns the new length. */
int64_t bjo_patch_diff_dense_fallback(const int64_t* idx, int64_t n, int64_t dense_len, float density, int64_t* out) {
  if (density < 0.0f) density = 0.0f;
  if (density > 1.0f) density = 1.0f;
  /* `as usize` saturates: a NaN density gives 0 tokens */
  const int64_t fallback = density != density ? 0 : (int64_t)ceilf((float)dense_len * density);
  const int64_t at_least = fallback > 1 ? fallback : 1;
  if (n == dense_len || (fallback < dense_len && n >= at_least)) {
    for (int64_t i = 0; i < dense_len; ++i) out[i] = i;
    return dense_len;
  }
  for (int64_t i = 0; i < n; ++i) out[i] = idx[i];
  return n;
}

/* :796-816 and :844-869  dilate_sparse_patch_mask: every token within `dilation` tiles of a
 * mask token (same tubelet), sorted and unique; no cap. Returns the new length. */
int64_t bjo_dilate_sparse_patch_mask(const int64_t* idx, int64_t n, int64_t depth, int64_t gh, int64_t gw,
                                     int64_t dilation, int64_t* out) {
  const int64_t len = depth * gh * gw;
  int dense_ordered = n == len;
  for (int64_t i = 0; dense_ordered && i < n; ++i) dense_ordered = idx[i] == i;
  if (dilation == 0 || dense_ordered) {
    for (int64_t i = 0; i < n; ++i) out[i] = idx[i];
    return n;
  }
  unsigned char* keep = (unsigned char*)calloc((size_t)(len > 0 ? len : 1), 1);
  if (!keep) return -1;
  const int64_t tpf = gh * gw > 0 ? gh * gw : 1;
  for (int64_t k = 0; k < n; ++k) {
    const int64_t index = idx[k];
    if (index < 0 || index >= len) continue;
    const int64_t t = index / tpf, local = index % tpf;
    const int64_t row = local / (gw > 0 ? gw : 1), col = local % (gw > 0 ? gw : 1);
    const int64_t r0 = row > dilation ? row - dilation : 0, c0 = col > dilation ? col - dilation : 0;
    const int64_t r1 = row + dilation < gh - 1 ? row + dilation : gh - 1;
    const int64_t c1 = col + dilation < gw - 1 ? col + dilation : gw - 1;
    for (int64_t r = r0; r <= r1; ++r)
      for (int64_t c = c0; c <= c1; ++c) keep[t * tpf + r * gw + c] = 1;
  }
  int64_t m = 0;
  for (int64_t i = 0; i < len; ++i)
    if (keep[i]) out[m++] = i;
  free(keep);
  return m;
}

/* :873-885  bucket_sparse_mask: padded_to_multiple(min(bucket, max(len / 4, 1))) for grids of at
 * least 256 tokens that are not dense-ordered. Returns the new length. */
int64_t bjo_bucket_sparse_mask(const int64_t* idx, int64_t n, int64_t dense_len, int64_t bucket_tokens, int64_t* out) {
  int dense_ordered = n == dense_len;
  for (int64_t i = 0; dense_ordered && i < n; ++i) dense_ordered = idx[i] == i;
  if (bucket_tokens <= 1 || dense_len < 256 || dense_ordered || n >= dense_len) {
    for (int64_t i = 0; i < n; ++i) out[i] = idx[i];
    return n;
  }
  int64_t quarter = dense_len / 4 > 1 ? dense_len / 4 : 1;
  const int64_t bucket = bucket_tokens < quarter ? bucket_tokens : quarter;
  int64_t target = (n + bucket - 1) / bucket * bucket;
  if (target > dense_len) target = dense_len;
  return bjo_padded_to_len(idx, n, dense_len, target, out);
}

/* training/mask.rs:557-563 */
uint64_t bjo_splitmix64(uint64_t value) {
  value += 0x9e3779b97f4a7c15ULL;
  uint64_t m = value;
  m = (m ^ (m >> 30)) * 0xbf58476d1ce4e5b9ULL;
  m = (m ^ (m >> 27)) * 0x94d049bb133111ebULL;
  return m ^ (m >> 31);
}
