// bjf.hpp -- C++ host API of the B200 sparse front end, layered on the C ABI in bjf.h.
//
// It mirrors the Rust types and calls of burn_jepa 0.21.0 that a caller of the sparse
// front end uses, with the same names, argument meaning and error texts, so that code
// written against the reference reads the same here:
//
//   TokenGridShape, token_index_to_coords, coords_to_token_index   src/tokens.rs:5-32,
//                                                                  src/positional.rs:10-21
//   SparseTokenMask (+ make_context_target_masks, ...)             src/tokens.rs:34-179, 477-528
//   SparseJepaPatchDiffSparsityConfig                              src/nodes.rs:97-157
//   patch_diff_token_scores / patch_diff_context_mask_from_scores /
//   patch_diff_context_mask_from_video                             src/nodes.rs:411-631
//   SparsePatchifyPlan, SparsePatchifyBatchPlan                    src/sparse_patchify.rs:236-330
//   SparsePatchify3dConfig, sparse_patchify3d_forward_cuda         burn_flex_gmm 0.21.2, called at
//                                                                  src/model.rs:1297-1327
//   sparse_3d_sincos_pos_embed, sparse_patchify3d_encoder_input_cuda src/positional.rs:42-87,
//                                                                  src/model.rs:690-703
//   InterframeJepaFeatureMemory(Config) (+ update_tokens, reset_rows) src/feature_memory.rs:7-645
//   FrontEnd (one frame step over S streams)                       src/highres_pipeline.rs:2021-2040
//   patch_diff_scores_from_rgba, patch_diff_dense_fallback,
//   dilate_sparse_patch_mask, bucket_sparse_mask                   src/viewer.rs:780-885, 1067-1270
//
// Rust's Result<T> becomes a return value or a thrown bjf::Error carrying the status and
// the message (the reference's wording where it has one).  Device tensors are bjf::Tensor:
// an owning, contiguous device buffer with a dtype and a shape.  All work is enqueued on
// the caller's CUDA stream; functions that return host data (masks, to_host) synchronise
// that stream, as the reference's own readbacks do.
//
// Header-only C++17; link with libbjf.so and the CUDA runtime.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <memory>
#include <optional>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "bjf.h"

namespace bjf {

// ---------------------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------------------
class Error : public std::runtime_error {
 public:
  Error(bjf_status status, const std::string& message) : std::runtime_error(message), status_(status) {}
  bjf_status status() const { return status_; }

 private:
  bjf_status status_;
};

inline std::string last_error_string() {
  char buf[2048];
  bjf_get_last_error_string(buf, sizeof(buf));
  return std::string(buf);
}

// Throws the library's last error when `st` is not BJF_OK.
inline void check(bjf_status st) {
  if (st != BJF_OK) throw Error(st, last_error_string());
}

// The reference's `ensure!(cond, msg)`.
inline void ensure(bool cond, const char* message) {
  if (!cond) throw Error(BJF_ERR_INVALID_ARGUMENT, message);
}

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(BJF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

inline bjf_stream_t to_bjf(cudaStream_t s) { return reinterpret_cast<bjf_stream_t>(s); }

// ---------------------------------------------------------------------------------------
// token grid and index math (src/tokens.rs:5-32, src/positional.rs:10-21)
// ---------------------------------------------------------------------------------------
struct TokenGridShape {
  size_t depth = 0, height = 0, width = 0;

  constexpr TokenGridShape() = default;
  constexpr TokenGridShape(size_t d, size_t h, size_t w) : depth(d), height(h), width(w) {}
  static constexpr TokenGridShape new_(size_t d, size_t h, size_t w) { return TokenGridShape(d, h, w); }

  constexpr size_t len() const { return depth * height * width; }
  constexpr bool is_empty() const { return depth == 0 || height == 0 || width == 0; }
  constexpr size_t tokens_per_frame() const { return height * width; }
  constexpr bool operator==(const TokenGridShape& o) const {
    return depth == o.depth && height == o.height && width == o.width;
  }
  constexpr bool operator!=(const TokenGridShape& o) const { return !(*this == o); }
  std::array<int64_t, 3> dims() const { return {(int64_t)depth, (int64_t)height, (int64_t)width}; }
};

inline std::tuple<size_t, size_t, size_t> token_index_to_coords(size_t index, TokenGridShape grid) {
  const size_t tpf = std::max<size_t>(grid.tokens_per_frame(), 1);
  const size_t w = std::max<size_t>(grid.width, 1);
  const size_t frame = index / tpf;
  const size_t rem = index - frame * tpf;
  const size_t row = rem / w;
  return {frame, row, rem - row * w};
}

inline size_t coords_to_token_index(size_t frame, size_t row, size_t col, TokenGridShape grid) {
  return frame * grid.tokens_per_frame() + row * grid.width + col;
}

// ---------------------------------------------------------------------------------------
// SparseTokenMask (src/tokens.rs:34-179): sorted, unique token indices into a dense grid.
// ---------------------------------------------------------------------------------------
class SparseTokenMask {
 public:
  SparseTokenMask() = default;

  // Sorts and dedups; errors as SparseTokenMask::new (src/tokens.rs:41-50).
  static SparseTokenMask new_(std::vector<size_t> indices, size_t dense_len) {
    std::sort(indices.begin(), indices.end());
    indices.erase(std::unique(indices.begin(), indices.end()), indices.end());
    ensure(dense_len > 0, "dense token count must be nonzero");
    ensure(std::all_of(indices.begin(), indices.end(), [&](size_t i) { return i < dense_len; }),
           "sparse token index outside dense token range");
    return SparseTokenMask(std::move(indices), dense_len);
  }

  static SparseTokenMask from_keep_ratio(size_t dense_len, float keep_ratio) {
    const float r = std::min(std::max(keep_ratio, 0.0f), 1.0f);
    size_t keep = (size_t)std::ceil((float)dense_len * r);
    keep = std::min(std::max<size_t>(keep, 1), std::max<size_t>(dense_len, 1));
    std::vector<size_t> idx(keep);
    for (size_t i = 0; i < keep; ++i) idx[i] = i;
    return SparseTokenMask(std::move(idx), dense_len);
  }

  static std::vector<size_t> evenly_spaced_indices(size_t dense_len, size_t keep) {
    keep = std::min(std::max<size_t>(keep, 1), std::max<size_t>(dense_len, 1));
    std::vector<size_t> out;
    if (keep == dense_len) {
      for (size_t i = 0; i < dense_len; ++i) out.push_back(i);
      return out;
    }
    const size_t last = dense_len ? dense_len - 1 : 0;
    for (size_t i = 0; i < keep; ++i) out.push_back((i * last + keep / 2) / keep);
    return out;
  }

  static SparseTokenMask evenly_spaced(size_t dense_len, size_t keep) {
    return new_(evenly_spaced_indices(dense_len, keep), dense_len);
  }

  static SparseTokenMask all(size_t dense_len) {
    std::vector<size_t> idx(dense_len);
    for (size_t i = 0; i < dense_len; ++i) idx[i] = i;
    return SparseTokenMask(std::move(idx), dense_len);
  }

  bool is_dense_ordered() const {
    if (indices_.size() != dense_len_) return false;
    for (size_t i = 0; i < indices_.size(); ++i)
      if (indices_[i] != i) return false;
    return true;
  }

  // Keeps every index and adds evenly spaced ones, then the lowest missing ones, up to
  // target_len (src/tokens.rs:94-128).
  SparseTokenMask padded_to_len(size_t target_len) const {
    if (target_len <= indices_.size()) return *this;
    if (target_len >= dense_len_) return all(dense_len_);
    std::vector<bool> keep(dense_len_, false);
    std::vector<size_t> idx = indices_;
    for (size_t i : idx) keep[i] = true;
    for (size_t i : evenly_spaced_indices(dense_len_, target_len)) {
      if (!keep[i]) {
        keep[i] = true;
        idx.push_back(i);
        if (idx.size() >= target_len) break;
      }
    }
    for (size_t i = 0; idx.size() < target_len && i < dense_len_; ++i) {
      if (!keep[i]) {
        keep[i] = true;
        idx.push_back(i);
      }
    }
    return new_(std::move(idx), dense_len_);
  }

  SparseTokenMask padded_to_multiple(size_t multiple) const {
    if (multiple <= 1 || indices_.size() >= dense_len_) return *this;
    const size_t target = std::min((indices_.size() + multiple - 1) / multiple * multiple, dense_len_);
    return padded_to_len(target);
  }

  SparseTokenMask complement() const {
    std::vector<bool> keep(dense_len_, false);
    for (size_t i : indices_) keep[i] = true;
    std::vector<size_t> idx;
    for (size_t i = 0; i < dense_len_; ++i)
      if (!keep[i]) idx.push_back(i);
    return SparseTokenMask(std::move(idx), dense_len_);
  }

  const std::vector<size_t>& indices() const { return indices_; }
  size_t dense_len() const { return dense_len_; }
  size_t len() const { return indices_.size(); }
  bool is_empty() const { return indices_.empty(); }
  bool operator==(const SparseTokenMask& o) const { return dense_len_ == o.dense_len_ && indices_ == o.indices_; }

 private:
  SparseTokenMask(std::vector<size_t> idx, size_t dense_len) : indices_(std::move(idx)), dense_len_(dense_len) {}
  std::vector<size_t> indices_;
  size_t dense_len_ = 0;
};

inline std::vector<size_t> dense_token_indices(TokenGridShape grid) {
  return SparseTokenMask::all(grid.len()).indices();
}

inline std::vector<size_t> complement_indices(const std::vector<size_t>& indices, size_t dense_len) {
  return SparseTokenMask::new_(indices, dense_len).complement().indices();
}

inline std::pair<SparseTokenMask, SparseTokenMask> make_context_target_masks(TokenGridShape grid,
                                                                           float context_keep_ratio) {
  SparseTokenMask context = SparseTokenMask::from_keep_ratio(grid.len(), context_keep_ratio);
  SparseTokenMask target = context.complement();
  return {context, target};
}

// src/tokens.rs:497-528
inline SparseTokenMask target_mask_from_context(const SparseTokenMask& context, size_t target_tokens) {
  const size_t dense_len = context.dense_len();
  const size_t free = dense_len > context.len() ? dense_len - context.len() : 0;
  target_tokens = std::min(std::max<size_t>(target_tokens, 1), std::max<size_t>(free, 1));
  std::vector<bool> blocked(dense_len, false);
  for (size_t i : context.indices()) blocked[i] = true;
  std::vector<size_t> target;
  for (size_t i : SparseTokenMask::evenly_spaced_indices(dense_len, target_tokens))
    if (!blocked[i]) target.push_back(i);
  for (size_t i : target) blocked[i] = true;
  for (size_t i = 0; target.size() < target_tokens && i < dense_len; ++i) {
    if (!blocked[i]) {
      target.push_back(i);
      blocked[i] = true;
    }
  }
  return SparseTokenMask::new_(std::move(target), dense_len);
}

// ---------------------------------------------------------------------------------------
// device tensors
// ---------------------------------------------------------------------------------------
inline size_t dtype_bytes(bjf_dtype dt) {
  switch (dt) {
    case BJF_DTYPE_F32: return 4;
    case BJF_DTYPE_F16: return 2;
    case BJF_DTYPE_BF16: return 2;
    case BJF_DTYPE_I32: return 4;
  }
  return 0;
}

// Owning, contiguous device tensor.  Move-only.
class Tensor {
 public:
  Tensor() = default;
  Tensor(std::vector<int64_t> shape, bjf_dtype dtype) : shape_(std::move(shape)), dtype_(dtype) {
    const size_t bytes = nbytes();
    if (bytes) check_cuda(cudaMalloc(&ptr_, bytes), "cudaMalloc");
  }
  ~Tensor() { release(); }
  Tensor(const Tensor&) = delete;
  Tensor& operator=(const Tensor&) = delete;
  Tensor(Tensor&& o) noexcept { *this = std::move(o); }
  Tensor& operator=(Tensor&& o) noexcept {
    if (this != &o) {
      release();
      ptr_ = o.ptr_;
      shape_ = std::move(o.shape_);
      dtype_ = o.dtype_;
      o.ptr_ = nullptr;
      o.shape_.clear();
    }
    return *this;
  }

  static Tensor empty(std::vector<int64_t> shape, bjf_dtype dtype) { return Tensor(std::move(shape), dtype); }
  static Tensor zeros(std::vector<int64_t> shape, bjf_dtype dtype, cudaStream_t st = nullptr) {
    Tensor t(std::move(shape), dtype);
    if (t.nbytes()) check_cuda(cudaMemsetAsync(t.ptr_, 0, t.nbytes(), st), "cudaMemsetAsync");
    return t;
  }
  // Copies host elements whose in-memory form is `dtype` (float for F32, int32_t for I32,
  // uint16_t bit patterns for F16 / BF16).
  template <typename H>
  static Tensor from_host(const std::vector<H>& values, std::vector<int64_t> shape, bjf_dtype dtype,
                          cudaStream_t st = nullptr) {
    ensure(sizeof(H) == dtype_bytes(dtype), "host element size does not match the tensor dtype");
    Tensor t(std::move(shape), dtype);
    ensure(values.size() == t.numel(), "host data length does not match the tensor shape");
    if (t.nbytes()) {
      check_cuda(cudaMemcpyAsync(t.ptr_, values.data(), t.nbytes(), cudaMemcpyHostToDevice, st), "H2D copy");
      check_cuda(cudaStreamSynchronize(st), "H2D copy");
    }
    return t;
  }
  template <typename H>
  std::vector<H> to_host(cudaStream_t st = nullptr) const {
    ensure(sizeof(H) == dtype_bytes(dtype_), "host element size does not match the tensor dtype");
    std::vector<H> out(numel());
    if (nbytes()) {
      check_cuda(cudaMemcpyAsync(out.data(), ptr_, nbytes(), cudaMemcpyDeviceToHost, st), "D2H copy");
      check_cuda(cudaStreamSynchronize(st), "D2H copy");
    }
    return out;
  }
  Tensor clone(cudaStream_t st = nullptr) const {
    Tensor t(shape_, dtype_);
    if (nbytes()) check_cuda(cudaMemcpyAsync(t.ptr_, ptr_, nbytes(), cudaMemcpyDeviceToDevice, st), "D2D copy");
    return t;
  }

  // The same storage under another shape of as many elements (burn's Tensor::reshape).
  Tensor reshape(std::vector<int64_t> shape) && {
    Tensor t;
    t.shape_ = std::move(shape);
    t.dtype_ = dtype_;
    ensure(t.numel() == numel(), "reshape must keep the element count");
    t.ptr_ = ptr_;
    ptr_ = nullptr;
    shape_.clear();
    return t;
  }

  void* data() { return ptr_; }
  const void* data() const { return ptr_; }
  bjf_dtype dtype() const { return dtype_; }
  const std::vector<int64_t>& shape() const { return shape_; }
  size_t rank() const { return shape_.size(); }
  size_t numel() const {
    size_t n = 1;
    for (int64_t d : shape_) n *= (size_t)d;
    return shape_.empty() ? 0 : n;
  }
  size_t nbytes() const { return numel() * dtype_bytes(dtype_); }

 private:
  void release() {
    if (ptr_) cudaFree(ptr_);
    ptr_ = nullptr;
  }
  void* ptr_ = nullptr;
  std::vector<int64_t> shape_;
  bjf_dtype dtype_ = BJF_DTYPE_F32;
};

// ---------------------------------------------------------------------------------------
// patch-diff mask (src/nodes.rs:97-157, 411-631)
// ---------------------------------------------------------------------------------------
struct SparseJepaPatchDiffSparsityConfig {
  float threshold = 0.0f;
  size_t context_tokens = 0;
  size_t target_tokens = 0;
  size_t dilation = 0;
  size_t min_context_tokens = 1;
  bool fill_to_context_tokens = true;
  bool allow_full_context = false;

  static SparseJepaPatchDiffSparsityConfig new_(float threshold, size_t context_tokens, size_t target_tokens) {
    SparseJepaPatchDiffSparsityConfig c;
    c.threshold = threshold;
    c.context_tokens = context_tokens;
    c.target_tokens = target_tokens;
    return c;
  }
  static SparseJepaPatchDiffSparsityConfig adaptive_threshold(float threshold, size_t min_context_tokens,
                                                              size_t max_context_tokens, size_t target_tokens) {
    SparseJepaPatchDiffSparsityConfig c;
    c.threshold = threshold;
    c.context_tokens = max_context_tokens;
    c.target_tokens = target_tokens;
    c.min_context_tokens = min_context_tokens;
    c.fill_to_context_tokens = false;
    c.allow_full_context = true;
    return c;
  }
  SparseJepaPatchDiffSparsityConfig with_dilation(size_t v) const { auto c = *this; c.dilation = v; return c; }
  SparseJepaPatchDiffSparsityConfig with_min_context_tokens(size_t v) const {
    auto c = *this;
    c.min_context_tokens = v;
    return c;
  }
  SparseJepaPatchDiffSparsityConfig with_fill_to_context_tokens(bool v) const {
    auto c = *this;
    c.fill_to_context_tokens = v;
    return c;
  }
  SparseJepaPatchDiffSparsityConfig with_allow_full_context(bool v) const {
    auto c = *this;
    c.allow_full_context = v;
    return c;
  }

  bjf_patch_diff_config to_c() const {
    bjf_patch_diff_config c{};
    c.threshold = threshold;
    c.context_tokens = (int64_t)context_tokens;
    c.target_tokens = (int64_t)target_tokens;
    c.dilation = (int64_t)dilation;
    c.min_context_tokens = (int64_t)min_context_tokens;
    c.fill_to_context_tokens = fill_to_context_tokens ? 1 : 0;
    c.allow_full_context = allow_full_context ? 1 : 0;
    return c;
  }
};

namespace detail {
inline std::array<int64_t, 5> video_dims(const Tensor& video) {
  ensure(video.rank() == 5, "video must be a [B, C, T, H, W] tensor");
  std::array<int64_t, 5> d{};
  for (int i = 0; i < 5; ++i) d[i] = video.shape()[i];
  return d;
}
inline SparseTokenMask mask_from_device(const Tensor& indices, const Tensor& counts, size_t dense_len,
                                        cudaStream_t st) {
  const std::vector<int32_t> c = counts.to_host<int32_t>(st);
  const std::vector<int32_t> idx = indices.to_host<int32_t>(st);
  std::vector<size_t> v(idx.begin(), idx.begin() + c[0]);
  return SparseTokenMask::new_(std::move(v), dense_len);
}
}  // namespace detail

// Per-tubelet mean |frame difference|, the batch summed into one map: f32 [N].
// `tubelet_size` and `patch_size` are the model config's (VJepaConfig).
inline Tensor patch_diff_token_scores(const Tensor& video, size_t tubelet_size, size_t patch_size,
                                      TokenGridShape grid, cudaStream_t st = nullptr) {
  const auto d = detail::video_dims(video);
  const size_t kt = std::max<size_t>(tubelet_size, 1), p = std::max<size_t>(patch_size, 1);
  ensure(TokenGridShape((size_t)d[2] / kt, (size_t)d[3] / p, (size_t)d[4] / p) == grid,
         "patch-diff sparsity grid must match the video shape");
  Tensor scores({(int64_t)grid.len()}, BJF_DTYPE_F32);
  check(bjf_patch_diff_token_scores(video.data(), video.dtype(), d.data(), 1, (int64_t)kt, (int64_t)p,
                                    static_cast<float*>(scores.data()), to_bjf(st)));
  return scores;
}

// Host scores -> mask (the reference takes the scores as a Vec<f32>).
inline SparseTokenMask patch_diff_context_mask_from_scores(const std::vector<float>& score_values,
                                                          TokenGridShape grid,
                                                          const SparseJepaPatchDiffSparsityConfig& config,
                                                          cudaStream_t st = nullptr) {
  ensure(score_values.size() == grid.len(), "patch-diff sparsity received unexpected score length");
  const Tensor scores = Tensor::from_host(score_values, {(int64_t)grid.len()}, BJF_DTYPE_F32, st);
  Tensor indices({(int64_t)grid.len()}, BJF_DTYPE_I32);
  Tensor counts({1}, BJF_DTYPE_I32);
  const bjf_patch_diff_config c = config.to_c();
  const auto g = grid.dims();
  check(bjf_patch_diff_context_mask_from_scores(static_cast<const float*>(scores.data()), 1, g.data(), &c,
                                                static_cast<int32_t*>(indices.data()),
                                                static_cast<int32_t*>(counts.data()), to_bjf(st)));
  return detail::mask_from_device(indices, counts, grid.len(), st);
}

inline SparseTokenMask patch_diff_context_mask_from_video(const Tensor& video, size_t tubelet_size,
                                                         size_t patch_size, TokenGridShape grid,
                                                         const SparseJepaPatchDiffSparsityConfig& config,
                                                         cudaStream_t st = nullptr) {
  const auto d = detail::video_dims(video);
  const int64_t n = (int64_t)std::max<size_t>(grid.len(), 1);
  Tensor scores({n}, BJF_DTYPE_F32);
  Tensor indices({n}, BJF_DTYPE_I32);
  Tensor counts({1}, BJF_DTYPE_I32);
  const bjf_patch_diff_config c = config.to_c();
  const auto g = grid.dims();
  check(bjf_patch_diff_context_mask(video.data(), video.dtype(), d.data(), 1,
                                    (int64_t)std::max<size_t>(tubelet_size, 1),
                                    (int64_t)std::max<size_t>(patch_size, 1), g.data(), &c,
                                    static_cast<float*>(scores.data()), static_cast<int32_t*>(indices.data()),
                                    static_cast<int32_t*>(counts.data()), to_bjf(st)));
  return detail::mask_from_device(indices, counts, grid.len(), st);
}

// ---------------------------------------------------------------------------------------
// live viewer policy (src/viewer.rs): RGBA scorer and mask post-processing
// ---------------------------------------------------------------------------------------
constexpr float DEFAULT_PATCH_DIFF_QUALITY = 0.97f;                               // :19
constexpr float DEFAULT_PATCH_DIFF_THRESHOLD = 1.0f - DEFAULT_PATCH_DIFF_QUALITY;  // :25
constexpr float DEFAULT_PATCH_DIFF_DENSE_FALLBACK_DENSITY = 0.75f;                // :27
constexpr size_t DEFAULT_PATCH_DIFF_DILATION_TILES = 1;                           // :29
constexpr size_t DEFAULT_SPARSE_MASK_BUCKET_TOKENS = 256;                         // :31
constexpr float DEFAULT_CONTEXT_DENSITY = 1.0f;                                   // :17
constexpr float DEFAULT_MIN_CONTEXT_DENSITY = 0.0f;                               // :21
constexpr bool DEFAULT_PATCH_DIFF_REFRESH_ENABLED = false;                        // :35
constexpr float DEFAULT_PATCH_DIFF_SUBTHRESHOLD_DECAY = 0.92f;                    // :37
constexpr float DEFAULT_PATCH_DIFF_SUBTHRESHOLD_TRIGGER = 1.0f;                   // :39
constexpr float DEFAULT_PATCH_DIFF_SUBTHRESHOLD_MAX_DENSITY = 0.04f;              // :41
constexpr uint64_t DEFAULT_PATCH_DIFF_AGE_REFRESH_INTERVAL_FRAMES = 90;           // :43
constexpr float DEFAULT_PATCH_DIFF_AGE_REFRESH_MAX_DENSITY = 0.01f;               // :45
constexpr float DEFAULT_PATCH_DIFF_BLUE_NOISE_REFRESH_DENSITY = 0.005f;           // :47
constexpr float DEFAULT_PATCH_DIFF_REFRESH_MAX_DENSITY = 0.05f;                   // :49

// DensityRound / density_tokens (src/viewer.rs:732-752): a density of `dense_tokens` as a
// token count in 1 ..= dense_tokens.
enum class DensityRound { Floor, Round, Ceil };
inline size_t density_tokens(size_t dense_tokens, float density, DensityRound round, float min_density) {
  density = std::min(std::max(density, min_density), 1.0f);
  const float x = (float)dense_tokens * density;
  const float r = round == DensityRound::Floor ? std::floor(x) : (round == DensityRound::Round ? std::round(x)
                                                                                               : std::ceil(x));
  const size_t t = r > 0.0f ? (size_t)r : 0;  // `as usize` saturates at zero
  return std::min(std::max<size_t>(t, 1), std::max<size_t>(dense_tokens, 1));
}

using RgbaPatchDiffFrameStats = bjf_rgba_frame_stats;

// patch_diff_scores_from_rgba (src/viewer.rs:1126-1157) for `streams` frame pairs:
// prev / current are device RGBA u8 [streams, height, width, 4].  Returns scores
// [streams, grid.height * grid.width]; fills `stats` (host) when given.
inline Tensor patch_diff_scores_from_rgba(const uint8_t* prev, const uint8_t* current, size_t width, size_t height,
                                          size_t patch_size, TokenGridShape grid, size_t streams = 1,
                                          std::vector<RgbaPatchDiffFrameStats>* stats = nullptr,
                                          cudaStream_t st = nullptr) {
  const auto gd = grid.dims();
  // 0 for arguments the call below rejects with the reference's message
  const size_t ws_bytes = std::max<size_t>(bjf_rgba_patch_diff_workspace_bytes((int64_t)streams, gd.data()), 256);
  Tensor ws({(int64_t)((ws_bytes + 3) / 4)}, BJF_DTYPE_F32);
  Tensor scores({(int64_t)streams, (int64_t)(grid.height * grid.width)}, BJF_DTYPE_F32);
  void* dstats = nullptr;
  if (stats) check_cuda(cudaMalloc(&dstats, sizeof(RgbaPatchDiffFrameStats) * streams), "cudaMalloc");
  const bjf_status rc = bjf_rgba_patch_diff_scores(prev, current, (int64_t)streams, (int64_t)width, (int64_t)height,
                                                   (int64_t)patch_size, gd.data(), static_cast<float*>(scores.data()),
                                                   static_cast<bjf_rgba_frame_stats*>(dstats), ws.data(), ws.nbytes(),
                                                   to_bjf(st));
  if (rc != BJF_OK) {
    if (dstats) cudaFree(dstats);
    throw Error(rc, last_error_string());
  }
  if (stats) {
    stats->resize(streams);
    cudaError_t e = cudaMemcpyAsync(stats->data(), dstats, sizeof(RgbaPatchDiffFrameStats) * streams,
                                    cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(dstats);
    check_cuda(e, "RGBA stats readback");
  }
  return scores;
}

// patch_diff_dense_fallback (src/viewer.rs:780-793): every token once the mask reaches
// ceil(len * density) tokens (below the whole grid).
inline SparseTokenMask patch_diff_dense_fallback(SparseTokenMask mask, TokenGridShape grid, float fallback_density) {
  const float d = std::min(std::max(fallback_density, 0.0f), 1.0f);
  const size_t fallback = (size_t)std::ceil((float)grid.len() * d);
  if (mask.len() == grid.len() || (fallback < grid.len() && mask.len() >= std::max<size_t>(fallback, 1)))
    return SparseTokenMask::all(grid.len());
  return mask;
}

// dilate_sparse_patch_mask (src/viewer.rs:796-816, 844-869): every token within `dilation`
// tiles of a mask token in the same tubelet; no cap.
inline SparseTokenMask dilate_sparse_patch_mask(SparseTokenMask mask, TokenGridShape grid, size_t dilation) {
  ensure(mask.dense_len() == grid.len(), "patch-diff dilation mask must match the token grid");
  if (dilation == 0 || mask.is_dense_ordered()) return mask;
  std::vector<bool> keep(grid.len(), false);
  std::vector<size_t> selected;
  for (size_t index : mask.indices()) {
    if (index >= grid.len()) continue;
    const auto [t, row, col] = token_index_to_coords(index, grid);
    const size_t r0 = row > dilation ? row - dilation : 0, c0 = col > dilation ? col - dilation : 0;
    const size_t r1 = std::min(row + dilation, grid.height - 1), c1 = std::min(col + dilation, grid.width - 1);
    for (size_t r = r0; r <= r1; ++r)
      for (size_t c = c0; c <= c1; ++c) {
        const size_t i = coords_to_token_index(t, r, c, grid);
        if (!keep[i]) {
          keep[i] = true;
          selected.push_back(i);
        }
      }
  }
  return SparseTokenMask::new_(std::move(selected), grid.len());
}

// bucket_sparse_mask (src/viewer.rs:873-885): pad to a multiple of min(bucket, len / 4).
inline SparseTokenMask bucket_sparse_mask(SparseTokenMask mask, TokenGridShape grid, size_t bucket_tokens) {
  if (bucket_tokens <= 1 || grid.len() < 256 || mask.is_dense_ordered()) return mask;
  return mask.padded_to_multiple(std::min(bucket_tokens, std::max<size_t>(grid.len() / 4, 1)));
}

constexpr std::array<float, 3> DEFAULT_SPARSE_MASK_BUCKET_DENSITIES = {0.10f, 0.25f, 0.50f};  // :33

enum class FeatureFrameSparseEncodeMode { Exact, BucketedContext };  // src/viewer.rs:128-137

// sparse_mask_bucket_widths (src/viewer.rs:887-925), with density_tokens(.., Ceil, 0.0) (:739-752).
inline std::vector<size_t> sparse_mask_bucket_widths(TokenGridShape grid, size_t bucket_tokens,
                                                     const std::vector<float>& bucket_densities) {
  const size_t n = grid.len();
  if (n < 256) return {};
  std::vector<size_t> widths;
  if (bucket_densities.empty()) {
    if (bucket_tokens > 1) {
      const size_t bucket = std::min(bucket_tokens, std::max<size_t>(n / 4, 1));
      for (size_t w = bucket; w < n; w += bucket) widths.push_back(w);
    }
  } else {
    for (float d : bucket_densities)
      if (std::isfinite(d) && d > 0.0f) {
        const size_t t = (size_t)std::ceil((float)n * std::min(d, 1.0f));
        widths.push_back(std::min(std::max<size_t>(t, 1), std::max<size_t>(n, 1)));
      }
  }
  widths.push_back(n);
  std::sort(widths.begin(), widths.end());
  widths.erase(std::unique(widths.begin(), widths.end()), widths.end());
  return widths;
}

// PatchDiffRefreshConfig (src/viewer.rs:186-270): bounded extra cache writes for slow or
// stale tokens.  Off by default.
struct PatchDiffRefreshConfig {
  bool enabled = DEFAULT_PATCH_DIFF_REFRESH_ENABLED;
  bool subthreshold_enabled = false;
  float subthreshold_decay = DEFAULT_PATCH_DIFF_SUBTHRESHOLD_DECAY;
  float subthreshold_gain = 1.0f;
  float subthreshold_trigger = DEFAULT_PATCH_DIFF_SUBTHRESHOLD_TRIGGER;
  float subthreshold_max_density = DEFAULT_PATCH_DIFF_SUBTHRESHOLD_MAX_DENSITY;
  bool age_refresh_enabled = false;
  uint64_t age_refresh_interval_frames = DEFAULT_PATCH_DIFF_AGE_REFRESH_INTERVAL_FRAMES;
  float age_refresh_max_density = DEFAULT_PATCH_DIFF_AGE_REFRESH_MAX_DENSITY;
  bool blue_noise_enabled = false;
  float blue_noise_refresh_density = DEFAULT_PATCH_DIFF_BLUE_NOISE_REFRESH_DENSITY;
  uint64_t blue_noise_seed = 0x9e3779b97f4a7c15ull;
  float max_extra_density = DEFAULT_PATCH_DIFF_REFRESH_MAX_DENSITY;

  static PatchDiffRefreshConfig disabled() {
    PatchDiffRefreshConfig c;
    c.enabled = false;
    c.subthreshold_max_density = 0.0f;
    c.age_refresh_max_density = 0.0f;
    c.blue_noise_refresh_density = 0.0f;
    c.max_extra_density = 0.0f;
    return c;
  }
  bjf_patch_diff_refresh_config to_c() const {
    bjf_patch_diff_refresh_config c{};
    c.enabled = enabled;
    c.subthreshold_enabled = subthreshold_enabled;
    c.subthreshold_decay = subthreshold_decay;
    c.subthreshold_gain = subthreshold_gain;
    c.subthreshold_trigger = subthreshold_trigger;
    c.subthreshold_max_density = subthreshold_max_density;
    c.age_refresh_enabled = age_refresh_enabled;
    c.age_refresh_interval_frames = age_refresh_interval_frames;
    c.age_refresh_max_density = age_refresh_max_density;
    c.blue_noise_enabled = blue_noise_enabled;
    c.blue_noise_refresh_density = blue_noise_refresh_density;
    c.blue_noise_seed = blue_noise_seed;
    c.max_extra_density = max_extra_density;
    return c;
  }
  bool can_add_tokens() const {
    return enabled && max_extra_density > 0.0f &&
           ((subthreshold_enabled && subthreshold_max_density > 0.0f) ||
            (age_refresh_enabled && age_refresh_interval_frames > 0 && age_refresh_max_density > 0.0f) ||
            (blue_noise_enabled && blue_noise_refresh_density > 0.0f));
  }
};

// The patch-diff fields of FeatureFrameViewerConfig (src/viewer.rs:544-602) with their defaults.
struct FeatureFrameViewerConfig {
  float context_density = DEFAULT_CONTEXT_DENSITY;
  float min_context_density = DEFAULT_MIN_CONTEXT_DENSITY;
  float patch_diff_threshold = DEFAULT_PATCH_DIFF_THRESHOLD;
  PatchDiffRefreshConfig patch_diff_refresh;
  float patch_diff_dense_fallback_density = DEFAULT_PATCH_DIFF_DENSE_FALLBACK_DENSITY;
  size_t patch_diff_dilation_tiles = DEFAULT_PATCH_DIFF_DILATION_TILES;
  FeatureFrameSparseEncodeMode sparse_encode_mode = FeatureFrameSparseEncodeMode::BucketedContext;
  size_t sparse_mask_bucket_tokens = DEFAULT_SPARSE_MASK_BUCKET_TOKENS;
  std::vector<float> sparse_mask_bucket_densities{DEFAULT_SPARSE_MASK_BUCKET_DENSITIES.begin(),
                                                  DEFAULT_SPARSE_MASK_BUCKET_DENSITIES.end()};

  std::vector<size_t> sparse_mask_bucket_widths(TokenGridShape grid) const {
    return bjf::sparse_mask_bucket_widths(grid, sparse_mask_bucket_tokens, sparse_mask_bucket_densities);
  }
  // :649-667
  size_t context_tokens(size_t dense_tokens) const {
    return density_tokens(dense_tokens, context_density, DensityRound::Round, 0.01f);
  }
  size_t min_context_tokens(size_t dense_tokens) const {
    return density_tokens(dense_tokens, min_context_density, DensityRound::Ceil, 0.0f);
  }
  bjf_viewer_mask_policy to_c() const {
    ensure(sparse_mask_bucket_densities.size() <= 32, "viewer mask policy holds 0..32 bucket densities");
    bjf_viewer_mask_policy p{};
    p.dense_fallback_density = patch_diff_dense_fallback_density;
    p.dilation = (int64_t)patch_diff_dilation_tiles;
    p.bucketed_encode = sparse_encode_mode == FeatureFrameSparseEncodeMode::BucketedContext ? 1 : 0;
    p.bucket_tokens = (int64_t)sparse_mask_bucket_tokens;
    p.bucket_density_count = (int32_t)sparse_mask_bucket_densities.size();
    for (size_t i = 0; i < sparse_mask_bucket_densities.size(); ++i) p.bucket_densities[i] = sparse_mask_bucket_densities[i];
    return p;
  }
};

struct FeatureFrameSparseMasks {  // src/viewer.rs:762-769
  SparseTokenMask write_mask;
  SparseTokenMask encode_mask;
};

// bucket_sparse_mask_with_config (src/viewer.rs:927-944)
inline SparseTokenMask bucket_sparse_mask_with_config(SparseTokenMask mask, TokenGridShape grid,
                                                      const FeatureFrameViewerConfig& config) {
  if (grid.len() < 256 || mask.is_dense_ordered()) return mask;
  for (size_t w : config.sparse_mask_bucket_widths(grid))
    if (w >= mask.len()) return mask.padded_to_len(w);
  return mask;
}

// finalize_patch_diff_encode_masks (src/viewer.rs:946-961)
inline FeatureFrameSparseMasks finalize_patch_diff_encode_masks(SparseTokenMask write_mask, TokenGridShape grid,
                                                                const FeatureFrameViewerConfig& config) {
  SparseTokenMask encode = config.sparse_encode_mode == FeatureFrameSparseEncodeMode::Exact
                               ? write_mask
                               : bucket_sparse_mask_with_config(write_mask, grid, config);
  return {std::move(write_mask), std::move(encode)};
}

// finalize_patch_diff_masks (src/viewer.rs:963-971)
inline FeatureFrameSparseMasks finalize_patch_diff_masks(SparseTokenMask mask, TokenGridShape grid,
                                                         const FeatureFrameViewerConfig& config) {
  return finalize_patch_diff_encode_masks(
      patch_diff_dense_fallback(std::move(mask), grid, config.patch_diff_dense_fallback_density), grid, config);
}

// patch_diff_sparsity_config (src/viewer.rs:1012-1028): the selection a viewer config asks for.
inline SparseJepaPatchDiffSparsityConfig patch_diff_sparsity_config(const FeatureFrameViewerConfig& config,
                                                                    TokenGridShape grid) {
  const size_t max_context = config.context_tokens(grid.len());
  const size_t min_context = std::min(config.min_context_tokens(grid.len()), max_context);
  const size_t target = std::max<size_t>(grid.len() > max_context ? grid.len() - max_context : 0, 1);
  return SparseJepaPatchDiffSparsityConfig::adaptive_threshold(config.patch_diff_threshold, min_context,
                                                               max_context, target)
      .with_dilation(config.patch_diff_dilation_tiles);
}

// patch_diff_can_use_dense_fast_path (src/viewer.rs:1031-1036)
inline bool patch_diff_can_use_dense_fast_path(const SparseJepaPatchDiffSparsityConfig& config,
                                               TokenGridShape grid) {
  return config.threshold <= 0.0f && config.allow_full_context && config.context_tokens >= grid.len();
}

// patch_diff_base_mask_from_scores (src/viewer.rs:819-829): selection without dilation, dense
// fallback, then the sparsity config's dilation.
inline SparseTokenMask patch_diff_base_mask_from_scores(const std::vector<float>& scores, TokenGridShape grid,
                                                        const SparseJepaPatchDiffSparsityConfig& sparsity,
                                                        const FeatureFrameViewerConfig& config,
                                                        cudaStream_t st = nullptr) {
  SparseTokenMask direct = patch_diff_context_mask_from_scores(scores, grid, sparsity.with_dilation(0), st);
  direct = patch_diff_dense_fallback(std::move(direct), grid, config.patch_diff_dense_fallback_density);
  return dilate_sparse_patch_mask(std::move(direct), grid, sparsity.dilation);
}

// patch_diff_masks_from_scores (src/viewer.rs:831-841) for one frame's host scores.
inline FeatureFrameSparseMasks patch_diff_masks_from_scores(const std::vector<float>& scores, TokenGridShape grid,
                                                            const SparseJepaPatchDiffSparsityConfig& sparsity,
                                                            const FeatureFrameViewerConfig& config,
                                                            cudaStream_t st = nullptr) {
  return finalize_patch_diff_encode_masks(patch_diff_base_mask_from_scores(scores, grid, sparsity, config, st), grid,
                                          config);
}

// Device masks of S streams: row s of each [S, N] buffer holds its count of ascending indices.
struct DeviceSparseMasks {
  Tensor write_indices, write_counts, encode_indices, encode_counts;
  size_t dense_len = 0;

  FeatureFrameSparseMasks stream(size_t s, cudaStream_t st = nullptr) const {
    const auto wc = write_counts.to_host<int32_t>(st), ec = encode_counts.to_host<int32_t>(st);
    const auto wi = write_indices.to_host<int32_t>(st), ei = encode_indices.to_host<int32_t>(st);
    ensure(s < wc.size(), "stream index outside the masks");
    const auto row = [&](const std::vector<int32_t>& v, int32_t c) {
      return SparseTokenMask::new_(std::vector<size_t>(v.begin() + s * dense_len, v.begin() + s * dense_len + c),
                                   dense_len);
    };
    return {row(wi, wc[s]), row(ei, ec[s])};
  }
};

// patch_diff_masks_from_scores (src/viewer.rs:831-841) on device scores [S, N] f32: the
// selection of `sparsity` without its dilation, then dense fallback, sparsity.dilation and the
// encode buckets, all on the device.
inline DeviceSparseMasks patch_diff_masks_from_scores(const Tensor& scores, TokenGridShape grid,
                                                      const SparseJepaPatchDiffSparsityConfig& sparsity,
                                                      const FeatureFrameViewerConfig& config,
                                                      cudaStream_t st = nullptr) {
  const int64_t n = (int64_t)grid.len();
  ensure(scores.numel() > 0 && scores.numel() % n == 0, "patch-diff sparsity received unexpected score length");
  const int64_t S = scores.numel() / n;
  DeviceSparseMasks m{Tensor({S, n}, BJF_DTYPE_I32), Tensor({S}, BJF_DTYPE_I32), Tensor({S, n}, BJF_DTYPE_I32),
                      Tensor({S}, BJF_DTYPE_I32), (size_t)n};
  const bjf_patch_diff_config c = sparsity.to_c();
  const bjf_viewer_mask_policy p = config.to_c();
  const auto g = grid.dims();
  check(bjf_viewer_patch_diff_masks_from_scores(
      static_cast<const float*>(scores.data()), S, g.data(), &c, &p, static_cast<int32_t*>(m.write_indices.data()),
      static_cast<int32_t*>(m.write_counts.data()), static_cast<int32_t*>(m.encode_indices.data()),
      static_cast<int32_t*>(m.encode_counts.data()), to_bjf(st)));
  return m;
}

// patch_diff_mask_from_rgba without refresh state (crates/bevy_jepa/src/mask.rs:126-175) for
// `streams` device RGBA frame pairs [streams, height, width, 4]: the dense fast paths, else the
// RGBA scores and patch_diff_masks_from_scores, all on the device.
inline DeviceSparseMasks patch_diff_masks_from_rgba(const uint8_t* prev, const uint8_t* current, size_t width,
                                                    size_t height, size_t patch_size, TokenGridShape grid,
                                                    const SparseJepaPatchDiffSparsityConfig& sparsity,
                                                    const FeatureFrameViewerConfig& config, size_t streams = 1,
                                                    cudaStream_t st = nullptr) {
  const int64_t n = (int64_t)grid.len(), S = (int64_t)streams;
  const auto g = grid.dims();
  const size_t ws_bytes = bjf_viewer_rgba_masks_workspace_bytes(S, g.data());
  ensure(ws_bytes > 0, "RGBA viewer masks support 1..65535 streams and grids up to 32768 tokens");
  Tensor ws({(int64_t)((ws_bytes + 3) / 4)}, BJF_DTYPE_F32);
  DeviceSparseMasks m{Tensor({S, n}, BJF_DTYPE_I32), Tensor({S}, BJF_DTYPE_I32), Tensor({S, n}, BJF_DTYPE_I32),
                      Tensor({S}, BJF_DTYPE_I32), (size_t)n};
  const bjf_patch_diff_config c = sparsity.to_c();
  const bjf_viewer_mask_policy p = config.to_c();
  check(bjf_viewer_patch_diff_masks_from_rgba(
      prev, current, S, (int64_t)width, (int64_t)height, (int64_t)patch_size, g.data(), &c, &p,
      static_cast<int32_t*>(m.write_indices.data()), static_cast<int32_t*>(m.write_counts.data()),
      static_cast<int32_t*>(m.encode_indices.data()), static_cast<int32_t*>(m.encode_counts.data()), nullptr,
      ws.data(), ws.nbytes(), to_bjf(st)));
  return m;
}

// PatchDiffRefreshState (src/viewer.rs:275-528): per-stream residuals of below-threshold
// motion and token ages that add bounded refresh writes to the patch-diff masks.  The state of
// `streams` streams lives in device memory; each call advances every stream one frame inside
// the viewer mask launch (the selection, dense fallback, dilation, refresh ranking and encode
// buckets all run there), so a frame loop reads nothing back.  The host accessors copy one
// value back for inspection.
class PatchDiffRefreshState {
 public:
  explicit PatchDiffRefreshState(size_t streams = 1) : streams_(std::max<size_t>(streams, 1)) {}

  // The reference clears the buffers; the next frame starts over on zeros.
  void reset() { dense_len_ = 0; }
  size_t streams() const { return streams_; }
  uint64_t frame_index(size_t stream = 0) const {
    if (dense_len_ == 0) return 0;
    ensure(stream < streams_, "stream index outside the refresh state");
    const auto v = frame_.to_host<int32_t>();
    return (uint64_t)(uint32_t)v[2 * stream] | ((uint64_t)(uint32_t)v[2 * stream + 1] << 32);
  }
  std::optional<float> subthreshold_residual(size_t index, size_t stream = 0) const {
    if (index >= dense_len_ || stream >= streams_) return std::nullopt;
    return residual_.to_host<float>()[stream * dense_len_ + index];
  }
  std::optional<uint32_t> age_frames(size_t index, size_t stream = 0) const {
    if (index >= dense_len_ || stream >= streams_) return std::nullopt;
    return (uint32_t)age_.to_host<int32_t>()[stream * dense_len_ + index];
  }

  // observe_write_mask (:309-313) of one stream's host mask (a single-stream state).
  void observe_write_mask(const SparseTokenMask& mask, TokenGridShape grid, cudaStream_t st = nullptr) {
    ensure(streams_ == 1, "a host write mask belongs to a single-stream refresh state");
    std::vector<int32_t> idx(grid.len(), 0);
    for (size_t k = 0; k < mask.len(); ++k) idx[k] = (int32_t)mask.indices()[k];
    const Tensor wi = Tensor::from_host(idx, {1, (int64_t)grid.len()}, BJF_DTYPE_I32, st);
    const Tensor wc = Tensor::from_host(std::vector<int32_t>{(int32_t)mask.len()}, {1}, BJF_DTYPE_I32, st);
    observe_write_masks(wi, wc, grid, st);
  }
  // observe_write_mask of every stream: write_indices [S, N], write_counts [S] on the device.
  void observe_write_masks(const Tensor& write_indices, const Tensor& write_counts, TokenGridShape grid,
                           cudaStream_t st = nullptr) {
    bjf_patch_diff_refresh_state s = begin(grid, st);
    const auto g = grid.dims();
    check(bjf_viewer_patch_diff_refresh_observe(static_cast<const int32_t*>(write_indices.data()),
                                                static_cast<const int32_t*>(write_counts.data()), (int64_t)streams_,
                                                g.data(), &s, to_bjf(st)));
  }

  // masks_from_scores (:312-356) on device scores [S, N] f32.
  DeviceSparseMasks masks_from_scores(const Tensor& scores, TokenGridShape grid,
                                      const SparseJepaPatchDiffSparsityConfig& sparsity,
                                      const FeatureFrameViewerConfig& config, cudaStream_t st = nullptr) {
    const int64_t n = (int64_t)grid.len(), S = (int64_t)streams_;
    ensure(scores.numel() == (size_t)(S * n), "patch-diff refresh received unexpected score length");
    DeviceSparseMasks m{Tensor({S, n}, BJF_DTYPE_I32), Tensor({S}, BJF_DTYPE_I32), Tensor({S, n}, BJF_DTYPE_I32),
                        Tensor({S}, BJF_DTYPE_I32), (size_t)n};
    bjf_patch_diff_refresh_state s = begin(grid, st);
    const bjf_patch_diff_config c = sparsity.to_c();
    const bjf_viewer_mask_policy p = config.to_c();
    const bjf_patch_diff_refresh_config r = config.patch_diff_refresh.to_c();
    const auto g = grid.dims();
    check(bjf_viewer_patch_diff_refresh_masks_from_scores(
        static_cast<const float*>(scores.data()), S, g.data(), &c, &p, &r, &s,
        static_cast<int32_t*>(m.write_indices.data()), static_cast<int32_t*>(m.write_counts.data()),
        static_cast<int32_t*>(m.encode_indices.data()), static_cast<int32_t*>(m.encode_counts.data()), to_bjf(st)));
    return m;
  }

  // masks_from_scores of one stream's host scores (the reference's Vec<f32>).
  FeatureFrameSparseMasks masks_from_scores(const std::vector<float>& scores, TokenGridShape grid,
                                            const SparseJepaPatchDiffSparsityConfig& sparsity,
                                            const FeatureFrameViewerConfig& config, cudaStream_t st = nullptr) {
    ensure(streams_ == 1, "host scores belong to a single-stream refresh state");
    ensure(scores.size() == grid.len(), "patch-diff refresh received unexpected score length");
    const Tensor d = Tensor::from_host(scores, {1, (int64_t)grid.len()}, BJF_DTYPE_F32, st);
    return masks_from_scores(d, grid, sparsity, config, st).stream(0, st);
  }

  // The RGBA mask node with this state (crates/bevy_jepa/src/mask.rs:126-185) for device frame
  // pairs [S, height, width, 4].
  DeviceSparseMasks masks_from_rgba(const uint8_t* prev, const uint8_t* current, size_t width, size_t height,
                                    size_t patch_size, TokenGridShape grid,
                                    const SparseJepaPatchDiffSparsityConfig& sparsity,
                                    const FeatureFrameViewerConfig& config, cudaStream_t st = nullptr) {
    const int64_t n = (int64_t)grid.len(), S = (int64_t)streams_;
    const auto g = grid.dims();
    const size_t ws_bytes = bjf_viewer_rgba_masks_workspace_bytes(S, g.data());
    ensure(ws_bytes > 0, "RGBA viewer masks support 1..65535 streams and grids up to 32768 tokens");
    Tensor ws({(int64_t)((ws_bytes + 3) / 4)}, BJF_DTYPE_F32);
    DeviceSparseMasks m{Tensor({S, n}, BJF_DTYPE_I32), Tensor({S}, BJF_DTYPE_I32), Tensor({S, n}, BJF_DTYPE_I32),
                        Tensor({S}, BJF_DTYPE_I32), (size_t)n};
    bjf_patch_diff_refresh_state s = begin(grid, st);
    const bjf_patch_diff_config c = sparsity.to_c();
    const bjf_viewer_mask_policy p = config.to_c();
    const bjf_patch_diff_refresh_config r = config.patch_diff_refresh.to_c();
    check(bjf_viewer_patch_diff_refresh_masks_from_rgba(
        prev, current, S, (int64_t)width, (int64_t)height, (int64_t)patch_size, g.data(), &c, &p, &r, &s,
        static_cast<int32_t*>(m.write_indices.data()), static_cast<int32_t*>(m.write_counts.data()),
        static_cast<int32_t*>(m.encode_indices.data()), static_cast<int32_t*>(m.encode_counts.data()), nullptr,
        ws.data(), ws.nbytes(), to_bjf(st)));
    return m;
  }

 private:
  // begin_frame's start-over (:352-359): new zeroed buffers when the token count changes.
  bjf_patch_diff_refresh_state begin(TokenGridShape grid, cudaStream_t st) {
    const int64_t n = (int64_t)grid.len(), S = (int64_t)streams_;
    if (dense_len_ != grid.len()) {
      residual_ = Tensor::zeros({S, n}, BJF_DTYPE_F32, st);
      age_ = Tensor::zeros({S, n}, BJF_DTYPE_I32, st);
      frame_ = Tensor::zeros({2 * S}, BJF_DTYPE_I32, st);
      dense_len_ = grid.len();
    }
    return {static_cast<float*>(residual_.data()), static_cast<uint32_t*>(age_.data()),
            static_cast<uint64_t*>(frame_.data())};
  }

  size_t streams_ = 1;
  size_t dense_len_ = 0;
  Tensor residual_, age_, frame_;  // [S, N] f32, [S, N] u32 (as i32), [S] u64 (as 2 i32)
};

// ---------------------------------------------------------------------------------------
// plans (src/sparse_patchify.rs:236-330): coords rows (b, t, r, c), batch-major
// ---------------------------------------------------------------------------------------
class SparsePatchifyPlan {
 public:
  static SparsePatchifyPlan new_(SparseTokenMask mask, TokenGridShape grid, size_t batch,
                                 cudaStream_t st = nullptr) {
    ensure(batch > 0, "sparse patchify batch must be nonzero");
    ensure(mask.dense_len() == grid.len(), "sparse patchify mask dense token count must match grid");
    SparsePatchifyPlan p;
    p.grid = grid;
    p.batch = batch;
    for (size_t b = 0; b < batch; ++b)
      for (size_t index : mask.indices()) {
        const auto [t, r, c] = token_index_to_coords(index, grid);
        p.coords_host.push_back({(uint32_t)b, (uint32_t)t, (uint32_t)r, (uint32_t)c});
      }
    p.mask = std::move(mask);
    p.upload(st);
    return p;
  }
  static SparsePatchifyPlan from_indices(std::vector<size_t> indices, TokenGridShape grid, size_t batch,
                                         cudaStream_t st = nullptr) {
    return new_(SparseTokenMask::new_(std::move(indices), grid.len()), grid, batch, st);
  }
  // Host half only (no device coords): for callers that build coords on the device.
  static std::vector<std::array<uint32_t, 4>> host_coords(const SparseTokenMask& mask, TokenGridShape grid,
                                                          size_t batch) {
    ensure(batch > 0, "sparse patchify batch must be nonzero");
    ensure(mask.dense_len() == grid.len(), "sparse patchify mask dense token count must match grid");
    std::vector<std::array<uint32_t, 4>> out;
    for (size_t b = 0; b < batch; ++b)
      for (size_t index : mask.indices()) {
        const auto [t, r, c] = token_index_to_coords(index, grid);
        out.push_back({(uint32_t)b, (uint32_t)t, (uint32_t)r, (uint32_t)c});
      }
    return out;
  }

  size_t token_count() const { return mask.len(); }
  size_t output_rows() const { return batch * mask.len(); }

  SparseTokenMask mask;
  TokenGridShape grid;
  size_t batch = 0;
  Tensor coords;  // [batch * tokens, 4] int32, device
  std::vector<std::array<uint32_t, 4>> coords_host;

 private:
  void upload(cudaStream_t st) {
    std::vector<int32_t> flat;
    for (const auto& c : coords_host)
      for (uint32_t v : c) flat.push_back((int32_t)v);
    coords = Tensor::from_host(flat, {(int64_t)coords_host.size(), 4}, BJF_DTYPE_I32, st);
  }
};

// Per-row masks of equal width (uniform or fixed-width); ragged rows are refused as in
// SparsePatchifyBatchPlan::new (src/sparse_patchify.rs:290-330).
// SparseMaskBatch (src/tokens.rs:180-442): per-batch-row masks, Uniform (one mask repeated),
// FixedWidth (equal-length rows) or Ragged (rows padded with their last index).  Host rows;
// indices_tensor() uploads the [batch, width] int32 index matrix.
class SparseMaskBatch {
 public:
  enum class Kind { Uniform, FixedWidth, Ragged };

  static SparseMaskBatch uniform(SparseTokenMask mask, size_t batch) {
    ensure(batch > 0, "sparse mask batch must be non-empty");
    SparseMaskBatch m;
    m.kind_ = Kind::Uniform;
    m.dense_len_ = mask.dense_len();
    m.rows_.assign(batch, mask.indices());
    m.lengths_.assign(batch, mask.len());
    return m;
  }
  static SparseMaskBatch fixed_width(std::vector<std::vector<size_t>> rows, size_t dense_len) {
    ensure(dense_len > 0, "dense token count must be nonzero");
    ensure(!rows.empty(), "sparse mask batch must be non-empty");
    const size_t width = rows[0].size();
    ensure(width > 0, "fixed-width sparse mask rows must be non-empty");
    ensure(std::all_of(rows.begin(), rows.end(), [&](const std::vector<size_t>& r) { return r.size() == width; }),
           "fixed-width sparse mask rows must have equal lengths");
    for (auto& row : rows) {
      std::sort(row.begin(), row.end());
      row.erase(std::unique(row.begin(), row.end()), row.end());
      ensure(row.size() == width, "fixed-width sparse mask row contains duplicate indices");
      ensure(std::all_of(row.begin(), row.end(), [&](size_t i) { return i < dense_len; }),
             "sparse token index outside dense token range");
    }
    SparseMaskBatch m;
    m.kind_ = Kind::FixedWidth;
    m.dense_len_ = dense_len;
    m.lengths_.assign(rows.size(), width);
    m.rows_ = std::move(rows);
    return m;
  }
  static SparseMaskBatch from_rows(std::vector<std::vector<size_t>> rows, size_t dense_len) {
    ensure(!rows.empty(), "sparse mask batch must be non-empty");
    if (std::all_of(rows.begin(), rows.end(), [&](const std::vector<size_t>& r) { return r == rows[0]; }))
      return uniform(SparseTokenMask::new_(rows[0], dense_len), rows.size());
    if (std::all_of(rows.begin(), rows.end(), [&](const std::vector<size_t>& r) { return r.size() == rows[0].size(); }))
      return fixed_width(std::move(rows), dense_len);
    return ragged(std::move(rows), dense_len);
  }
  static SparseMaskBatch ragged(std::vector<std::vector<size_t>> rows, size_t dense_len) {
    ensure(dense_len > 0, "dense token count must be nonzero");
    ensure(!rows.empty(), "ragged sparse mask batch must be non-empty");
    SparseMaskBatch m;
    m.kind_ = Kind::Ragged;
    m.dense_len_ = dense_len;
    for (auto& row : rows) {
      std::sort(row.begin(), row.end());
      row.erase(std::unique(row.begin(), row.end()), row.end());
      ensure(!row.empty(), "ragged sparse mask rows must be non-empty");
      ensure(std::all_of(row.begin(), row.end(), [&](size_t i) { return i < dense_len; }),
             "sparse token index outside dense token range");
      m.lengths_.push_back(row.size());
    }
    m.rows_ = std::move(rows);
    return m;
  }

  size_t batch() const { return rows_.size(); }
  size_t dense_len() const { return dense_len_; }
  size_t len() const { return lengths_.empty() ? 0 : *std::max_element(lengths_.begin(), lengths_.end()); }
  bool is_empty() const { return len() == 0; }
  bool is_uniform() const { return kind_ == Kind::Uniform; }
  bool is_ragged() const { return kind_ == Kind::Ragged; }
  bool is_dense_ordered() const {
    if (kind_ == Kind::Ragged) return false;
    return std::all_of(rows_.begin(), rows_.end(), [&](const std::vector<size_t>& r) {
      if (r.size() != dense_len_) return false;
      for (size_t i = 0; i < r.size(); ++i)
        if (r[i] != i) return false;
      return true;
    });
  }
  size_t valid_token_count() const {
    size_t n = 0;
    for (size_t l : lengths_) n += l;
    return n;
  }
  std::optional<SparseTokenMask> uniform_mask() const {
    if (kind_ != Kind::Uniform) return std::nullopt;
    return SparseTokenMask::new_(rows_[0], dense_len_);
  }
  SparseTokenMask first_mask() const { return SparseTokenMask::new_(rows_[0], dense_len_); }
  const std::vector<std::vector<size_t>>& rows() const { return rows_; }
  // every row padded to len() with its last index (padded_rows_from_normalized, :444-454)
  std::vector<std::vector<size_t>> padded_rows() const {
    std::vector<std::vector<size_t>> out = rows_;
    const size_t w = len();
    for (auto& r : out)
      if (!r.empty()) r.resize(w, r.back());
    return out;
  }
  // 1 for a row's own tokens, 0 for its padding ([batch, len()]); ragged batches only (:405-426)
  std::optional<std::vector<float>> valid_token_mask() const {
    if (kind_ != Kind::Ragged) return std::nullopt;
    const size_t w = len();
    std::vector<float> v;
    for (size_t l : lengths_)
      for (size_t i = 0; i < w; ++i) v.push_back(i < l ? 1.0f : 0.0f);
    return v;
  }
  Tensor indices_tensor(cudaStream_t st = nullptr) const {
    std::vector<int32_t> flat;
    for (const auto& r : padded_rows())
      for (size_t i : r) flat.push_back((int32_t)i);
    return Tensor::from_host(flat, {(int64_t)batch(), (int64_t)len()}, BJF_DTYPE_I32, st);
  }

 private:
  Kind kind_ = Kind::Uniform;
  size_t dense_len_ = 0;
  std::vector<std::vector<size_t>> rows_;
  std::vector<size_t> lengths_;
};

class SparsePatchifyBatchPlan {
 public:
  // SparsePatchifyBatchPlan::new (src/sparse_patchify.rs:290-327)
  static SparsePatchifyBatchPlan new_(const SparseMaskBatch& mask, TokenGridShape grid, cudaStream_t st = nullptr) {
    ensure(mask.batch() > 0, "sparse patchify batch must be nonzero");
    ensure(!mask.is_ragged(),
           "sparse patchify batch plans require uniform or fixed-width masks; use ragged rollout grouping");
    ensure(mask.dense_len() == grid.len(), "sparse patchify batch mask dense token count must match grid");
    return from_rows(mask.rows(), grid, st);
  }
  static SparsePatchifyBatchPlan from_rows(std::vector<std::vector<size_t>> rows, TokenGridShape grid,
                                           cudaStream_t st = nullptr) {
    ensure(!rows.empty(), "sparse patchify batch must be nonzero");
    const size_t dense_len = grid.len();
    for (auto& row : rows) {
      std::sort(row.begin(), row.end());
      row.erase(std::unique(row.begin(), row.end()), row.end());
      ensure(std::all_of(row.begin(), row.end(), [&](size_t i) { return i < dense_len; }),
             "sparse token index outside dense token range");
    }
    const size_t width = rows[0].size();
    ensure(std::all_of(rows.begin(), rows.end(), [&](const std::vector<size_t>& r) { return r.size() == width; }),
           "sparse patchify batch plans require uniform or fixed-width masks; use ragged rollout grouping");
    ensure(width > 0, "fixed-width sparse mask rows must be non-empty");
    SparsePatchifyBatchPlan p;
    p.grid = grid;
    p.batch = rows.size();
    p.width = width;
    std::vector<int32_t> flat;
    for (size_t b = 0; b < rows.size(); ++b)
      for (size_t index : rows[b]) {
        const auto [t, r, c] = token_index_to_coords(index, grid);
        p.coords_host.push_back({(uint32_t)b, (uint32_t)t, (uint32_t)r, (uint32_t)c});
        flat.insert(flat.end(), {(int32_t)b, (int32_t)t, (int32_t)r, (int32_t)c});
      }
    p.rows = std::move(rows);
    p.coords = Tensor::from_host(flat, {(int64_t)p.coords_host.size(), 4}, BJF_DTYPE_I32, st);
    return p;
  }
  size_t token_count() const { return width; }
  size_t output_rows() const { return batch * width; }

  std::vector<std::vector<size_t>> rows;
  TokenGridShape grid;
  size_t batch = 0, width = 0;
  Tensor coords;
  std::vector<std::array<uint32_t, 4>> coords_host;
};

// The plan caches of the stream drivers (ensure_patchify_plan, src/temporal.rs:325-345, and
// cached_sparse_patchify_batch_plan, src/highres_pipeline.rs:2768-2793): a plan is rebuilt (and
// its coordinates uploaded) only when the mask rows, the grid or the batch change.
class SparsePatchifyPlanCache {
 public:
  // True when the cached plan already matches (nothing is rebuilt).
  bool ensure(const SparseTokenMask& mask, TokenGridShape grid, size_t batch, cudaStream_t st = nullptr) {
    if (plan_ && plan_->grid == grid && plan_->batch == batch && plan_->mask.dense_len() == mask.dense_len() &&
        plan_->mask.indices() == mask.indices())
      return true;
    plan_ = std::make_unique<SparsePatchifyPlan>(SparsePatchifyPlan::new_(mask, grid, batch, st));
    return false;
  }
  const SparsePatchifyPlan& plan() const {
    bjf::ensure(plan_ != nullptr, "sparse patchify plan cache is empty");
    return *plan_;
  }
  void reset() { plan_.reset(); }

 private:
  std::unique_ptr<SparsePatchifyPlan> plan_;
};

class SparsePatchifyBatchPlanCache {
 public:
  const SparsePatchifyBatchPlan& get(const SparseMaskBatch& mask, TokenGridShape grid, cudaStream_t st = nullptr) {
    if (!(plan_ && plan_->grid == grid && plan_->rows == mask.rows()))
      plan_ = std::make_unique<SparsePatchifyBatchPlan>(SparsePatchifyBatchPlan::new_(mask, grid, st));
    return *plan_;
  }
  void reset() { plan_.reset(); }

 private:
  std::unique_ptr<SparsePatchifyBatchPlan> plan_;
};

// ---------------------------------------------------------------------------------------
// sparse patchify (burn_flex_gmm::cuda::sparse_patchify3d_forward_cuda)
// ---------------------------------------------------------------------------------------
struct SparsePatchify3dConfig {
  size_t in_channels = 0, out_channels = 0, frames = 0, height = 0, width = 0;
  size_t tubelet_size = 0, patch_h = 0, patch_w = 0;

  bjf_patchify_config to_c() const {
    return bjf_patchify_config{(int64_t)in_channels, (int64_t)out_channels, (int64_t)frames, (int64_t)height,
                               (int64_t)width, (int64_t)tubelet_size, (int64_t)patch_h, (int64_t)patch_w};
  }
};

// out[M, D] = Conv3d(input, weight, stride = kernel) + bias at the coords rows.  `bias` may be
// null (zeros, as the reference's caller substitutes, src/model.rs:1307-1318).  The output
// dtype defaults to the input's.
inline Tensor sparse_patchify3d_forward_cuda(const SparsePatchify3dConfig& config, const Tensor& input,
                                             const Tensor& coords, const Tensor& weight, const Tensor* bias,
                                             cudaStream_t st = nullptr, int out_dtype = -1) {
  const auto d = detail::video_dims(input);
  ensure(weight.rank() == 5, "sparse patchify weight must be [D, C, kt, ph, pw]");
  ensure(coords.rank() == 2 && coords.shape()[1] == 4 && coords.dtype() == BJF_DTYPE_I32,
         "sparse patchify coords must be an int32 [M, 4] tensor");
  std::array<int64_t, 5> wd{};
  for (int i = 0; i < 5; ++i) wd[i] = weight.shape()[i];
  const bjf_patchify_config c = config.to_c();
  const bjf_dtype odt = out_dtype < 0 ? input.dtype() : (bjf_dtype)out_dtype;
  const int64_t rows = coords.shape()[0];
  Tensor out({rows, (int64_t)config.out_channels}, odt);
  check(bjf_sparse_patchify3d_forward(&c, input.data(), input.dtype(), d.data(),
                                      static_cast<const int32_t*>(coords.data()), rows, weight.data(),
                                      weight.dtype(), wd.data(),
                                      bias ? static_cast<const float*>(bias->data()) : nullptr, out.data(), odt,
                                      to_bjf(st)));
  return out;
}

// The sparse patch-embed methods of VJepaEncoder on the CUDA lane (src/model.rs:1092-1328): the
// checks of the input against the plan and the V-JEPA config, then the flex-gmm patch embed,
// reshaped to [batch, plan tokens, embed_dim].  `weight` [D, C, tubelet, P, P] (video) or
// [D, C, 1, P, P] (image, the tubelet-1 image embed); `bias` [D] f32 or null (zeros).
struct VJepaSparsePatchEmbed {
  size_t in_channels = 3, embed_dim = 0, tubelet_size = 2, patch_size = 16;

  // sparse_patchify_video_cuda (:1273-1328); video [B, C, T, H, W]
  Tensor sparse_patchify_video_cuda(const Tensor& video, const SparsePatchifyPlan& plan, const Tensor& weight,
                                    const Tensor* bias, cudaStream_t st = nullptr) const {
    const auto d = detail::video_dims(video);
    ensure((size_t)d[0] == plan.batch, "video batch does not match sparse patchify plan");
    ensure((size_t)d[1] == in_channels, "video channel count does not match V-JEPA config");
    const size_t kt = std::max<size_t>(tubelet_size, 1), p = std::max<size_t>(patch_size, 1);
    ensure(TokenGridShape((size_t)d[2] / kt, (size_t)d[3] / p, (size_t)d[4] / p) == plan.grid,
           "video token grid does not match sparse patchify plan");
    SparsePatchify3dConfig c;
    c.in_channels = (size_t)d[1];
    c.out_channels = embed_dim;
    c.frames = (size_t)d[2];
    c.height = (size_t)d[3];
    c.width = (size_t)d[4];
    c.tubelet_size = tubelet_size;
    c.patch_h = patch_size;
    c.patch_w = patch_size;
    return sparse_patchify3d_forward_cuda(c, video, plan.coords, weight, bias, st)
        .reshape({d[0], (int64_t)plan.token_count(), (int64_t)embed_dim});
  }

  // sparse_patchify_image_cuda (:1094-1148); image [B, C, H, W], one frame of tubelet 1
  Tensor sparse_patchify_image_cuda(const Tensor& image, const SparsePatchifyPlan& plan, const Tensor& weight,
                                    const Tensor* bias, cudaStream_t st = nullptr) const {
    ensure(image.rank() == 4, "image must be a [B, C, H, W] tensor");
    const auto& sh = image.shape();
    ensure((size_t)sh[0] == plan.batch, "image batch does not match sparse patchify plan");
    ensure((size_t)sh[1] == in_channels, "image channel count does not match V-JEPA config");
    const size_t p = std::max<size_t>(patch_size, 1);
    ensure(TokenGridShape(1, (size_t)sh[2] / p, (size_t)sh[3] / p) == plan.grid,
           "image token grid does not match sparse patchify plan");
    SparsePatchify3dConfig c;
    c.in_channels = (size_t)sh[1];
    c.out_channels = embed_dim;
    c.frames = 1;
    c.height = (size_t)sh[2];
    c.width = (size_t)sh[3];
    c.tubelet_size = 1;
    c.patch_h = patch_size;
    c.patch_w = patch_size;
    // the image as a one-frame clip [B, C, 1, H, W]: the same memory, a borrowed view
    const int64_t vd[5] = {sh[0], sh[1], 1, sh[2], sh[3]};
    ensure(weight.rank() == 5, "sparse patchify weight must be [D, C, kt, ph, pw]");
    std::array<int64_t, 5> wd{};
    for (int i = 0; i < 5; ++i) wd[i] = weight.shape()[i];
    const bjf_patchify_config cc = c.to_c();
    const int64_t rows = plan.coords.shape()[0];
    Tensor out({rows, (int64_t)embed_dim}, image.dtype());
    check(bjf_sparse_patchify3d_forward(&cc, image.data(), image.dtype(), vd,
                                        static_cast<const int32_t*>(plan.coords.data()), rows, weight.data(),
                                        weight.dtype(), wd.data(),
                                        bias ? static_cast<const float*>(bias->data()) : nullptr, out.data(),
                                        image.dtype(), to_bjf(st)));
    return std::move(out).reshape({sh[0], (int64_t)plan.token_count(), (int64_t)embed_dim});
  }
};

// sparse_3d_sincos_pos_embed (src/positional.rs:46-87): [indices.size(), embed_dim] f32 on the
// host, the frame / row / column sin-cos blocks of even(D/2), even(D/4), even(rest) dims.
inline std::vector<float> sparse_3d_sincos_pos_embed(size_t embed_dim, TokenGridShape grid,
                                                     const std::vector<size_t>& indices) {
  auto even = [](size_t d) { return d - (d % 2); };
  const size_t d_dim = even(embed_dim / 2), h_dim = even(embed_dim / 4);
  const size_t w_dim = even(embed_dim > d_dim + h_dim ? embed_dim - (d_dim + h_dim) : 0);
  const size_t rem = embed_dim > d_dim + h_dim + w_dim ? embed_dim - (d_dim + h_dim + w_dim) : 0;
  auto block = [](std::vector<float>& out, size_t dim, float pos) {
    if (dim == 0) return;
    const size_t half = dim / 2;
    const float h = (float)std::max<size_t>(half, 1);
    for (size_t i = 0; i < half; ++i) out.push_back(std::sin(pos * (1.0f / std::pow(10000.0f, (float)i / h))));
    for (size_t i = 0; i < half; ++i) out.push_back(std::cos(pos * (1.0f / std::pow(10000.0f, (float)i / h))));
    if (dim % 2 == 1) out.push_back(0.0f);
  };
  std::vector<float> out;
  out.reserve(indices.size() * embed_dim);
  for (size_t index : indices) {
    const auto [frame, row, col] = token_index_to_coords(index, grid);
    block(out, d_dim, (float)frame);
    block(out, h_dim, (float)row);
    block(out, w_dim, (float)col);
    out.insert(out.end(), rem, 0.0f);
  }
  return out;
}

inline std::vector<float> get_3d_sincos_pos_embed(size_t embed_dim, TokenGridShape grid) {
  return sparse_3d_sincos_pos_embed(embed_dim, grid, dense_token_indices(grid));
}

// The encoder's input tokens (src/model.rs:690-703): sparse_patchify3d_forward_cuda, then the
// row's position embedding (position_table [grid tokens, D] f32, nullable) and the modality
// embedding ([D] f32, nullable), in the reference's order, fused into the GEMM epilogue.
inline Tensor sparse_patchify3d_encoder_input_cuda(const SparsePatchify3dConfig& config, const Tensor& input,
                                                   const Tensor& coords, const Tensor& weight, const Tensor* bias,
                                                   const Tensor* position_table, const Tensor* modality_embed,
                                                   cudaStream_t st = nullptr, int out_dtype = -1) {
  const auto d = detail::video_dims(input);
  ensure(weight.rank() == 5, "sparse patchify weight must be [D, C, kt, ph, pw]");
  ensure(coords.rank() == 2 && coords.shape()[1] == 4 && coords.dtype() == BJF_DTYPE_I32,
         "sparse patchify coords must be an int32 [M, 4] tensor");
  std::array<int64_t, 5> wd{};
  for (int i = 0; i < 5; ++i) wd[i] = weight.shape()[i];
  const bjf_patchify_config c = config.to_c();
  const bjf_dtype odt = out_dtype < 0 ? input.dtype() : (bjf_dtype)out_dtype;
  const int64_t rows = coords.shape()[0];
  Tensor out({rows, (int64_t)config.out_channels}, odt);
  auto fptr = [](const Tensor* t) { return t ? static_cast<const float*>(t->data()) : nullptr; };
  check(bjf_sparse_patchify3d_forward_encoder_input(&c, input.data(), input.dtype(), d.data(),
                                                    static_cast<const int32_t*>(coords.data()), rows, weight.data(),
                                                    weight.dtype(), wd.data(), fptr(bias), fptr(position_table),
                                                    fptr(modality_embed), out.data(), odt, to_bjf(st)));
  return out;
}

// ---------------------------------------------------------------------------------------
// InterframeJepaFeatureMemory, AssignLatest mode (src/feature_memory.rs:137-645)
// ---------------------------------------------------------------------------------------
struct InterframeJepaFeatureMemoryOutput {
  const Tensor* features;  // [B, N, D]
  const Tensor* observed;  // [B, N] f32
  const Tensor* age_frames;  // [B, N] f32
  TokenGridShape grid;
  size_t step;
  size_t updated_tokens;
  size_t dense_tokens;
};

// InterframeJepaFeatureMemoryConfig (src/feature_memory.rs:7-49): AssignLatest or Ema { alpha }.
struct InterframeJepaFeatureMemoryConfig {
  enum class UpdateMode { AssignLatest, Ema };
  UpdateMode update_mode = UpdateMode::AssignLatest;
  float alpha = 0.0f;  // Ema only

  static InterframeJepaFeatureMemoryConfig assign_latest() { return {}; }
  static InterframeJepaFeatureMemoryConfig ema(float alpha) {
    InterframeJepaFeatureMemoryConfig c;
    c.update_mode = UpdateMode::Ema;
    c.alpha = alpha;
    return c;
  }
  // alpha clamped to [0, 1] (a NaN stays NaN), as the reference normalises it
  InterframeJepaFeatureMemoryConfig normalized() const {
    InterframeJepaFeatureMemoryConfig c = *this;
    if (c.alpha < 0.0f) c.alpha = 0.0f;
    if (c.alpha > 1.0f) c.alpha = 1.0f;
    return c;
  }
};

class InterframeJepaFeatureMemory {
 public:
  // `features_dtype` f32 as the reference, or f16 / bf16 for a half-size cache.
  static InterframeJepaFeatureMemory new_(size_t batch, TokenGridShape grid, size_t embed_dim,
                                          bjf_dtype features_dtype = BJF_DTYPE_F32, cudaStream_t st = nullptr) {
    return with_config(InterframeJepaFeatureMemoryConfig::assign_latest(), batch, grid, embed_dim, features_dtype,
                       st);
  }
  static InterframeJepaFeatureMemory with_config(const InterframeJepaFeatureMemoryConfig& config, size_t batch,
                                                 TokenGridShape grid, size_t embed_dim,
                                                 bjf_dtype features_dtype = BJF_DTYPE_F32, cudaStream_t st = nullptr) {
    ensure(batch > 0, "feature memory batch must be nonzero");
    ensure(!grid.is_empty(), "feature memory grid must be nonempty");
    ensure(embed_dim > 0, "feature memory embed dim must be nonzero");
    InterframeJepaFeatureMemory m;
    m.config_ = config.normalized();
    m.batch_ = batch;
    m.grid_ = grid;
    m.embed_dim_ = embed_dim;
    const int64_t B = (int64_t)batch, N = (int64_t)grid.len(), D = (int64_t)embed_dim;
    m.features_ = Tensor::zeros({B, N, D}, features_dtype, st);
    m.observed_ = Tensor::zeros({B, N}, BJF_DTYPE_F32, st);
    m.age_frames_ = Tensor::zeros({B, N}, BJF_DTYPE_F32, st);
    return m;
  }

  size_t batch() const { return batch_; }
  TokenGridShape grid() const { return grid_; }
  size_t dense_tokens() const { return grid_.len(); }
  size_t embed_dim() const { return embed_dim_; }
  size_t step() const { return step_; }
  InterframeJepaFeatureMemoryConfig config() const { return config_; }
  InterframeJepaFeatureMemoryOutput snapshot() const { return output(last_updated_tokens_); }
  Tensor& features() { return features_; }
  Tensor& observed() { return observed_; }
  Tensor& age_frames() { return age_frames_; }

  // update_tokens (src/feature_memory.rs:227-290) in the configured mode, on the device.
  InterframeJepaFeatureMemoryOutput update_tokens(const Tensor& tokens, const Tensor& token_indices,
                                                  TokenGridShape grid, cudaStream_t st = nullptr) {
    return update_tokens_tiled_assign_cuda(tokens, token_indices, grid, st);
  }

  // tokens [B, S, D], token_indices [B, S] int32.  In place (the reference copies the cache
  // first; a caller that keeps the previous snapshot clones it before this call).  In EMA
  // mode the reference falls back to its portable update (src/feature_memory.rs:624-626);
  // here the EMA update runs on the device too.
  InterframeJepaFeatureMemoryOutput update_tokens_tiled_assign_cuda(const Tensor& tokens,
                                                                   const Tensor& token_indices,
                                                                   TokenGridShape grid, cudaStream_t st = nullptr) {
    ensure(grid == grid_, "encoder output grid does not match feature memory grid");
    ensure(tokens.rank() == 3 && token_indices.rank() == 2, "tokens must be [B, S, D] and indices [B, S]");
    const int64_t b = tokens.shape()[0], s = tokens.shape()[1], d = tokens.shape()[2];
    ensure((size_t)b == batch_, "encoder output batch does not match feature memory batch");
    ensure((size_t)d == embed_dim_, "encoder output dim does not match feature memory dim");
    ensure(token_indices.shape()[0] == b && token_indices.shape()[1] == s,
           "token index shape must match sparse encoder token shape");
    ensure(s > 0, "sparse update must include at least one token");
    ensure(token_indices.dtype() == BJF_DTYPE_I32, "token indices must be int32");
    const int64_t fd[3] = {features_.shape()[0], features_.shape()[1], features_.shape()[2]};
    const int64_t od[2] = {observed_.shape()[0], observed_.shape()[1]};
    const int64_t ad[2] = {age_frames_.shape()[0], age_frames_.shape()[1]};
    const int64_t td[3] = {b, s, d};
    const int64_t id[2] = {b, s};
    if (config_.update_mode == InterframeJepaFeatureMemoryConfig::UpdateMode::Ema)
      check(bjf_feature_memory_update_ema(features_.data(), features_.dtype(), fd,
                                          static_cast<float*>(observed_.data()), od,
                                          static_cast<float*>(age_frames_.data()), ad, tokens.data(), tokens.dtype(),
                                          td, static_cast<const int32_t*>(token_indices.data()), id, config_.alpha,
                                          step_ > 0 ? 1 : 0, to_bjf(st)));
    else
      check(bjf_feature_memory_assign_latest(features_.data(), features_.dtype(), fd,
                                             static_cast<float*>(observed_.data()), od,
                                             static_cast<float*>(age_frames_.data()), ad, tokens.data(),
                                             tokens.dtype(), td, static_cast<const int32_t*>(token_indices.data()),
                                             id, step_ > 0 ? 1 : 0, to_bjf(st)));
    step_ += 1;
    last_updated_tokens_ = (size_t)(b * s);
    return output(last_updated_tokens_);
  }

  // update_masked_tokens with the tiled assign: one mask shared by every batch row.
  InterframeJepaFeatureMemoryOutput update_masked_tokens_tiled_assign_cuda(const Tensor& tokens,
                                                                          const SparseTokenMask& mask,
                                                                          TokenGridShape grid,
                                                                          cudaStream_t st = nullptr) {
    ensure(mask.dense_len() == dense_tokens(), "sparse mask dense length must match feature memory grid");
    std::vector<int32_t> idx;
    for (size_t b = 0; b < batch_; ++b)
      for (size_t i : mask.indices()) idx.push_back((int32_t)i);
    const Tensor ti = Tensor::from_host(idx, {(int64_t)batch_, (int64_t)mask.len()}, BJF_DTYPE_I32, st);
    return update_tokens_tiled_assign_cuda(tokens, ti, grid, st);
  }

  void reset(cudaStream_t st = nullptr) {
    check_cuda(cudaMemsetAsync(features_.data(), 0, features_.nbytes(), st), "cudaMemsetAsync");
    check_cuda(cudaMemsetAsync(observed_.data(), 0, observed_.nbytes(), st), "cudaMemsetAsync");
    check_cuda(cudaMemsetAsync(age_frames_.data(), 0, age_frames_.nbytes(), st), "cudaMemsetAsync");
    step_ = 0;
    last_updated_tokens_ = 0;
  }

  // reset_rows (src/feature_memory.rs:348-375): rows is a device int32 tensor [R]; rows outside
  // the batch are skipped.
  void reset_rows(const Tensor& rows, cudaStream_t st = nullptr) {
    ensure(rows.rank() == 1 && rows.dtype() == BJF_DTYPE_I32, "feature memory reset rows must be an int32 [R] tensor");
    if (rows.numel() == 0) return;
    const int64_t fd[3] = {features_.shape()[0], features_.shape()[1], features_.shape()[2]};
    check(bjf_feature_memory_reset_rows(features_.data(), features_.dtype(), fd, static_cast<float*>(observed_.data()),
                                        static_cast<float*>(age_frames_.data()),
                                        static_cast<const int32_t*>(rows.data()), (int64_t)rows.numel(), to_bjf(st)));
  }

  // Zeroes the features and metadata of the given batch rows (src/feature_memory.rs:377-385).
  void reset_row_indices(const std::vector<size_t>& rows, cudaStream_t st = nullptr) {
    if (rows.empty()) return;
    ensure(std::all_of(rows.begin(), rows.end(), [&](size_t r) { return r < batch_; }),
           "feature memory row reset index outside batch");
    const size_t N = dense_tokens();
    const size_t frow = N * embed_dim_ * dtype_bytes(features_.dtype());
    for (size_t r : rows) {
      check_cuda(cudaMemsetAsync(static_cast<char*>(features_.data()) + r * frow, 0, frow, st), "cudaMemsetAsync");
      check_cuda(cudaMemsetAsync(static_cast<float*>(observed_.data()) + r * N, 0, N * 4, st), "cudaMemsetAsync");
      check_cuda(cudaMemsetAsync(static_cast<float*>(age_frames_.data()) + r * N, 0, N * 4, st),
                 "cudaMemsetAsync");
    }
  }

 private:
  InterframeJepaFeatureMemoryOutput output(size_t updated) const {
    return {&features_, &observed_, &age_frames_, grid_, step_, updated, grid_.len()};
  }
  InterframeJepaFeatureMemoryConfig config_;
  size_t batch_ = 0, embed_dim_ = 0, step_ = 0, last_updated_tokens_ = 0;
  TokenGridShape grid_;
  Tensor features_, observed_, age_frames_;
};

// ---------------------------------------------------------------------------------------
// FrontEnd: one frame step over S independent streams, fully on the device
// (patch-diff scores -> selection -> gather-GEMM with bias -> in-place
// token-cache write; three kernels chained with programmatic dependent launch).
// ---------------------------------------------------------------------------------------
class FrontEnd {
 public:
  FrontEnd(size_t streams, size_t channels, size_t frames, size_t height, size_t width, size_t tubelet_size,
           size_t patch_size, size_t embed_dim, const SparseJepaPatchDiffSparsityConfig& mask,
           bjf_dtype video_dtype, bjf_dtype cache_dtype, cudaStream_t st = nullptr) {
    desc_.streams = (int64_t)streams;
    desc_.channels = (int64_t)channels;
    desc_.frames = (int64_t)frames;
    desc_.height = (int64_t)height;
    desc_.width = (int64_t)width;
    desc_.tubelet_size = (int64_t)tubelet_size;
    desc_.patch_size = (int64_t)patch_size;
    desc_.embed_dim = (int64_t)embed_dim;
    desc_.video_dtype = video_dtype;
    desc_.weight_dtype = video_dtype;
    desc_.cache_dtype = cache_dtype;
    desc_.mask = mask.to_c();
    const size_t ws = bjf_front_end_workspace_bytes(&desc_);
    if (ws == 0) throw Error(BJF_ERR_INVALID_ARGUMENT, last_error_string());
    grid_ = TokenGridShape(frames / tubelet_size, height / patch_size, width / patch_size);
    workspace_ = Tensor::empty({(int64_t)((ws + 3) / 4)}, BJF_DTYPE_F32);  // cudaMalloc: 256-byte aligned
    counts_ = Tensor::zeros({(int64_t)streams}, BJF_DTYPE_I32, st);
    caches_ = Tensor::zeros({(int64_t)streams, (int64_t)grid_.len(), (int64_t)embed_dim}, cache_dtype, st);
    observed_ = Tensor::zeros({(int64_t)streams, (int64_t)grid_.len()}, BJF_DTYPE_F32, st);
    age_ = Tensor::zeros({(int64_t)streams, (int64_t)grid_.len()}, BJF_DTYPE_F32, st);
  }

  // video [S, C, T, H, W] (one clip per stream), weight [D, C, kt, P, P] (video dtype),
  // bias [D] f32 or null.  Returns the per-stream active counts (device [S] int32).
  const Tensor& step(const Tensor& video, const Tensor& weight, const Tensor* bias, cudaStream_t st = nullptr) {
    check(bjf_front_end_step(&desc_, video.data(), weight.data(), bias ? static_cast<const float*>(bias->data()) : nullptr,
                             caches_.data(), static_cast<float*>(observed_.data()), static_cast<float*>(age_.data()),
                             steps_ > 0 ? 1 : 0, workspace_.data(), workspace_.nbytes(),
                             static_cast<int32_t*>(counts_.data()), to_bjf(st)));
    ++steps_;
    return counts_;
  }

  // The live step on a frame ring [S, C, R, H, W] (frames = tubelet = 2): the clip is
  // (ring[prev_slot], ring[cur_slot]); results as step() on that clip.
  const Tensor& step_ring(const Tensor& ring, int32_t prev_slot, int32_t cur_slot, const Tensor& weight,
                          const Tensor* bias, cudaStream_t st = nullptr) {
    if (ring.shape().size() != 5) throw Error(BJF_ERR_INVALID_ARGUMENT, "frame ring must be [S, C, R, H, W]");
    check(bjf_front_end_step_ring(&desc_, ring.data(), (int32_t)ring.shape()[2], prev_slot, cur_slot, weight.data(),
                                  bias ? static_cast<const float*>(bias->data()) : nullptr, caches_.data(),
                                  static_cast<float*>(observed_.data()), static_cast<float*>(age_.data()),
                                  steps_ > 0 ? 1 : 0, workspace_.data(), workspace_.nbytes(),
                                  static_cast<int32_t*>(counts_.data()), to_bjf(st)));
    ++steps_;
    return counts_;
  }

  TokenGridShape grid() const { return grid_; }
  size_t steps() const { return steps_; }
  Tensor& caches() { return caches_; }
  Tensor& observed() { return observed_; }
  Tensor& age_frames() { return age_; }
  const bjf_front_end_desc& desc() const { return desc_; }

 private:
  bjf_front_end_desc desc_{};
  TokenGridShape grid_;
  size_t steps_ = 0;
  Tensor workspace_, counts_, caches_, observed_, age_;
};

// Reports (and clears) a bounded-wait timeout recorded by any kernel of the library.
inline bool device_error_check(cudaStream_t st = nullptr) {
  int32_t flag = 0;
  check(bjf_device_error_check(to_bjf(st), &flag));
  return flag != 0;
}

}  // namespace bjf
