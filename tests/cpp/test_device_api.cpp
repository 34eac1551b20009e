// test_device_api.cpp -- ports of the reference's own device-path tests onto the C++ API of
// include/bjf.hpp, checked against the reference's known answers and, for the patch-embed
// arithmetic, against the CPU oracle (oracle/bjf_oracle.h, test infrastructure).
// Needs a CUDA GPU (sm_100a).
#include <cstring>
#include <set>

#include "../../include/bjf.hpp"
#include "../../oracle/bjf_oracle.h"
#include "check.hpp"

using namespace bjf;

namespace {

// IEEE 754 binary16 / bfloat16 encodings with round-to-nearest-even (from the formats'
// definitions; host-side test data only).
uint16_t f32_to_f16_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t e8 = (int32_t)((x >> 23) & 0xffu);
  uint32_t mant = x & 0x7fffffu;
  if (e8 == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
  const int32_t e = e8 - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    const int shift = 14 - e;
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}

float f16_bits_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, mant = h & 0x3ffu;
  if (e == 0) {
    const float v = std::ldexp((float)mant, -24);
    return sign ? -v : v;
  }
  const uint32_t x = sign | (e == 31 ? 0x7f800000u | (mant << 13) : ((e - 15 + 127) << 23) | (mant << 13));
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

uint16_t f32_to_bf16_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}

float bf16_bits_to_f32(uint16_t h) {
  const uint32_t x = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// Seeded uniform[-1, 1) from the reference's splitmix64 mixer.
std::vector<float> seeded(uint64_t seed, size_t n, float scale) {
  std::vector<float> v(n);
  for (size_t i = 0; i < n; ++i) {
    const uint64_t z = bjo_splitmix64(seed + 0x9E3779B97F4A7C15ull * (i + 1));
    v[i] = scale * (float)((double)(z >> 40) * (1.0 / 8388608.0) - 1.0);
  }
  return v;
}

float max_abs_diff(const std::vector<float>& a, const std::vector<float>& b) {
  float m = 0.0f;
  for (size_t i = 0; i < a.size(); ++i) m = std::max(m, std::fabs(a[i] - b[i]));
  return m;
}

float max_rel_err(const std::vector<float>& got, const std::vector<float>& ref) {
  float den = 1e-30f;
  for (float r : ref) den = std::max(den, std::fabs(r));
  return max_abs_diff(got, ref) / den;
}

std::vector<float> host_f32(const Tensor& t) { return t.to_host<float>(); }

// Dense Conv3d patch embed (oracle) gathered at the plan's coords rows.
std::vector<float> dense_at_coords(const bjo_patchify_config& cfg, int64_t batch, const std::vector<float>& video,
                                   const std::vector<float>& weight, const std::vector<float>& bias,
                                   const std::vector<std::array<uint32_t, 4>>& coords) {
  const int64_t gd = cfg.frames / cfg.tubelet_size, gh = cfg.height / cfg.patch_h, gw = cfg.width / cfg.patch_w;
  const int64_t n = gd * gh * gw, d = cfg.out_channels;
  std::vector<float> dense((size_t)(batch * n * d));
  CHECK_EQ(bjo_patch_embed3d_dense(&cfg, batch, video.data(), weight.data(), bias.data(), dense.data()), 0);
  std::vector<float> out;
  for (const auto& c : coords) {
    const int64_t tok = ((int64_t)c[1] * gh + c[2]) * gw + c[3];
    const float* row = dense.data() + ((int64_t)c[0] * n + tok) * d;
    out.insert(out.end(), row, row + d);
  }
  return out;
}

bjo_patchify_config oracle_cfg(const SparsePatchify3dConfig& c) {
  return bjo_patchify_config{(int64_t)c.in_channels, (int64_t)c.out_channels, (int64_t)c.frames, (int64_t)c.height,
                             (int64_t)c.width, (int64_t)c.tubelet_size, (int64_t)c.patch_h, (int64_t)c.patch_w};
}

// tests/sparse_patchify_cuda.rs:15
constexpr float kCudaParityTolerance = 2.0e-3f;

}  // namespace

// tests/sparse_patchify_cuda.rs:45-82 on the tiny config (src/config.rs:94-128): the sparse
// patchify rows equal the dense Conv3d patch embed at the selected tokens.
TEST(cuda_sparse_patchify_matches_dense_encoder_on_selected_tokens) {
  const SparsePatchify3dConfig cfg{3, 32, 4, 32, 32, 2, 16, 16};
  const TokenGridShape grid(2, 2, 2);
  const auto plan = SparsePatchifyPlan::new_(SparseTokenMask::new_({0, 3, 7}, grid.len()), grid, 1);
  std::vector<float> video(3 * 4 * 32 * 32);
  for (size_t i = 0; i < video.size(); ++i) video[i] = std::sin((float)i) * 0.01f;
  const auto weight = seeded(11, 32 * 3 * 2 * 16 * 16, 0.05f);
  const auto bias = seeded(12, 32, 0.02f);
  const Tensor v = Tensor::from_host(video, {1, 3, 4, 32, 32}, BJF_DTYPE_F32);
  const Tensor w = Tensor::from_host(weight, {32, 3, 2, 16, 16}, BJF_DTYPE_F32);
  const Tensor b = Tensor::from_host(bias, {32}, BJF_DTYPE_F32);
  const Tensor out = sparse_patchify3d_forward_cuda(cfg, v, plan.coords, w, &b);
  CHECK(out.shape() == (std::vector<int64_t>{3, 32}));
  const auto want = dense_at_coords(oracle_cfg(cfg), 1, video, weight, bias, plan.coords_host);
  CHECK(max_abs_diff(host_f32(out), want) <= kCudaParityTolerance);
}

// tests/sparse_patchify_cuda.rs:84-119: the image path reshapes [B, C, H, W] to
// [B, C, 1, H, W] with tubelet 1 (src/model.rs:1094-1206).
TEST(cuda_sparse_image_patchify_matches_dense_image_encoder_on_selected_tokens) {
  const SparsePatchify3dConfig cfg{3, 32, 1, 32, 32, 1, 16, 16};
  const TokenGridShape grid(1, 2, 2);
  const auto plan = SparsePatchifyPlan::new_(SparseTokenMask::new_({0, 3}, grid.len()), grid, 1);
  std::vector<float> image(3 * 32 * 32);
  for (size_t i = 0; i < image.size(); ++i) image[i] = std::sin((float)i) * 0.01f;
  const auto weight = seeded(21, 32 * 3 * 1 * 16 * 16, 0.05f);
  const std::vector<float> zeros(32, 0.0f);
  const Tensor v = Tensor::from_host(image, {1, 3, 1, 32, 32}, BJF_DTYPE_F32);
  const Tensor w = Tensor::from_host(weight, {32, 3, 1, 16, 16}, BJF_DTYPE_F32);
  const Tensor out = sparse_patchify3d_forward_cuda(cfg, v, plan.coords, w, nullptr);  // no bias: zeros
  const auto want = dense_at_coords(oracle_cfg(cfg), 1, image, weight, zeros, plan.coords_host);
  CHECK(max_abs_diff(host_f32(out), want) <= kCudaParityTolerance);
}

// src/model.rs:1273-1328 and 1094-1148: the encoder methods check the input against the plan
// and the config, then return the rows as [batch, plan tokens, D].
TEST(encoder_sparse_patchify_methods_check_the_plan_and_reshape) {
  const TokenGridShape grid(2, 2, 2);
  const auto plan = SparsePatchifyPlan::new_(SparseTokenMask::new_({0, 3, 7}, grid.len()), grid, 2);
  VJepaSparsePatchEmbed enc;
  enc.in_channels = 3;
  enc.embed_dim = 32;
  enc.tubelet_size = 2;
  enc.patch_size = 16;
  const auto video = seeded(51, 2 * 3 * 4 * 32 * 32, 1.0f);
  const auto weight = seeded(52, 32 * 3 * 2 * 16 * 16, 0.05f);
  const auto bias = seeded(53, 32, 0.02f);
  const Tensor v = Tensor::from_host(video, {2, 3, 4, 32, 32}, BJF_DTYPE_F32);
  const Tensor w = Tensor::from_host(weight, {32, 3, 2, 16, 16}, BJF_DTYPE_F32);
  const Tensor b = Tensor::from_host(bias, {32}, BJF_DTYPE_F32);
  const Tensor out = enc.sparse_patchify_video_cuda(v, plan, w, &b);
  CHECK(out.shape() == (std::vector<int64_t>{2, 3, 32}));
  const SparsePatchify3dConfig cfg{3, 32, 4, 32, 32, 2, 16, 16};
  CHECK(max_abs_diff(host_f32(out), dense_at_coords(oracle_cfg(cfg), 2, video, weight, bias, plan.coords_host)) <=
        kCudaParityTolerance);
  const auto one = SparsePatchifyPlan::new_(SparseTokenMask::new_({0, 3, 7}, grid.len()), grid, 1);
  CHECK_THROWS_WITH(enc.sparse_patchify_video_cuda(v, one, w, &b), "video batch does not match sparse patchify plan");
  VJepaSparsePatchEmbed four = enc;
  four.in_channels = 4;
  CHECK_THROWS_WITH(four.sparse_patchify_video_cuda(v, plan, w, &b), "video channel count does not match V-JEPA config");
  const auto other = SparsePatchifyPlan::new_(SparseTokenMask::new_({0, 3}, 4), TokenGridShape(1, 2, 2), 2);
  CHECK_THROWS_WITH(enc.sparse_patchify_video_cuda(v, other, w, &b), "video token grid does not match sparse patchify plan");

  // the image twin: [B, C, H, W] as one frame of tubelet 1
  const TokenGridShape igrid(1, 2, 2);
  const auto iplan = SparsePatchifyPlan::new_(SparseTokenMask::new_({1, 2}, igrid.len()), igrid, 2);
  const auto image = seeded(54, 2 * 3 * 32 * 32, 1.0f);
  const auto iweight = seeded(55, 32 * 3 * 1 * 16 * 16, 0.05f);
  const Tensor im = Tensor::from_host(image, {2, 3, 32, 32}, BJF_DTYPE_F32);
  const Tensor iw = Tensor::from_host(iweight, {32, 3, 1, 16, 16}, BJF_DTYPE_F32);
  const Tensor iout = enc.sparse_patchify_image_cuda(im, iplan, iw, nullptr);
  CHECK(iout.shape() == (std::vector<int64_t>{2, 2, 32}));
  const SparsePatchify3dConfig icfg{3, 32, 1, 32, 32, 1, 16, 16};
  const std::vector<float> zeros(32, 0.0f);
  CHECK(max_abs_diff(host_f32(iout), dense_at_coords(oracle_cfg(icfg), 2, image, iweight, zeros, iplan.coords_host)) <=
        kCudaParityTolerance);
  CHECK_THROWS_WITH(enc.sparse_patchify_image_cuda(im, plan, iw, nullptr), "image token grid does not match sparse patchify plan");
}

// src/temporal.rs:325-345, src/highres_pipeline.rs:2768-2793: plans are rebuilt only when the
// mask rows, the grid or the batch change
TEST(plan_caches_rebuild_only_on_change) {
  const TokenGridShape grid(2, 3, 4);
  SparsePatchifyPlanCache cache;
  CHECK(!cache.ensure(SparseTokenMask::new_({0, 7, 23}, grid.len()), grid, 2));
  CHECK(cache.ensure(SparseTokenMask::new_({23, 7, 0}, grid.len()), grid, 2));  // the same mask
  CHECK_EQ(cache.plan().coords_host.size(), (size_t)6);
  CHECK(!cache.ensure(SparseTokenMask::new_({0, 7}, grid.len()), grid, 2));
  CHECK(!cache.ensure(SparseTokenMask::new_({0, 7}, grid.len()), grid, 1));
  CHECK_EQ(cache.plan().coords.to_host<int32_t>(), (std::vector<int32_t>{0, 0, 0, 0, 0, 0, 1, 3}));
  SparsePatchifyBatchPlanCache bcache;
  const auto& p1 = bcache.get(SparseMaskBatch::from_rows({{0, 1}, {2, 3}}, grid.len()), grid);
  const void* first = &p1;
  const auto& p2 = bcache.get(SparseMaskBatch::from_rows({{1, 0}, {3, 2}}, grid.len()), grid);
  CHECK(&p2 == first);  // same rows after normalisation: reused
  CHECK_EQ(p2.coords_host.size(), (size_t)4);
  cache.reset();
  CHECK_THROWS_WITH(cache.plan(), "sparse patchify plan cache is empty");
}

// The tensor-core path (f16 and bf16 operands, f32 accumulation) on a fixed-width batch plan,
// against the oracle evaluated on the same rounded inputs; normwise relative error <= 1e-2.
static void half_patchify_case(bjf_dtype dt) {
  const SparsePatchify3dConfig cfg{3, 256, 4, 64, 64, 2, 16, 16};
  const TokenGridShape grid(2, 4, 4);
  std::vector<std::vector<size_t>> rows = {{0, 1, 5, 9, 12, 17, 20, 22, 25, 28, 30, 31},
                                           {2, 3, 4, 6, 7, 8, 10, 11, 13, 14, 15, 16}};
  const auto plan = SparsePatchifyBatchPlan::from_rows(rows, grid);
  const size_t nv = 2 * 3 * 4 * 64 * 64, nw = 256 * 3 * 2 * 16 * 16;
  auto video = seeded(31, nv, 1.0f);
  auto weight = seeded(32, nw, 0.05f);
  const auto bias = seeded(33, 256, 0.02f);
  auto enc = dt == BJF_DTYPE_F16 ? f32_to_f16_bits : f32_to_bf16_bits;
  auto dec = dt == BJF_DTYPE_F16 ? f16_bits_to_f32 : bf16_bits_to_f32;
  std::vector<uint16_t> vh(nv), wh(nw);
  for (size_t i = 0; i < nv; ++i) video[i] = dec(vh[i] = enc(video[i]));
  for (size_t i = 0; i < nw; ++i) weight[i] = dec(wh[i] = enc(weight[i]));
  const Tensor v = Tensor::from_host(vh, {2, 3, 4, 64, 64}, dt);
  const Tensor w = Tensor::from_host(wh, {256, 3, 2, 16, 16}, dt);
  const Tensor b = Tensor::from_host(bias, {256}, BJF_DTYPE_F32);
  const Tensor out = sparse_patchify3d_forward_cuda(cfg, v, plan.coords, w, &b, nullptr, BJF_DTYPE_F32);
  CHECK(out.shape() == (std::vector<int64_t>{24, 256}));
  const auto want = dense_at_coords(oracle_cfg(cfg), 2, video, weight, bias, plan.coords_host);
  CHECK(max_rel_err(host_f32(out), want) <= 1e-2f);
}
TEST(tensor_core_sparse_patchify_f16_matches_oracle) { half_patchify_case(BJF_DTYPE_F16); }
TEST(tensor_core_sparse_patchify_bf16_matches_oracle) { half_patchify_case(BJF_DTYPE_BF16); }

// tests/feature_memory.rs:9-65
TEST(sparse_updates_accumulate_dense_features_observed_mask_and_age) {
  const TokenGridShape grid(1, 2, 2);
  auto memory = InterframeJepaFeatureMemory::new_(1, grid, 2);
  auto step = [&](std::vector<float> tok, std::vector<int32_t> idx) {
    const int64_t s = (int64_t)idx.size();
    const Tensor t = Tensor::from_host(tok, {1, s, 2}, BJF_DTYPE_F32);
    const Tensor i = Tensor::from_host(idx, {1, s}, BJF_DTYPE_I32);
    return memory.update_tokens_tiled_assign_cuda(t, i, grid);
  };
  auto first = step({10, 11, 20, 21}, {0, 2});
  CHECK_EQ(first.step, (size_t)1);
  CHECK_EQ(first.updated_tokens, (size_t)2);
  CHECK_EQ(host_f32(*first.features), (std::vector<float>{10, 11, 0, 0, 20, 21, 0, 0}));
  CHECK_EQ(host_f32(*first.observed), (std::vector<float>{1, 0, 1, 0}));
  CHECK_EQ(host_f32(*first.age_frames), (std::vector<float>{0, 0, 0, 0}));
  auto second = step({30, 31}, {1});
  CHECK_EQ(second.step, (size_t)2);
  CHECK_EQ(host_f32(*second.features), (std::vector<float>{10, 11, 30, 31, 20, 21, 0, 0}));
  CHECK_EQ(host_f32(*second.observed), (std::vector<float>{1, 1, 1, 0}));
  CHECK_EQ(host_f32(*second.age_frames), (std::vector<float>{1, 0, 1, 0}));
  auto third = step({99, 98}, {0});
  CHECK_EQ(host_f32(*third.features), (std::vector<float>{99, 98, 30, 31, 20, 21, 0, 0}));
  CHECK_EQ(host_f32(*third.age_frames), (std::vector<float>{0, 1, 2, 0}));
}

// tests/feature_memory.rs:67-115
TEST(sparse_updates_write_by_token_index_not_sparse_position) {
  const TokenGridShape grid(1, 3, 3);
  auto memory = InterframeJepaFeatureMemory::new_(1, grid, 1);
  auto step = [&](std::vector<float> tok, std::vector<int32_t> idx) {
    const int64_t s = (int64_t)idx.size();
    return memory.update_tokens_tiled_assign_cuda(Tensor::from_host(tok, {1, s, 1}, BJF_DTYPE_F32),
                                                  Tensor::from_host(idx, {1, s}, BJF_DTYPE_I32), grid);
  };
  auto first = step({8, 0, 4}, {8, 0, 4});
  CHECK_EQ(host_f32(*first.features), (std::vector<float>{0, 0, 0, 0, 4, 0, 0, 0, 8}));
  CHECK_EQ(host_f32(*first.observed), (std::vector<float>{1, 0, 0, 0, 1, 0, 0, 0, 1}));
  auto second = step({2, 18}, {2, 8});
  CHECK_EQ(host_f32(*second.features), (std::vector<float>{0, 0, 2, 0, 4, 0, 0, 0, 18}));
  CHECK_EQ(host_f32(*second.observed), (std::vector<float>{1, 0, 1, 0, 1, 0, 0, 0, 1}));
  CHECK_EQ(host_f32(*second.age_frames), (std::vector<float>{1, 0, 0, 0, 1, 0, 0, 0, 0}));
}

// tests/feature_memory.rs:117-143
TEST(sparse_updates_eventually_fill_spatial_cache_over_time) {
  const TokenGridShape grid(1, 2, 2);
  auto memory = InterframeJepaFeatureMemory::new_(1, grid, 1);
  for (int32_t i = 0; i < 4; ++i)
    memory.update_tokens_tiled_assign_cuda(Tensor::from_host(std::vector<float>{(float)(i + 1)}, {1, 1, 1}, BJF_DTYPE_F32),
                                           Tensor::from_host(std::vector<int32_t>{i}, {1, 1}, BJF_DTYPE_I32), grid);
  const auto snap = memory.snapshot();
  CHECK_EQ(host_f32(*snap.observed), (std::vector<float>{1, 1, 1, 1}));
  CHECK_EQ(host_f32(*snap.features), (std::vector<float>{1, 2, 3, 4}));
}

// tests/feature_memory.rs:209-260 (token_values :466-472) on a half-precision cache
TEST(high_density_sparse_update_preserves_unwritten_512_grid_tokens) {
  const TokenGridShape grid(1, 32, 32);
  const size_t n = grid.len(), d = 4, keep = (n * 98 + 99) / 100;
  auto memory = InterframeJepaFeatureMemory::new_(1, grid, d);
  auto values = [&](size_t count, float offset) {
    std::vector<float> v;
    for (size_t t = 0; t < count; ++t)
      for (size_t c = 0; c < d; ++c) v.push_back(offset + 10.0f * (float)t + (float)c);
    return v;
  };
  std::vector<int32_t> all(n), first(keep);
  for (size_t i = 0; i < n; ++i) all[i] = (int32_t)i;
  for (size_t i = 0; i < keep; ++i) first[i] = (int32_t)i;
  memory.update_tokens_tiled_assign_cuda(Tensor::from_host(values(n, 1000.0f), {1, (int64_t)n, (int64_t)d}, BJF_DTYPE_F32),
                                         Tensor::from_host(all, {1, (int64_t)n}, BJF_DTYPE_I32), grid);
  const auto out = memory.update_tokens_tiled_assign_cuda(
      Tensor::from_host(values(keep, 2000.0f), {1, (int64_t)keep, (int64_t)d}, BJF_DTYPE_F32),
      Tensor::from_host(first, {1, (int64_t)keep}, BJF_DTYPE_I32), grid);
  const auto f = host_f32(*out.features), age = host_f32(*out.age_frames), obs = host_f32(*out.observed);
  const auto prime = values(n, 1000.0f), upd = values(keep, 2000.0f);
  for (size_t t = 0; t < n; ++t)
    for (size_t c = 0; c < d; ++c) CHECK_EQ(f[t * d + c], t < keep ? upd[t * d + c] : prime[t * d + c]);
  CHECK(std::all_of(obs.begin(), obs.end(), [](float o) { return o == 1.0f; }));
  CHECK_EQ(age[0], 0.0f);
  CHECK_EQ(age[keep - 1], 0.0f);
  CHECK_EQ(age[keep], 1.0f);
}

// tests/feature_memory.rs:262-298
TEST(masked_and_index_updates_write_the_same_canvas) {
  const TokenGridShape grid(1, 2, 2);
  auto memory = InterframeJepaFeatureMemory::new_(1, grid, 2);
  memory.update_masked_tokens_tiled_assign_cuda(Tensor::from_host(std::vector<float>{1, 2, 7, 8}, {1, 2, 2}, BJF_DTYPE_F32),
                                                SparseTokenMask::new_({0, 3}, 4), grid);
  const auto out = memory.update_tokens_tiled_assign_cuda(
      Tensor::from_host(std::vector<float>{5, 6}, {1, 1, 2}, BJF_DTYPE_F32),
      Tensor::from_host(std::vector<int32_t>{2}, {1, 1}, BJF_DTYPE_I32), grid);
  CHECK_EQ(host_f32(*out.features), (std::vector<float>{1, 2, 0, 0, 5, 6, 7, 8}));
}

// tests/feature_memory.rs:300-340
TEST(reset_rows_and_reset_clear_memory) {
  const TokenGridShape grid(1, 1, 3);
  auto memory = InterframeJepaFeatureMemory::new_(2, grid, 1);
  memory.update_tokens_tiled_assign_cuda(Tensor::from_host(std::vector<float>{1, 2, 3, 4}, {2, 2, 1}, BJF_DTYPE_F32),
                                         Tensor::from_host(std::vector<int32_t>{0, 1, 1, 2}, {2, 2}, BJF_DTYPE_I32),
                                         grid);
  memory.reset_row_indices({1});
  auto snap = memory.snapshot();
  CHECK_EQ(host_f32(*snap.features), (std::vector<float>{1, 2, 0, 0, 0, 0}));
  CHECK_EQ(host_f32(*snap.observed), (std::vector<float>{1, 1, 0, 0, 0, 0}));
  memory.reset_row_indices({0});
  snap = memory.snapshot();
  CHECK_EQ(host_f32(*snap.features), std::vector<float>(6, 0.0f));
  CHECK_EQ(host_f32(*snap.observed), std::vector<float>(6, 0.0f));
  CHECK_THROWS_WITH(memory.reset_row_indices({2}), "feature memory row reset index outside batch");
  memory.reset();
  CHECK_EQ(memory.step(), (size_t)0);
  CHECK_EQ(host_f32(*memory.snapshot().age_frames), std::vector<float>(6, 0.0f));
}

// tests/feature_memory.rs:145-177 (EMA on the device; the reference runs it on its portable path)
TEST(ema_updates_assign_first_observation_then_blend_repeated_tokens) {
  const TokenGridShape grid(1, 1, 2);
  auto memory = InterframeJepaFeatureMemory::with_config(InterframeJepaFeatureMemoryConfig::ema(0.25f), 1, grid, 1);
  memory.update_tokens(Tensor::from_host(std::vector<float>{8}, {1, 1, 1}, BJF_DTYPE_F32),
                       Tensor::from_host(std::vector<int32_t>{0}, {1, 1}, BJF_DTYPE_I32), grid);
  const auto out = memory.update_tokens(Tensor::from_host(std::vector<float>{12}, {1, 1, 1}, BJF_DTYPE_F32),
                                        Tensor::from_host(std::vector<int32_t>{0}, {1, 1}, BJF_DTYPE_I32), grid);
  CHECK_EQ(host_f32(*out.features), (std::vector<float>{9, 0}));
  CHECK(InterframeJepaFeatureMemoryConfig::ema(3.0f).normalized().alpha == 1.0f);
}

// tests/feature_memory.rs:300-339 with the device-tensor form of reset_rows
TEST(reset_rows_device_tensor_clears_rows) {
  const TokenGridShape grid(1, 1, 3);
  auto memory = InterframeJepaFeatureMemory::new_(2, grid, 1);
  memory.update_tokens(Tensor::from_host(std::vector<float>{1, 2, 3, 4}, {2, 2, 1}, BJF_DTYPE_F32),
                       Tensor::from_host(std::vector<int32_t>{0, 1, 1, 2}, {2, 2}, BJF_DTYPE_I32), grid);
  memory.reset_rows(Tensor::from_host(std::vector<int32_t>{1}, {1}, BJF_DTYPE_I32));
  auto snap = memory.snapshot();
  CHECK_EQ(host_f32(*snap.features), (std::vector<float>{1, 2, 0, 0, 0, 0}));
  CHECK_EQ(host_f32(*snap.observed), (std::vector<float>{1, 1, 0, 0, 0, 0}));
}

// tests/feature_memory.rs:341-377
TEST(update_rejects_incompatible_shapes) {
  const TokenGridShape grid(1, 2, 2);
  auto memory = InterframeJepaFeatureMemory::new_(1, grid, 2);
  const Tensor t = Tensor::from_host(std::vector<float>{1, 2}, {1, 1, 2}, BJF_DTYPE_F32);
  CHECK_THROWS_WITH(memory.update_tokens_tiled_assign_cuda(
                        t, Tensor::from_host(std::vector<int32_t>{0}, {1, 1}, BJF_DTYPE_I32), TokenGridShape(1, 1, 4)),
                    "grid");
  CHECK_THROWS_WITH(
      memory.update_tokens_tiled_assign_cuda(t, Tensor::from_host(std::vector<int32_t>{0, 1}, {1, 2}, BJF_DTYPE_I32), grid),
      "index shape");
}

// tests/sparse_pipeline.rs:89-136: a 16x16 change in frame 1 selects token (0, 1, 1).
TEST(patch_diff_selects_the_changed_patch) {
  std::vector<float> video(3 * 4 * 32 * 32, 0.0f);
  for (int c = 0; c < 3; ++c)
    for (int y = 16; y < 32; ++y)
      for (int x = 16; x < 32; ++x) video[((c * 4 + 1) * 32 + y) * 32 + x] = 1.0f;
  const Tensor v = Tensor::from_host(video, {1, 3, 4, 32, 32}, BJF_DTYPE_F32);
  const TokenGridShape grid(2, 2, 2);
  for (float threshold : {0.1f, 0.0f}) {
    const auto cfg = SparseJepaPatchDiffSparsityConfig::new_(threshold, 1, 2);
    const auto context = patch_diff_context_mask_from_video(v, 2, 16, grid, cfg);
    CHECK_EQ(context.indices(), (std::vector<size_t>{coords_to_token_index(0, 1, 1, grid)}));
    CHECK_EQ(target_mask_from_context(context, 2).len(), (size_t)2);
  }
  const auto scores = patch_diff_token_scores(v, 2, 16, grid).to_host<float>();
  CHECK(scores[3] > 0.0f);
  CHECK_EQ(scores[0] + scores[1] + scores[2] + scores[4] + scores[5] + scores[6] + scores[7], 0.0f);
}

// tests/highres_anyup_pca_pipeline.rs:583-653 (helper :1468-1494)
TEST(adaptive_patch_diff_threshold_cases) {
  auto two_frame = [](std::vector<std::pair<int, int>> patches) {
    std::vector<float> v(3 * 2 * 32 * 32, 0.0f);
    for (auto [r, c] : patches)
      for (int ch = 0; ch < 3; ++ch)
        for (int y = r * 16; y < (r + 1) * 16; ++y)
          for (int x = c * 16; x < (c + 1) * 16; ++x) v[((ch * 2 + 1) * 32 + y) * 32 + x] = 1.0f;
    return Tensor::from_host(v, {1, 3, 2, 32, 32}, BJF_DTYPE_F32);
  };
  const TokenGridShape g22(1, 2, 2);
  const auto adaptive = SparseJepaPatchDiffSparsityConfig::adaptive_threshold(0.5f, 1, 4, 1);
  CHECK_EQ(patch_diff_context_mask_from_video(two_frame({{0, 1}, {1, 0}}), 2, 16, g22, adaptive).indices(),
           (std::vector<size_t>{1, 2}));
  CHECK_EQ(patch_diff_context_mask_from_video(two_frame({}), 2, 16, g22, adaptive).len(), (size_t)1);
  CHECK_EQ(patch_diff_context_mask_from_scores({0.9f, 0.0f, 0.8f, 0.7f, 0.0f, 0.6f}, TokenGridShape(1, 2, 3),
                                               SparseJepaPatchDiffSparsityConfig::adaptive_threshold(0.5f, 1, 1, 1))
               .indices(),
           (std::vector<size_t>{0, 2, 3, 5}));
  CHECK_EQ(patch_diff_context_mask_from_scores({0.0f, 0.1f, 0.2f, 0.3f}, g22,
                                               SparseJepaPatchDiffSparsityConfig::adaptive_threshold(0.0f, 1, 1, 1))
               .indices(),
           (std::vector<size_t>{0, 1, 2, 3}));
}

// src/viewer.rs:1391-1403 on the device scorer
TEST(rgba_patch_diff_ignores_uniform_lighting_shift) {
  const std::vector<int32_t> prev_words(64 * 64, 0x50505050), cur_words(64 * 64, 0x6e6e6e6e);  // 80 / 110 per byte
  const Tensor prev = Tensor::from_host(prev_words, {64 * 64}, BJF_DTYPE_I32);
  const Tensor cur = Tensor::from_host(cur_words, {64 * 64}, BJF_DTYPE_I32);
  std::vector<RgbaPatchDiffFrameStats> stats;
  const auto scores = patch_diff_scores_from_rgba(static_cast<const uint8_t*>(prev.data()),
                                                  static_cast<const uint8_t*>(cur.data()), 64, 64, 16,
                                                  TokenGridShape(1, 4, 4), 1, &stats)
                          .to_host<float>();
  for (float v : scores) CHECK(v < DEFAULT_PATCH_DIFF_THRESHOLD);
  CHECK_EQ(stats.size(), (size_t)1);
  CHECK_EQ(stats[0].compensate_global_lighting, 1);
}

// patch_diff_masks_from_scores on the device against the host policy composition
// (src/viewer.rs:819-841, 946-961), for several streams and viewer configs.
TEST(viewer_masks_from_scores_match_host_policy) {
  const TokenGridShape grid(1, 32, 32);
  const size_t S = 5, N = grid.len();
  auto u = seeded(77, S * N, 1.0f);
  std::vector<float> scores(S * N);
  for (size_t s = 0; s < S; ++s)
    for (size_t i = 0; i < N; ++i) scores[s * N + i] = std::pow(std::fabs(u[s * N + i]), 1.0f + 3.0f * (float)s);
  const Tensor dscores = Tensor::from_host(scores, {(int64_t)S, (int64_t)N}, BJF_DTYPE_F32);
  FeatureFrameViewerConfig exact;
  exact.sparse_encode_mode = FeatureFrameSparseEncodeMode::Exact;
  FeatureFrameViewerConfig legacy;
  legacy.sparse_mask_bucket_densities.clear();
  legacy.sparse_mask_bucket_tokens = 100;
  for (const auto& cfg : {FeatureFrameViewerConfig{}, exact, legacy})
    for (size_t dilation : {0, 1, 2}) {
      const auto sparsity = SparseJepaPatchDiffSparsityConfig::adaptive_threshold(0.2f, 4, N, 1).with_dilation(dilation);
      const auto dev = patch_diff_masks_from_scores(dscores, grid, sparsity, cfg);
      for (size_t s = 0; s < S; ++s) {
        const std::vector<float> row(scores.begin() + s * N, scores.begin() + (s + 1) * N);
        const auto direct = patch_diff_context_mask_from_scores(row, grid, sparsity.with_dilation(0));
        const auto write = dilate_sparse_patch_mask(
            patch_diff_dense_fallback(direct, grid, cfg.patch_diff_dense_fallback_density), grid, dilation);
        const auto host = finalize_patch_diff_encode_masks(write, grid, cfg);
        const auto got = dev.stream(s);
        CHECK_EQ(got.write_mask.indices(), host.write_mask.indices());
        CHECK_EQ(got.encode_mask.indices(), host.encode_mask.indices());
      }
    }
}

// src/viewer.rs:1486-1527 through the device RGBA mask node: 16 of 64 patches change, below
// the 0.60 sampled fallback, so the masks come from the scores (direct hits dilated by one
// tile); with 48 of 64 changed the sampled fast path gives every token.
TEST(rgba_mask_node_sampled_dense_fast_path) {
  const TokenGridShape grid(1, 8, 8);
  const size_t P = 16, W = 128, H = 128;
  const auto frames = [&](size_t rows, size_t cols) {
    std::vector<int32_t> prev(W * H, (int32_t)0xff000000), cur(W * H, (int32_t)0xff000000);
    for (size_t y = 0; y < rows * P; ++y)
      for (size_t x = 0; x < cols * P; ++x) cur[y * W + x] = (int32_t)0xffffffff;
    return std::make_pair(Tensor::from_host(prev, {(int64_t)(W * H)}, BJF_DTYPE_I32),
                          Tensor::from_host(cur, {(int64_t)(W * H)}, BJF_DTYPE_I32));
  };
  const auto cfg = SparseJepaPatchDiffSparsityConfig::adaptive_threshold(0.10f, 1, grid.len(), grid.len()).with_dilation(1);
  FeatureFrameViewerConfig viewer;
  viewer.patch_diff_dense_fallback_density = 0.60f;
  {
    const auto [prev, cur] = frames(4, 4);
    const auto m = patch_diff_masks_from_rgba(static_cast<const uint8_t*>(prev.data()),
                                              static_cast<const uint8_t*>(cur.data()), W, H, P, grid, cfg, viewer)
                       .stream(0);
    CHECK_EQ(m.write_mask.len(), (size_t)25);  // the 4x4 block dilated by one tile
    CHECK(!m.write_mask.is_dense_ordered());
  }
  {
    const auto [prev, cur] = frames(6, 8);
    const auto m = patch_diff_masks_from_rgba(static_cast<const uint8_t*>(prev.data()),
                                              static_cast<const uint8_t*>(cur.data()), W, H, P, grid, cfg, viewer)
                       .stream(0);
    CHECK(m.write_mask.is_dense_ordered());
    CHECK(m.encode_mask.is_dense_ordered());
  }
}

// src/viewer.rs:1528-1575: repeated below-threshold motion is refreshed on the third frame
TEST(subthreshold_patch_diff_accumulates_slow_motion) {
  const TokenGridShape grid(1, 4, 4);
  const size_t slow_index = coords_to_token_index(0, 2, 1, grid);
  FeatureFrameViewerConfig config;
  config.context_density = 0.25f;
  config.min_context_density = 0.0f;
  config.patch_diff_threshold = 0.10f;
  config.patch_diff_dense_fallback_density = 1.0f;
  config.patch_diff_dilation_tiles = 0;
  config.sparse_encode_mode = FeatureFrameSparseEncodeMode::Exact;
  config.patch_diff_refresh.enabled = true;
  config.patch_diff_refresh.subthreshold_enabled = true;
  config.patch_diff_refresh.subthreshold_decay = 1.0f;
  config.patch_diff_refresh.subthreshold_trigger = 1.0f;
  config.patch_diff_refresh.subthreshold_max_density = 0.25f;
  config.patch_diff_refresh.age_refresh_enabled = false;
  config.patch_diff_refresh.blue_noise_enabled = false;
  config.patch_diff_refresh.max_extra_density = 0.25f;
  const auto sparsity = patch_diff_sparsity_config(config, grid);
  PatchDiffRefreshState state;
  std::vector<float> scores(grid.len(), 0.0f);
  scores[0] = 0.09f;
  scores[slow_index] = 0.04f;
  const auto contains = [](const SparseTokenMask& m, size_t i) {
    return std::find(m.indices().begin(), m.indices().end(), i) != m.indices().end();
  };
  CHECK(!contains(state.masks_from_scores(scores, grid, sparsity, config).write_mask, slow_index));
  CHECK(!contains(state.masks_from_scores(scores, grid, sparsity, config).write_mask, slow_index));
  CHECK(contains(state.masks_from_scores(scores, grid, sparsity, config).write_mask, slow_index));
  CHECK(state.subthreshold_residual(slow_index) == std::optional<float>(0.0f));
  CHECK(state.age_frames(slow_index) == std::optional<uint32_t>(0u));
}

// src/viewer.rs:1595-1632: refresh never exceeds the context budget
TEST(subthreshold_refresh_fills_only_unused_context_budget) {
  const TokenGridShape grid(1, 4, 4);
  FeatureFrameViewerConfig config;
  config.context_density = 2.0f / 16.0f;
  config.min_context_density = 0.0f;
  config.patch_diff_threshold = 0.10f;
  config.patch_diff_dense_fallback_density = 1.0f;
  config.patch_diff_dilation_tiles = 0;
  config.sparse_encode_mode = FeatureFrameSparseEncodeMode::Exact;
  config.patch_diff_refresh.enabled = true;
  config.patch_diff_refresh.subthreshold_enabled = true;
  config.patch_diff_refresh.subthreshold_decay = 1.0f;
  config.patch_diff_refresh.subthreshold_trigger = 0.5f;
  config.patch_diff_refresh.subthreshold_max_density = 1.0f;
  config.patch_diff_refresh.age_refresh_enabled = false;
  config.patch_diff_refresh.blue_noise_enabled = false;
  config.patch_diff_refresh.max_extra_density = 1.0f;
  const auto sparsity = patch_diff_sparsity_config(config, grid);
  PatchDiffRefreshState state;
  std::vector<float> scores(grid.len(), 0.06f);
  scores[0] = 0.09f;
  CHECK_EQ(state.masks_from_scores(scores, grid, sparsity, config).write_mask.len(), (size_t)2);
}

// src/viewer.rs:1634-1672: stale tokens are refreshed once their age reaches the interval
TEST(age_priority_refresh_selects_stale_tokens) {
  const TokenGridShape grid(1, 4, 4);
  FeatureFrameViewerConfig config;
  config.context_density = 0.50f;
  config.min_context_density = 0.0f;
  config.patch_diff_threshold = 0.10f;
  config.patch_diff_dense_fallback_density = 1.0f;
  config.patch_diff_dilation_tiles = 0;
  config.sparse_encode_mode = FeatureFrameSparseEncodeMode::Exact;
  config.patch_diff_refresh.subthreshold_enabled = false;
  config.patch_diff_refresh.enabled = true;
  config.patch_diff_refresh.age_refresh_enabled = true;
  config.patch_diff_refresh.age_refresh_interval_frames = 2;
  config.patch_diff_refresh.age_refresh_max_density = 0.25f;
  config.patch_diff_refresh.blue_noise_enabled = false;
  config.patch_diff_refresh.max_extra_density = 0.25f;
  const auto sparsity = patch_diff_sparsity_config(config, grid);
  PatchDiffRefreshState state;
  std::vector<float> scores(grid.len(), 0.0f);
  scores[0] = 0.09f;
  const size_t first = state.masks_from_scores(scores, grid, sparsity, config).write_mask.len();
  CHECK_EQ(first, (size_t)1);
  CHECK(state.masks_from_scores(scores, grid, sparsity, config).write_mask.len() > first);
}

// src/viewer.rs:1674-1703: blue-noise refresh depends only on the state and the seed
TEST(blue_noise_refresh_is_deterministic_for_same_state) {
  const TokenGridShape grid(1, 4, 4);
  FeatureFrameViewerConfig config;
  config.context_density = 0.50f;
  config.min_context_density = 0.0f;
  config.patch_diff_threshold = 0.10f;
  config.patch_diff_dense_fallback_density = 1.0f;
  config.patch_diff_dilation_tiles = 0;
  config.sparse_encode_mode = FeatureFrameSparseEncodeMode::Exact;
  config.patch_diff_refresh.subthreshold_enabled = false;
  config.patch_diff_refresh.age_refresh_enabled = false;
  config.patch_diff_refresh.enabled = true;
  config.patch_diff_refresh.blue_noise_enabled = true;
  config.patch_diff_refresh.blue_noise_refresh_density = 0.25f;
  config.patch_diff_refresh.max_extra_density = 0.25f;
  config.patch_diff_refresh.blue_noise_seed = 7;
  const auto sparsity = patch_diff_sparsity_config(config, grid);
  PatchDiffRefreshState left, right;
  const std::vector<float> scores(grid.len(), 0.0f);
  const auto l = left.masks_from_scores(scores, grid, sparsity, config).write_mask;
  const auto r = right.masks_from_scores(scores, grid, sparsity, config).write_mask;
  CHECK_EQ(l.indices(), r.indices());
  CHECK(l.len() > (size_t)0);
}

// src/viewer.rs:1405-1453 through the viewer config: the sparsity config dilates direct hits
TEST(patch_diff_sparsity_config_dilates_direct_hits) {
  const TokenGridShape grid(1, 4, 4);
  const size_t center = coords_to_token_index(0, 2, 1, grid);
  std::vector<float> scores(grid.len(), 0.0f);
  scores[center] = 0.5f;
  FeatureFrameViewerConfig config;
  config.context_density = 1.0f;
  config.min_context_density = 0.0f;
  config.patch_diff_threshold = 0.10f;
  config.patch_diff_dilation_tiles = 1;
  config.patch_diff_refresh = PatchDiffRefreshConfig::disabled();
  config.sparse_encode_mode = FeatureFrameSparseEncodeMode::Exact;
  const auto dilated = patch_diff_context_mask_from_scores(scores, grid, patch_diff_sparsity_config(config, grid));
  std::vector<size_t> want;
  for (size_t r = 1; r <= 3; ++r)
    for (size_t c = 0; c <= 2; ++c) want.push_back(coords_to_token_index(0, r, c, grid));
  CHECK_EQ(dilated.indices(), want);
  config.patch_diff_dilation_tiles = 0;
  CHECK_EQ(patch_diff_context_mask_from_scores(scores, grid, patch_diff_sparsity_config(config, grid)).indices(),
           (std::vector<size_t>{center}));
}

// The fused step over S streams against the oracle's per-stream composition.  Unchanged
// tubelets score exactly 0, so a small positive threshold selects exactly the changed ones
// whatever the summation order.
TEST(front_end_step_matches_oracle_streams) {
  const size_t S = 3, C = 3, T = 2, H = 64, W = 64, KT = 2, P = 16, D = 128;
  const TokenGridShape grid(1, 4, 4);
  const size_t N = grid.len(), K = C * KT * P * P;
  std::vector<float> video(S * C * T * H * W);
  const auto base = seeded(41, C * H * W, 1.0f);
  const auto noise = seeded(42, S * C * H * W, 0.3f);
  for (size_t s = 0; s < S; ++s)
    for (size_t c = 0; c < C; ++c)
      for (size_t y = 0; y < H; ++y)
        for (size_t x = 0; x < W; ++x) {
          const size_t tok = (y / P) * 4 + x / P;
          const bool changed = (tok * 7 + s * 3) % 5 == 0;
          const float b = base[(c * H + y) * W + x];
          video[(((s * C + c) * T + 0) * H + y) * W + x] = b;
          video[(((s * C + c) * T + 1) * H + y) * W + x] = b + (changed ? noise[((s * C + c) * H + y) * W + x] : 0.0f);
        }
  std::vector<uint16_t> vh(video.size());
  for (size_t i = 0; i < video.size(); ++i) video[i] = f16_bits_to_f32(vh[i] = f32_to_f16_bits(video[i]));
  auto weight = seeded(43, D * K, 0.05f);
  std::vector<uint16_t> wh(weight.size());
  for (size_t i = 0; i < weight.size(); ++i) weight[i] = f16_bits_to_f32(wh[i] = f32_to_f16_bits(weight[i]));
  const auto bias = seeded(44, D, 0.02f);
  const auto mcfg = SparseJepaPatchDiffSparsityConfig::adaptive_threshold(1e-4f, 1, N, 1);

  FrontEnd fe(S, C, T, H, W, KT, P, D, mcfg, BJF_DTYPE_F16, BJF_DTYPE_F32);
  const Tensor v = Tensor::from_host(vh, {(int64_t)S, (int64_t)C, (int64_t)T, (int64_t)H, (int64_t)W}, BJF_DTYPE_F16);
  const Tensor w = Tensor::from_host(wh, {(int64_t)D, (int64_t)C, (int64_t)KT, (int64_t)P, (int64_t)P}, BJF_DTYPE_F16);
  const Tensor b = Tensor::from_host(bias, {(int64_t)D}, BJF_DTYPE_F32);
  for (int step = 0; step < 2; ++step) fe.step(v, w, &b);
  const auto counts = fe.step(v, w, &b).to_host<int32_t>();

  const bjo_patchify_config pc{(int64_t)C, (int64_t)D, (int64_t)T, (int64_t)H, (int64_t)W, (int64_t)KT, (int64_t)P, (int64_t)P};
  const bjf_patch_diff_config mc = mcfg.to_c();
  bjo_patch_diff_config omc;
  std::memcpy(&omc, &mc, sizeof(omc));
  std::vector<float> caches(S * N * D, 0.0f), observed(S * N, 0.0f), age(S * N, 0.0f);
  std::vector<int64_t> want_counts(S);
  for (int step = 0; step < 3; ++step)
    CHECK_EQ(bjo_front_end_streams(video.data(), (int64_t)S, &pc, &omc, weight.data(), bias.data(), caches.data(),
                                   observed.data(), age.data(), step > 0 ? 1 : 0, want_counts.data()),
             0);
  for (size_t s = 0; s < S; ++s) CHECK_EQ((int64_t)counts[s], want_counts[s]);
  CHECK_EQ(host_f32(fe.observed()), observed);
  CHECK_EQ(host_f32(fe.age_frames()), age);
  CHECK(max_rel_err(host_f32(fe.caches()), caches) <= 1e-2f);
  CHECK(!device_error_check());
}

TEST_MAIN()
