// test_host_api.cpp -- host-side ports of the reference's own tests onto the C++ API of
// include/bjf.hpp.  Needs no GPU: every case here is decided before any device work.
#include <set>

#include "../../include/bjf.hpp"
#include "check.hpp"

using namespace bjf;

// src/positional.rs:97-103
TEST(token_index_round_trip_uses_depth_height_width_order) {
  const TokenGridShape grid(3, 4, 5);
  const size_t index = coords_to_token_index(2, 3, 4, grid);
  CHECK_EQ(index, (size_t)59);
  CHECK(token_index_to_coords(index, grid) == std::make_tuple((size_t)2, (size_t)3, (size_t)4));
}

// src/tokens.rs:563-568
TEST(complement_preserves_sorted_indices) {
  const auto mask = SparseTokenMask::new_({3, 1, 1}, 5);
  CHECK_EQ(mask.indices(), (std::vector<size_t>{1, 3}));
  CHECK_EQ(mask.complement().indices(), (std::vector<size_t>{0, 2, 4}));
}

// src/tokens.rs:570-580
TEST(padded_mask_keeps_existing_tokens_and_rounds_to_bucket) {
  const auto mask = SparseTokenMask::new_({7, 1, 3}, 10);
  const auto padded = mask.padded_to_multiple(4);
  CHECK_EQ(padded.len(), (size_t)4);
  for (size_t index : {1, 3, 7})
    CHECK(std::find(padded.indices().begin(), padded.indices().end(), index) != padded.indices().end());
  CHECK(!padded.is_dense_ordered());
}

// src/tokens.rs:582-589
TEST(padded_mask_promotes_to_dense_when_bucket_reaches_dense_len) {
  const auto mask = SparseTokenMask::new_({0, 2, 4, 6, 8}, 10);
  const auto padded = mask.padded_to_multiple(16);
  CHECK_EQ(padded.indices(), SparseTokenMask::all(10).indices());
  CHECK(padded.is_dense_ordered());
}

// src/tokens.rs:591-603
TEST(target_mask_from_context_is_disjoint_and_fills_budget) {
  const auto context = SparseTokenMask::new_({0, 2, 4}, 6);
  const auto target = target_mask_from_context(context, 2);
  CHECK_EQ(target.len(), (size_t)2);
  for (size_t i : target.indices())
    CHECK(std::find(context.indices().begin(), context.indices().end(), i) == context.indices().end());
}

// src/config.rs:373-378 (tiny grid has 8 tokens) and src/tokens.rs:488-495
TEST(tiny_grid_context_target_masks) {
  const TokenGridShape grid(4 / 2, 32 / 16, 32 / 16);
  CHECK_EQ(grid.len(), (size_t)8);
  const auto [context, target] = make_context_target_masks(grid, 0.5f);
  CHECK_EQ(context.indices(), (std::vector<size_t>{0, 1, 2, 3}));
  CHECK_EQ(target.indices(), (std::vector<size_t>{4, 5, 6, 7}));
}

// src/tokens.rs:41-50
TEST(sparse_token_mask_rejects_bad_input) {
  CHECK_THROWS_WITH(SparseTokenMask::new_({0}, 0), "dense token count must be nonzero");
  CHECK_THROWS_WITH(SparseTokenMask::new_({0, 5}, 5), "sparse token index outside dense token range");
}

TEST(evenly_spaced_and_keep_ratio) {
  CHECK_EQ(SparseTokenMask::evenly_spaced_indices(10, 3), (std::vector<size_t>{0, 3, 6}));
  CHECK_EQ(SparseTokenMask::evenly_spaced_indices(4, 9), (std::vector<size_t>{0, 1, 2, 3}));
  CHECK_EQ(SparseTokenMask::from_keep_ratio(10, 0.25f).len(), (size_t)3);
  CHECK_EQ(SparseTokenMask::from_keep_ratio(10, -1.0f).len(), (size_t)1);
}

// src/sparse_patchify.rs:676-693
TEST(sparse_patchify_plan_coords_are_batch_major) {
  const TokenGridShape grid(2, 3, 4);
  const auto mask = SparseTokenMask::new_({0, 7, 23}, grid.len());
  const auto coords = SparsePatchifyPlan::host_coords(mask, grid, 2);
  const std::vector<std::array<uint32_t, 4>> want = {
      {0, 0, 0, 0}, {0, 0, 1, 3}, {0, 1, 2, 3}, {1, 0, 0, 0}, {1, 0, 1, 3}, {1, 1, 2, 3}};
  CHECK(coords == want);
}

// src/sparse_patchify.rs:243-247, 291-299
TEST(sparse_patchify_plans_reject_bad_input) {
  const TokenGridShape grid(1, 2, 2);
  CHECK_THROWS_WITH(SparsePatchifyPlan::host_coords(SparseTokenMask::new_({0}, 4), grid, 0),
                    "sparse patchify batch must be nonzero");
  CHECK_THROWS_WITH(SparsePatchifyPlan::host_coords(SparseTokenMask::new_({0}, 5), grid, 1),
                    "sparse patchify mask dense token count must match grid");
  CHECK_THROWS_WITH(SparsePatchifyBatchPlan::from_rows({{0, 1}, {2}}, grid),
                    "sparse patchify batch plans require uniform or fixed-width masks");
}

// src/nodes.rs:97-157
TEST(patch_diff_config_builders) {
  const auto a = SparseJepaPatchDiffSparsityConfig::adaptive_threshold(0.5f, 2, 64, 3);
  CHECK_EQ(a.context_tokens, (size_t)64);
  CHECK_EQ(a.min_context_tokens, (size_t)2);
  CHECK(!a.fill_to_context_tokens);
  CHECK(a.allow_full_context);
  const auto n = SparseJepaPatchDiffSparsityConfig::new_(0.1f, 4, 2).with_dilation(1);
  CHECK_EQ(n.min_context_tokens, (size_t)1);
  CHECK(n.fill_to_context_tokens);
  CHECK(!n.allow_full_context);
  CHECK_EQ(n.to_c().dilation, (int64_t)1);
}

// src/nodes.rs:463-466
TEST(mask_from_scores_rejects_wrong_length) {
  const auto cfg = SparseJepaPatchDiffSparsityConfig::new_(0.1f, 1, 1);
  CHECK_THROWS_WITH(patch_diff_context_mask_from_scores({0.1f, 0.2f}, TokenGridShape(1, 1, 3), cfg),
                    "patch-diff sparsity received unexpected score length");
}

// src/feature_memory.rs:152-162
TEST(feature_memory_rejects_empty_shapes) {
  CHECK_THROWS_WITH(InterframeJepaFeatureMemory::new_(0, TokenGridShape(1, 2, 2), 4),
                    "feature memory batch must be nonzero");
  CHECK_THROWS_WITH(InterframeJepaFeatureMemory::new_(1, TokenGridShape(0, 2, 2), 4),
                    "feature memory grid must be nonempty");
  CHECK_THROWS_WITH(InterframeJepaFeatureMemory::new_(1, TokenGridShape(1, 2, 2), 0),
                    "feature memory embed dim must be nonzero");
}

// src/nodes.rs:427-432, through the C ABI's host-side validation
TEST(front_end_rejects_indivisible_geometry) {
  const auto cfg = SparseJepaPatchDiffSparsityConfig::adaptive_threshold(0.1f, 1, 4, 1);
  CHECK_THROWS_WITH(FrontEnd(1, 3, 3, 32, 32, 2, 16, 64, cfg, BJF_DTYPE_F16, BJF_DTYPE_F16),
                    "patch-diff sparsity requires frames/height/width divisible by tubelet and patch sizes");
}

// src/viewer.rs:1455-1481: direct mask -> dense fallback -> dilation
TEST(dense_cutoff_runs_before_dilation) {
  const TokenGridShape grid(1, 5, 5);
  const size_t center = coords_to_token_index(0, 2, 2, grid);
  const auto direct = SparseTokenMask::new_({center}, grid.len());
  const auto write = dilate_sparse_patch_mask(patch_diff_dense_fallback(direct, grid, 0.25f), grid, 1);
  CHECK_EQ(write.len(), (size_t)9);
  CHECK(!write.is_dense_ordered());
  CHECK(std::find(write.indices().begin(), write.indices().end(), center) != write.indices().end());
  CHECK(patch_diff_dense_fallback(SparseTokenMask::new_({0, 1, 2, 3, 4, 5, 6}, 25), grid, 0.25f).is_dense_ordered());
}

// crates/bevy_jepa/src/tests.rs:1917-1928
TEST(sparse_mask_bucket_preserves_changed_tokens) {
  const TokenGridShape grid(1, 32, 32);
  std::vector<size_t> idx(103);
  for (size_t i = 0; i < idx.size(); ++i) idx[i] = i;
  const auto changed = SparseTokenMask::new_(idx, grid.len());
  const auto bucketed = bucket_sparse_mask(changed, grid, DEFAULT_SPARSE_MASK_BUCKET_TOKENS);
  CHECK_EQ(bucketed.len(), (size_t)256);
  for (size_t i : changed.indices())
    CHECK(std::find(bucketed.indices().begin(), bucketed.indices().end(), i) != bucketed.indices().end());
  CHECK(!bucketed.is_dense_ordered());
}

// src/viewer.rs:1322-1340
TEST(bucketed_masks_keep_writes_exact_and_widen_encode_context) {
  const TokenGridShape grid(1, 32, 32);
  const size_t changed_index = coords_to_token_index(0, 15, 16, grid);
  const auto changed = SparseTokenMask::new_({changed_index}, grid.len());
  const auto masks = finalize_patch_diff_masks(changed, grid, FeatureFrameViewerConfig{});
  CHECK_EQ(masks.write_mask.indices(), changed.indices());
  CHECK_EQ(masks.encode_mask.len(), (size_t)103);
  CHECK(std::find(masks.encode_mask.indices().begin(), masks.encode_mask.indices().end(), changed_index) !=
        masks.encode_mask.indices().end());
}

// src/viewer.rs:1342-1376: the widths behind the prewarm lists (768 of the legacy step
// finalizes to the dense mask under the 0.75 fallback, so the reference's prewarm list omits it)
TEST(bucket_widths_follow_densities_or_legacy_step) {
  const FeatureFrameViewerConfig cfg;
  CHECK_EQ(cfg.sparse_mask_bucket_widths(TokenGridShape(1, 32, 32)), (std::vector<size_t>{103, 256, 512, 1024}));
  CHECK_EQ(cfg.sparse_mask_bucket_widths(TokenGridShape(1, 64, 64)), (std::vector<size_t>{410, 1024, 2048, 4096}));
  FeatureFrameViewerConfig legacy;
  legacy.sparse_mask_bucket_densities.clear();
  CHECK_EQ(legacy.sparse_mask_bucket_widths(TokenGridShape(1, 32, 32)), (std::vector<size_t>{256, 512, 768, 1024}));
  CHECK(finalize_patch_diff_masks(SparseTokenMask::evenly_spaced(1024, 768), TokenGridShape(1, 32, 32), legacy)
            .encode_mask.is_dense_ordered());
}

// src/viewer.rs:1377-1389
TEST(bucket_density_list_selects_next_configured_width) {
  const TokenGridShape grid(1, 32, 32);
  const auto mask = SparseTokenMask::evenly_spaced(grid.len(), 120);
  const auto masks = finalize_patch_diff_masks(mask, grid, FeatureFrameViewerConfig{});
  CHECK_EQ(masks.write_mask.indices(), mask.indices());
  CHECK_EQ(masks.encode_mask.len(), (size_t)256);
}

// src/viewer.rs:649-667, 732-752, 1012-1028: the selection a viewer config asks for
TEST(viewer_config_derives_the_patch_diff_selection) {
  FeatureFrameViewerConfig config;
  config.context_density = 0.25f;
  const TokenGridShape grid(1, 4, 4);
  const auto sp = patch_diff_sparsity_config(config, grid);
  CHECK_EQ(sp.context_tokens, (size_t)4);
  CHECK_EQ(sp.min_context_tokens, (size_t)1);  // min density 0 still keeps one token
  CHECK_EQ(sp.target_tokens, (size_t)12);
  CHECK_EQ(sp.dilation, DEFAULT_PATCH_DIFF_DILATION_TILES);
  CHECK(sp.allow_full_context && !sp.fill_to_context_tokens);
  CHECK_EQ(density_tokens(16, 0.0f, DensityRound::Round, 0.01f), (size_t)1);
  CHECK_EQ(density_tokens(1000, 0.1234f, DensityRound::Floor, 0.0f), (size_t)123);
  CHECK_EQ(density_tokens(1000, 0.1234f, DensityRound::Ceil, 0.0f), (size_t)124);
  CHECK_EQ(density_tokens(10, 5.0f, DensityRound::Round, 0.0f), (size_t)10);
  CHECK(!PatchDiffRefreshConfig{}.can_add_tokens());  // refresh is off by default
  CHECK(!PatchDiffRefreshConfig::disabled().can_add_tokens());
}

// src/tokens.rs:180-442 (SparseMaskBatch) and src/sparse_patchify.rs:290-300: uniform,
// fixed-width and ragged batches, their normalisation, padding and errors
TEST(sparse_mask_batch_kinds_padding_and_errors) {
  const auto u = SparseMaskBatch::from_rows({{3, 0}, {3, 0}}, 8);
  CHECK(u.is_uniform() && !u.is_ragged());
  // rows compare before they are sorted, as in the reference: equal sets in another order
  // make a fixed-width batch
  CHECK(!SparseMaskBatch::from_rows({{3, 0}, {0, 3}}, 8).is_uniform());
  CHECK_EQ(u.batch(), (size_t)2);
  CHECK_EQ(u.len(), (size_t)2);
  CHECK_EQ(u.valid_token_count(), (size_t)4);
  CHECK_EQ(u.rows()[1], (std::vector<size_t>{0, 3}));
  const auto f = SparseMaskBatch::from_rows({{5, 1}, {2, 7}}, 8);
  CHECK(!f.is_uniform() && !f.is_ragged());
  CHECK_EQ(f.rows()[0], (std::vector<size_t>{1, 5}));
  CHECK(!f.valid_token_mask().has_value());
  const auto r = SparseMaskBatch::from_rows({{4, 1, 6}, {2}}, 8);
  CHECK(r.is_ragged());
  CHECK_EQ(r.len(), (size_t)3);
  CHECK_EQ(r.valid_token_count(), (size_t)4);
  CHECK_EQ(r.padded_rows()[1], (std::vector<size_t>{2, 2, 2}));
  CHECK_EQ(*r.valid_token_mask(), (std::vector<float>{1, 1, 1, 1, 0, 0}));
  CHECK(!r.is_dense_ordered());
  CHECK(SparseMaskBatch::uniform(SparseTokenMask::all(4), 3).is_dense_ordered());
  CHECK_THROWS_WITH(SparseMaskBatch::uniform(SparseTokenMask::all(4), 0), "sparse mask batch must be non-empty");
  CHECK_THROWS_WITH(SparseMaskBatch::fixed_width({{1, 1}}, 4), "fixed-width sparse mask row contains duplicate indices");
  CHECK_THROWS_WITH(SparseMaskBatch::fixed_width({{1, 2}, {3}}, 4), "fixed-width sparse mask rows must have equal lengths");
  CHECK_THROWS_WITH(SparseMaskBatch::ragged({{1}, {}}, 4), "ragged sparse mask rows must be non-empty");
  CHECK_THROWS_WITH(SparseMaskBatch::ragged({{9}}, 4), "sparse token index outside dense token range");
  CHECK_THROWS_WITH(SparsePatchifyBatchPlan::new_(r, TokenGridShape(2, 2, 2)),
                    "sparse patchify batch plans require uniform or fixed-width masks; use ragged rollout grouping");
  CHECK_THROWS_WITH(SparsePatchifyBatchPlan::new_(f, TokenGridShape(1, 2, 2)),
                    "sparse patchify batch mask dense token count must match grid");
}

// src/positional.rs:104-111
TEST(sparse_positional_encoding_has_expected_shape) {
  const auto values = sparse_3d_sincos_pos_embed(10, TokenGridShape(2, 2, 2), {0, 7});
  CHECK_EQ(values.size(), (size_t)20);
  CHECK_EQ(values[0], 0.0f);
  CHECK_EQ(values[3], 1.0f);
}

TEST(abi_version_matches_header) { CHECK_EQ(bjf_abi_version(), BJF_ABI_VERSION); }

TEST_MAIN()
