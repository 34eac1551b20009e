"""Pins the CPU oracle to the reference's own known answers (CPU only).

Every case here is an assertion of the reference's test suite (file:line in the
fixture), or torch F.conv3d for the patch-embed arithmetic.  The oracle must pass all
of them before it is trusted as the checker of the CUDA library.
"""
import numpy as np
import pytest

import oracle
from helpers import changed_patch_video, conv3d_cases, conv3d_inputs, known_answers, token_values, two_frame_changed_patches

KA = known_answers()


def test_positional_round_trip():
    c = KA["positional_round_trip"]
    g = oracle.TokenGridShape(*c["grid"])
    assert oracle.coords_to_token_index(*c["coords"], g) == c["index"]
    assert oracle.token_index_to_coords(c["index"], g) == tuple(c["coords"])


def test_tiny_grid_and_context_target_masks():
    c = KA["tiny_config_grid"]
    g = oracle.TokenGridShape(c["num_frames"] // c["tubelet_size"], c["image_size"] // c["patch_size"],
                              c["image_size"] // c["patch_size"])
    assert [g.depth, g.height, g.width] == c["grid"] and len(g) == c["num_patches"]
    m = KA["context_target_masks_tiny"]
    ctx, tgt = oracle.make_context_target_masks(g, m["keep_ratio"])
    assert ctx.tolist() == m["context"] and tgt.tolist() == m["target"]


def test_token_mask_helpers():
    c = KA["mask_sort_dedup_complement"]
    mask = oracle.sparse_token_mask_new(c["indices"], c["dense_len"])
    assert mask.tolist() == c["mask"]
    assert oracle.complement(mask, c["dense_len"]).tolist() == c["complement"]
    c = KA["padded_to_multiple_bucket"]
    p = oracle.padded_to_multiple(oracle.sparse_token_mask_new(c["indices"], c["dense_len"]), c["dense_len"],
                                  c["multiple"])
    assert len(p) == c["len"] and all(i in p for i in c["contains"])
    assert not (len(p) == c["dense_len"] and p.tolist() == list(range(c["dense_len"])))
    c = KA["padded_to_multiple_dense"]
    p = oracle.padded_to_multiple(np.array(c["indices"]), c["dense_len"], c["multiple"])
    assert p.tolist() == c["mask"]
    c = KA["target_mask_from_context"]
    t = oracle.target_mask_from_context(c["context"], c["dense_len"], c["target_tokens"])
    assert len(t) == c["len"] and not set(t.tolist()) & set(c["context"])


def test_sparse_token_mask_errors():
    with pytest.raises(oracle.OracleError, match="outside dense token range"):
        oracle.sparse_token_mask_new([0, 9], 5)
    with pytest.raises(oracle.OracleError, match="nonzero"):
        oracle.sparse_token_mask_new([], 0)


def test_plan_coords_golden():
    c = KA["plan_coords"]
    g = oracle.TokenGridShape(*c["grid"])
    coords = oracle.sparse_patchify_plan_coords(c["mask"], g, c["batch"])
    assert coords.tolist() == c["coords"]


@pytest.mark.parametrize("case", KA["patch_diff_changed_patch"]["cases"], ids=lambda c: f"thr{c['threshold']}")
def test_patch_diff_selects_changed_patch(case):
    c = KA["patch_diff_changed_patch"]
    ch = c["changed"]
    video = changed_patch_video(c["video_shape"], ch["frame"], ch["y0"], ch["y1"], ch["x0"], ch["x1"])
    g = oracle.TokenGridShape(*c["grid"])
    cfg = oracle.PatchDiffConfig.new(case["threshold"], c["context_tokens"], c["target_tokens"])
    ctx = oracle.patch_diff_context_mask_from_video(video, c["tubelet_size"], c["patch_size"], g, cfg)
    assert ctx.tolist() == case["context"]
    tgt = oracle.target_mask_from_context(ctx, len(g), c["target_tokens"])
    assert len(tgt) == c["target_len"]


def test_adaptive_threshold_cases():
    for key in ("adaptive_changed_patches", "adaptive_static_keeps_minimum"):
        c = KA[key]
        video = two_frame_changed_patches(c["video_shape"], c["changed_patches"], c["patch_size"], c["frame"])
        g = oracle.TokenGridShape(*c["grid"])
        cfg = oracle.PatchDiffConfig.adaptive_threshold(*c["config"]["adaptive_threshold"])
        ctx = oracle.patch_diff_context_mask_from_video(video, c["tubelet_size"], c["patch_size"], g, cfg)
        if "context" in c:
            assert ctx.tolist() == c["context"], key
        else:
            assert len(ctx) == c["context_len"], key
    for key in ("adaptive_no_cap_above_threshold", "adaptive_zero_threshold_keeps_all"):
        c = KA[key]
        g = oracle.TokenGridShape(*c["grid"])
        cfg = oracle.PatchDiffConfig.adaptive_threshold(*c["config"]["adaptive_threshold"])
        ctx = oracle.patch_diff_context_mask_from_scores(np.array(c["scores"], np.float32), g, cfg)
        assert ctx.tolist() == c["context"], key


def test_patch_diff_threshold_errors():
    g = oracle.TokenGridShape(1, 2, 2)
    for bad in (float("nan"), -0.5, float("inf")):
        with pytest.raises(oracle.OracleError, match="finite and non-negative"):
            oracle.patch_diff_context_mask_from_scores(np.zeros(4, np.float32), g,
                                                       oracle.PatchDiffConfig.new(bad, 1, 1))
    with pytest.raises(oracle.OracleError, match="unexpected score length"):
        oracle.patch_diff_context_mask_from_scores(np.zeros(3, np.float32), g, oracle.PatchDiffConfig.new(0.1, 1, 1))


def _run_memory_steps(case):
    B, (d, h, w), D = case["batch"], case["grid"], case["embed_dim"]
    N = d * h * w
    feats = np.zeros((B, N, D), np.float32)
    obs = np.zeros((B, N), np.float32)
    age = np.zeros((B, N), np.float32)
    step = 0
    for st in case["steps"]:
        tok = np.array(st["tokens"], np.float32).reshape(st["tokens_shape"])
        idx = np.array(st["indices"], np.int32).reshape(B, -1)
        oracle.feature_memory_assign_latest(feats, obs, age, tok, idx, age_observed=step > 0)
        step += 1
        if "features" in st:
            np.testing.assert_allclose(feats.ravel(), st["features"], atol=1e-5)
        if "observed" in st:
            np.testing.assert_allclose(obs.ravel(), st["observed"], atol=1e-5)
        if "age" in st:
            np.testing.assert_allclose(age.ravel(), st["age"], atol=1e-5)
        if "step" in st:
            assert step == st["step"]
    return feats, obs, age


@pytest.mark.parametrize("key", ["feature_memory_sequences", "feature_memory_write_by_index",
                                 "feature_memory_fill_over_time", "feature_memory_masked_then_encoder_output"])
def test_feature_memory_sequences(key):
    c = KA[key]
    feats, obs, _ = _run_memory_steps(c)
    if "final_features" in c:
        np.testing.assert_allclose(feats.ravel(), c["final_features"], atol=1e-5)
        np.testing.assert_allclose(obs.ravel(), c["final_observed"], atol=1e-5)


def test_feature_memory_high_density():
    c = KA["feature_memory_high_density_512"]
    N, D = c["grid"][0] * c["grid"][1] * c["grid"][2], c["embed_dim"]
    keep = -(-N * c["keep_percent"] // 100)
    assert keep == c["keep"]
    initial = token_values(N, D, c["initial_offset"])
    feats = initial[None].copy()
    obs = np.ones((1, N), np.float32)  # dense-ordered prime (feature_memory.rs:292-335)
    age = np.zeros((1, N), np.float32)
    upd = token_values(keep, D, c["update_offset"])
    oracle.feature_memory_assign_latest(feats, obs, age, upd[None], np.arange(keep, dtype=np.int32)[None],
                                        age_observed=True)
    np.testing.assert_allclose(feats[0, :keep], upd, atol=1e-5)
    np.testing.assert_allclose(feats[0, keep:], initial[keep:], atol=1e-5)
    assert np.all(np.abs(obs - 1) < 1e-5)
    assert age[0, 0] == 0 and age[0, keep - 1] == 0 and age[0, keep] == 1


def test_feature_memory_skips_out_of_range_indices():
    feats = np.zeros((1, 4, 2), np.float32)
    obs = np.zeros((1, 4), np.float32)
    age = np.zeros((1, 4), np.float32)
    oracle.feature_memory_assign_latest(feats, obs, age, np.ones((1, 3, 2), np.float32),
                                        np.array([[-1, 2, 4]], np.int32), age_observed=False)
    assert obs.ravel().tolist() == [0, 0, 1, 0]
    assert feats[0, 2].tolist() == [1, 1] and feats.sum() == 2


@pytest.mark.parametrize("case_and_ref", conv3d_cases(), ids=lambda c: c[0]["name"])
def test_oracle_patchify_matches_torch_conv3d(case_and_ref):
    case, ref = case_and_ref
    x, w, b = conv3d_inputs(case)
    cfg = oracle.PatchifyConfig(case["C"], case["D"], case["T"], case["H"], case["W"], case["kt"], case["P"], case["P"])
    dense = oracle.patch_embed3d_dense(cfg, x, w, b)
    np.testing.assert_allclose(dense, ref, rtol=1e-5, atol=1e-6)
    # sparse == dense gathered at the selected tokens (tests/sparse_patchify_cuda.rs:45-82 semantics)
    n = ref.shape[1]
    g = oracle.TokenGridShape(case["T"] // case["kt"], case["H"] // case["P"], case["W"] // case["P"])
    mask = np.array(sorted({0, n // 3, n - 1}), dtype=np.int64)
    coords = oracle.sparse_patchify_plan_coords(mask, g, case["batch"])
    sparse = oracle.sparse_patchify3d_forward(cfg, x, coords, w, b)
    np.testing.assert_allclose(sparse.reshape(case["batch"], len(mask), -1), ref[:, mask], rtol=1e-5, atol=1e-6)


def test_apply_token_mask_gather_semantics():
    c = KA["apply_token_mask_gather"]
    tokens = np.array(c["tokens"], np.float32).reshape(c["shape"])
    assert tokens[:, c["indices"]].ravel().tolist() == c["gathered"]


def test_splitmix64_matches_reference_mixer():
    from burn_jepa_b200 import workloads

    seq = workloads.splitmix64(12345, 3)
    g = 0x9E3779B97F4A7C15
    for i in range(3):
        assert int(seq[i]) == oracle.splitmix64((12345 + i * g) & 0xFFFFFFFFFFFFFFFF)
