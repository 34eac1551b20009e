"""Parity of the CUDA front end (through the C ABI) with the CPU oracle and the
reference's golden vectors.

Bars: token indices, counts and cache slots bit-exact; features within a normwise max
relative error of 1e-2 for f16/bf16 inputs and 1e-4 for f32 inputs (the tolerance the
front end is specified to); patch-diff scores within 1e-5 relative (f32 accumulation in a
different order than the oracle's f64)."""
import numpy as np
import pytest

import burn_jepa_b200 as bj
import oracle
from burn_jepa_b200 import workloads
from helpers import (changed_patch_video, conv3d_cases, conv3d_inputs, known_answers, max_rel_err,
                     token_values, two_frame_changed_patches)

pytestmark = pytest.mark.gpu

KA = known_answers()
TOL_HALF = 1e-2
TOL_F32 = 1e-4
TOL_SCORES = 1e-5


def _t(a, dev, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


@pytest.fixture(autouse=True)
def _no_device_timeouts(cuda_device):
    yield
    assert not bj.device_error_check(), "a kernel reported a bounded-wait timeout"


def _dt(name):
    import torch

    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


def _as_oracle_input(t):
    """The exact f32 values of a (possibly half-precision) device tensor."""
    return t.float().cpu().numpy()


# ---------------------------------------------------------------------------
# patch-diff scores + selection
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", KA["patch_diff_changed_patch"]["cases"], ids=lambda c: f"thr{c['threshold']}")
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_patch_diff_changed_patch_golden(cuda_device, case, dtype):
    c = KA["patch_diff_changed_patch"]
    ch = c["changed"]
    video = changed_patch_video(c["video_shape"], ch["frame"], ch["y0"], ch["y1"], ch["x0"], ch["x1"])
    cfg = bj.PatchDiffConfig.new(case["threshold"], c["context_tokens"], c["target_tokens"])
    scores, idx, counts = bj.patch_diff_context_mask(_t(video, cuda_device, _dt(dtype)), c["tubelet_size"],
                                                     c["patch_size"], c["grid"], cfg)
    n = int(counts[0])
    assert idx[0, :n].cpu().tolist() == case["context"]
    ref = oracle.patch_diff_token_scores(video, c["tubelet_size"], c["patch_size"])
    np.testing.assert_allclose(scores[0].cpu().numpy(), ref, rtol=TOL_SCORES, atol=1e-7)


@pytest.mark.parametrize("key", ["adaptive_changed_patches", "adaptive_static_keeps_minimum"])
def test_adaptive_video_golden(cuda_device, key):
    c = KA[key]
    video = two_frame_changed_patches(c["video_shape"], c["changed_patches"], c["patch_size"], c["frame"])
    cfg = bj.PatchDiffConfig.adaptive_threshold(*c["config"]["adaptive_threshold"])
    _, idx, counts = bj.patch_diff_context_mask(_t(video, cuda_device), c["tubelet_size"], c["patch_size"],
                                                c["grid"], cfg)
    got = idx[0, :int(counts[0])].cpu().tolist()
    if "context" in c:
        assert got == c["context"]
    else:
        assert len(got) == c["context_len"]
        ref = oracle.patch_diff_context_mask_from_video(video, c["tubelet_size"], c["patch_size"],
                                                        oracle.TokenGridShape(*c["grid"]),
                                                        oracle.PatchDiffConfig.adaptive_threshold(
                                                            *c["config"]["adaptive_threshold"]))
        assert got == ref.tolist()


@pytest.mark.parametrize("key", ["adaptive_no_cap_above_threshold", "adaptive_zero_threshold_keeps_all"])
def test_adaptive_scores_golden(cuda_device, key):
    c = KA[key]
    cfg = bj.PatchDiffConfig.adaptive_threshold(*c["config"]["adaptive_threshold"])
    idx, counts = bj.patch_diff_context_mask_from_scores(_t(np.array(c["scores"], np.float32), cuda_device),
                                                         c["grid"], cfg)
    assert idx[0, :int(counts[0])].cpu().tolist() == c["context"]


SCORE_SHAPES = [
    # (streams, B, C, T, H, W, kt, P)
    (1, 1, 3, 16, 64, 64, 2, 16),   # ViT-L clip geometry, reduced frame size
    (3, 1, 3, 2, 96, 128, 2, 16),   # live streams, two-frame steps
    (1, 2, 3, 4, 32, 48, 2, 16),    # batch summed into one map
    (2, 1, 3, 5, 32, 32, 1, 16),    # tubelet 1: pairs (t-1, t), zeros for t = 0
    (1, 1, 2, 6, 24, 40, 3, 8),     # tubelet 3 (two pairs), patch 8
    (1, 1, 3, 4, 36, 36, 2, 12),    # patch 12: generic (scalar) kernel
]


@pytest.mark.parametrize("shape", SCORE_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_patch_diff_scores_match_oracle(cuda_device, shape, dtype):
    S, B, C, T, H, W, kt, P = shape
    video = workloads.rect_perturbation_clips(seed=hash(shape) & 0xFFFF, streams=S * B, channels=C, frames=T,
                                              height=H, width=W, area_fraction=0.3).reshape(S, B, C, T, H, W)
    v = _t(video, cuda_device, _dt(dtype))
    scores = bj.patch_diff_token_scores(v if S > 1 else v[0], kt, P)
    scores = scores.reshape(S, -1).cpu().numpy()
    xs = _as_oracle_input(v)
    for s in range(S):
        ref = oracle.patch_diff_token_scores(xs[s], kt, P)
        np.testing.assert_allclose(scores[s], ref, rtol=TOL_SCORES, atol=1e-7)


@pytest.mark.parametrize("density", [0.05, 0.25, 0.6])
def test_patch_diff_masks_bit_exact_with_gap_threshold(cuda_device, density):
    S, C, T, H, W, kt, P = 4, 3, 2, 128, 128, 2, 16
    video = workloads.rect_perturbation_clips(seed=int(density * 1000), streams=S, channels=C, frames=T, height=H,
                                              width=W, area_fraction=density)
    v = _t(video, cuda_device, _dt("f16")).reshape(S, 1, C, T, H, W)
    xs = _as_oracle_input(v)
    grid = (T // kt, H // P, W // P)
    n = grid[0] * grid[1] * grid[2]
    for s in range(S):
        ref_scores = oracle.patch_diff_token_scores(xs[s], kt, P)
        thr = workloads.choose_threshold(ref_scores, density)
        cfg = bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
        _, idx, counts = bj.patch_diff_context_mask(v[s], kt, P, grid, cfg)
        ref = oracle.patch_diff_context_mask_from_video(xs[s], kt, P, oracle.TokenGridShape(*grid),
                                                        oracle.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1))
        assert idx[0, :int(counts[0])].cpu().numpy().tolist() == ref.tolist()


def _oracle_cfg(c: bj.PatchDiffConfig) -> oracle.PatchDiffConfig:
    return oracle.PatchDiffConfig(c.threshold, c.context_tokens, c.target_tokens, c.dilation, c.min_context_tokens,
                                  c.fill_to_context_tokens, c.allow_full_context)


SELECT_CONFIGS = {
    "new_cap_binds": bj.PatchDiffConfig.new(0.2, 40, 8),
    "new_fill_to_context": bj.PatchDiffConfig.new(0.95, 60, 8),
    "topk_threshold_zero": bj.PatchDiffConfig.new(0.0, 77, 8),
    "adaptive_no_cap": bj.PatchDiffConfig.adaptive_threshold(0.5, 5, 10, 1),
    "adaptive_min_fill": bj.PatchDiffConfig.adaptive_threshold(0.99, 17, 300, 1),
    "adaptive_zero_threshold": bj.PatchDiffConfig.adaptive_threshold(0.0, 1, 1, 1),
    "dilated_union": bj.PatchDiffConfig.adaptive_threshold(0.97, 1, 4096, 1).with_dilation(1),
    "dilated_cap_binds": bj.PatchDiffConfig.new(0.8, 50, 8).with_dilation(1),
    "dilated_fill": bj.PatchDiffConfig.new(0.999, 90, 8).with_dilation(2),
    "full_context_allowed": bj.PatchDiffConfig.new(0.3, 10**9, 8).with_allow_full_context(True),
}


@pytest.mark.parametrize("name", sorted(SELECT_CONFIGS))
@pytest.mark.parametrize("ties", [False, True])
def test_selection_matches_oracle(cuda_device, name, ties):
    cfg = SELECT_CONFIGS[name]
    grid = (2, 12, 16)
    n = grid[0] * grid[1] * grid[2]
    streams = 3
    rng = np.random.default_rng(5 + ties)
    scores = rng.uniform(0, 1, size=(streams, n)).astype(np.float32)
    if ties:
        scores = np.round(scores * 8) / 8  # many equal scores: ties break by ascending index
    idx, counts = bj.patch_diff_context_mask_from_scores(_t(scores, cuda_device), grid, cfg)
    for s in range(streams):
        ref = oracle.patch_diff_context_mask_from_scores(scores[s], oracle.TokenGridShape(*grid), _oracle_cfg(cfg))
        assert idx[s, :int(counts[s])].cpu().numpy().tolist() == ref.tolist(), (name, s)


@pytest.mark.parametrize("n", [2, 5, 1000, 4096, 32768])
def test_selection_sizes(cuda_device, n):
    grid = (1, 1, n)
    scores = np.random.default_rng(n).uniform(0, 1, size=(2, n)).astype(np.float32)
    for cfg in (bj.PatchDiffConfig.new(0.5, n // 3 + 1, 1), bj.PatchDiffConfig.adaptive_threshold(0.9, 2, n, 1)):
        idx, counts = bj.patch_diff_context_mask_from_scores(_t(scores, cuda_device), grid, cfg)
        for s in range(2):
            ref = oracle.patch_diff_context_mask_from_scores(scores[s], oracle.TokenGridShape(*grid), _oracle_cfg(cfg))
            assert idx[s, :int(counts[s])].cpu().numpy().tolist() == ref.tolist()


def test_selection_rejects_oversized_grid(cuda_device):
    import torch

    scores = torch.zeros((1, 40000), device=cuda_device)
    with pytest.raises(bj.BjfError, match="up to 32768 tokens"):
        bj.patch_diff_context_mask_from_scores(scores, (1, 1, 40000), bj.PatchDiffConfig.new(0.5, 10, 1))


# ---------------------------------------------------------------------------
# plans
# ---------------------------------------------------------------------------
def test_plan_coords_golden_uniform(cuda_device):
    import torch

    c = KA["plan_coords"]
    idx = torch.tensor([c["mask"]], dtype=torch.int32, device=cuda_device)
    coords, total = bj.sparse_patchify_plan_coords(idx, c["grid"], batch=c["batch"])
    assert int(total.item()) == len(c["coords"])
    assert coords.cpu().tolist() == c["coords"]


def test_plan_coords_ragged_batch(cuda_device):
    import torch

    grid = (3, 5, 7)
    n = 105
    rng = np.random.default_rng(0)
    rows = [np.sort(rng.choice(n, size=k, replace=False)) for k in (5, 0, 17, 1)]
    stride = n
    idx = np.zeros((4, stride), np.int32)
    for b, r in enumerate(rows):
        idx[b, :len(r)] = r
    counts = torch.tensor([len(r) for r in rows], dtype=torch.int32, device=cuda_device)
    coords, total = bj.sparse_patchify_plan_coords(_t(idx, cuda_device), grid, batch=4, counts=counts,
                                                   capacity=4 * n)
    tot = int(total.item())
    assert tot == sum(len(r) for r in rows)
    expect = np.concatenate([oracle.sparse_patchify_plan_coords(r.astype(np.int64), oracle.TokenGridShape(*grid), 1)
                             * np.array([0, 1, 1, 1], np.int32) + np.array([b, 0, 0, 0], np.int32)
                             for b, r in enumerate(rows) if len(r)])
    assert coords[:tot].cpu().numpy().tolist() == expect.tolist()


# ---------------------------------------------------------------------------
# sparse patchify (gather-GEMM)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case_and_ref", conv3d_cases(), ids=lambda c: c[0]["name"])
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_patchify_conv3d_golden(cuda_device, case_and_ref, dtype):
    case, ref = case_and_ref
    x, w, b = conv3d_inputs(case)
    g = oracle.TokenGridShape(case["T"] // case["kt"], case["H"] // case["P"], case["W"] // case["P"])
    n = len(g)
    mask = np.arange(n, dtype=np.int64) if n <= 8 else np.array(sorted({0, 1, n // 2, n - 2, n - 1}), np.int64)
    coords = oracle.sparse_patchify_plan_coords(mask, g, case["batch"])
    cfg = bj.PatchifyConfig(case["C"], case["D"], case["T"], case["H"], case["W"], case["kt"], case["P"], case["P"])
    xd, wd = _t(x, cuda_device, _dt(dtype)), _t(w, cuda_device, _dt(dtype))
    out = bj.sparse_patchify3d_forward(cfg, xd, _t(coords, cuda_device), wd,
                                       None if b is None else _t(b, cuda_device))
    got = out.cpu().numpy().reshape(case["batch"], len(mask), -1)
    if dtype == "f32":
        assert max_rel_err(got, ref[:, mask]) <= TOL_F32
    else:
        # against the golden Conv3d on the original f32 values (includes input rounding) ...
        assert max_rel_err(got, ref[:, mask]) <= TOL_HALF
        # ... and tighter against the oracle on the exact half-precision values
        o = oracle.sparse_patchify3d_forward(cfg_o(cfg), _as_oracle_input(xd), coords, _as_oracle_input(wd), b)
        assert max_rel_err(got.reshape(o.shape), o) <= 1e-4


def cfg_o(c: bj.PatchifyConfig) -> oracle.PatchifyConfig:
    return oracle.PatchifyConfig(c.in_channels, c.out_channels, c.frames, c.height, c.width, c.tubelet_size,
                                 c.patch_h, c.patch_w)


PATCHIFY_SHAPES = [
    # (batch, C, T, H, W, kt, P, D, rows)
    (1, 3, 16, 64, 64, 2, 16, 1024, 300),    # ViT-L/16 width, rows not a multiple of 128
    (2, 3, 2, 128, 96, 2, 16, 1408, 131),    # ViT-g/16 width (six 240-column tiles)
    (2, 3, 2, 64, 128, 2, 16, 257, 300),     # two 144-column tiles, odd D (unaligned output rows)
    (1, 3, 4, 64, 64, 2, 16, 1100, 400),     # five 224-column tiles (split K applies)
    (4, 3, 2, 64, 64, 2, 16, 768, 512),      # ViT-B width, several full M tiles
    (1, 3, 4, 32, 32, 2, 16, 32, 4),         # tiny config
    (3, 3, 2, 32, 64, 2, 16, 96, 1),         # a single row
]


@pytest.mark.parametrize("shape", PATCHIFY_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype,out_dtype", [("f16", "f32"), ("bf16", "f32"), ("f16", "f16"), ("bf16", "bf16"),
                                             ("f32", "f32")])
def test_patchify_matches_oracle(cuda_device, shape, dtype, out_dtype):
    B, C, T, H, W, kt, P, D, rows = shape
    g = oracle.TokenGridShape(T // kt, H // P, W // P)
    x = workloads.splitmix_uniform(1000 + rows, (B, C, T, H, W))
    w = workloads.splitmix_normal(2000 + D, (D, C, kt, P, P), 0.02)
    b = workloads.splitmix_normal(3000 + D, (D,), 0.02)
    rng = np.random.default_rng(rows)
    coords = np.stack([rng.integers(0, B, rows), rng.integers(0, g.depth, rows), rng.integers(0, g.height, rows),
                       rng.integers(0, g.width, rows)], axis=1).astype(np.int32)
    cfg = bj.PatchifyConfig(C, D, T, H, W, kt, P, P)
    xd, wd = _t(x, cuda_device, _dt(dtype)), _t(w, cuda_device, _dt(dtype))
    out = bj.sparse_patchify3d_forward(cfg, xd, _t(coords, cuda_device), wd, _t(b, cuda_device),
                                       out_dtype=_dt(out_dtype))
    ref = oracle.sparse_patchify3d_forward(cfg_o(cfg), _as_oracle_input(xd), coords, _as_oracle_input(wd), b)
    err = max_rel_err(out.float().cpu().numpy(), ref)
    assert err <= (TOL_F32 if dtype == "f32" else TOL_HALF), err
    if dtype != "f32" and out_dtype == "f32":
        assert err <= 1e-4, err  # f32 accumulation of exact half products


def test_patchify_out_of_range_rows_are_zero_and_bias_optional(cuda_device):
    B, C, T, H, W, kt, P, D = 1, 3, 2, 64, 64, 2, 16, 256
    x = workloads.splitmix_uniform(5, (B, C, T, H, W))
    w = workloads.splitmix_normal(6, (D, C, kt, P, P), 0.02)
    coords = np.array([[0, 0, 1, 1], [1, 0, 0, 0], [0, 1, 0, 0], [0, 0, 4, 0], [0, 0, 0, -1], [0, 0, 3, 3]],
                      np.int32)
    cfg = bj.PatchifyConfig(C, D, T, H, W, kt, P, P)
    for dt in ("f16", "f32"):
        out = bj.sparse_patchify3d_forward(cfg, _t(x, cuda_device, _dt(dt)), _t(coords, cuda_device),
                                           _t(w, cuda_device, _dt(dt)), None).cpu().numpy()
        assert np.all(out[1:5] == 0)
        ref = oracle.sparse_patchify3d_forward(cfg_o(cfg), x, coords, w, None)
        assert max_rel_err(out, ref) <= TOL_HALF


# ---------------------------------------------------------------------------
# token-cache write
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("key", ["feature_memory_sequences", "feature_memory_write_by_index",
                                 "feature_memory_fill_over_time", "feature_memory_masked_then_encoder_output"])
def test_feature_memory_golden_sequences(cuda_device, key):
    import torch

    c = KA[key]
    B, (d, h, w), D = c["batch"], c["grid"], c["embed_dim"]
    N = d * h * w
    feats = torch.zeros((B, N, D), device=cuda_device)
    obs = torch.zeros((B, N), device=cuda_device)
    age = torch.zeros((B, N), device=cuda_device)
    for step, st in enumerate(c["steps"]):
        tok = _t(np.array(st["tokens"], np.float32).reshape(st["tokens_shape"]), cuda_device)
        idx = _t(np.array(st["indices"], np.int32).reshape(B, -1), cuda_device)
        bj.feature_memory_assign_latest(feats, obs, age, tok, idx, age_observed=step > 0)
        if "features" in st:
            np.testing.assert_allclose(feats.cpu().numpy().ravel(), st["features"], atol=1e-5)
        if "observed" in st:
            np.testing.assert_allclose(obs.cpu().numpy().ravel(), st["observed"], atol=1e-5)
        if "age" in st:
            np.testing.assert_allclose(age.cpu().numpy().ravel(), st["age"], atol=1e-5)
    if "final_features" in c:
        np.testing.assert_allclose(feats.cpu().numpy().ravel(), c["final_features"], atol=1e-5)
        np.testing.assert_allclose(obs.cpu().numpy().ravel(), c["final_observed"], atol=1e-5)


def test_feature_memory_high_density_golden(cuda_device):
    import torch

    c = KA["feature_memory_high_density_512"]
    N, D, keep = 1024, c["embed_dim"], c["keep"]
    initial = token_values(N, D, c["initial_offset"])
    feats = _t(initial[None], cuda_device)
    obs = torch.ones((1, N), device=cuda_device)
    age = torch.zeros((1, N), device=cuda_device)
    upd = token_values(keep, D, c["update_offset"])
    bj.feature_memory_assign_latest(feats, obs, age, _t(upd[None], cuda_device),
                                    _t(np.arange(keep, dtype=np.int32)[None], cuda_device), age_observed=True)
    f = feats.cpu().numpy()[0]
    np.testing.assert_allclose(f[:keep], upd, atol=1e-5)
    np.testing.assert_allclose(f[keep:], initial[keep:], atol=1e-5)
    a = age.cpu().numpy()[0]
    assert a[0] == 0 and a[keep - 1] == 0 and a[keep] == 1


def test_feature_memory_shape_errors_on_device(cuda_device):
    import torch

    feats = torch.zeros((1, 4, 2), device=cuda_device)
    obs = torch.zeros((1, 4), device=cuda_device)
    with pytest.raises(bj.BjfError, match="index dims mismatch"):
        bj.feature_memory_assign_latest(feats, obs, obs.clone(), torch.zeros((1, 1, 2), device=cuda_device),
                                        torch.zeros((1, 2), dtype=torch.int32, device=cuda_device), False)
    with pytest.raises(bj.BjfError, match="requires at least one token"):
        bj.feature_memory_assign_latest(feats, obs, obs.clone(), torch.zeros((1, 0, 2), device=cuda_device),
                                        torch.zeros((1, 0), dtype=torch.int32, device=cuda_device), False)


@pytest.mark.parametrize("cache_dtype,tok_dtype,D", [("f32", "f32", 1024), ("f16", "f16", 1024), ("f16", "f32", 1024),
                                                     ("bf16", "f32", 768), ("f32", "f32", 13), ("f16", "f16", 40)])
def test_feature_memory_random_matches_oracle(cuda_device, cache_dtype, tok_dtype, D):
    B, N, S = 3, 4096 if D > 64 else 300, 410 if D > 64 else 37
    rng = np.random.default_rng(D)
    cache0 = workloads.splitmix_normal(D, (B, N, D))
    obs0 = (rng.uniform(size=(B, N)) < 0.5).astype(np.float32)
    age0 = rng.integers(0, 5, size=(B, N)).astype(np.float32)
    idx = np.stack([np.sort(rng.choice(N, S, replace=False)) for _ in range(B)]).astype(np.int32)
    idx[0, 0] = -3  # skipped
    idx[1, -1] = N + 7  # skipped
    tok = workloads.splitmix_normal(D + 1, (B, S, D))
    feats = _t(cache0, cuda_device, _dt(cache_dtype))
    obs, age = _t(obs0, cuda_device), _t(age0, cuda_device)
    tokd = _t(tok, cuda_device, _dt(tok_dtype))
    bj.feature_memory_assign_latest(feats, obs, age, tokd, _t(idx, cuda_device), age_observed=True)
    ref_f = _as_oracle_input(_t(cache0, cuda_device, _dt(cache_dtype)))
    ref_o, ref_a = obs0.copy(), age0.copy()
    oracle.feature_memory_assign_latest(ref_f, ref_o, ref_a, _as_oracle_input(tokd), idx, age_observed=True)
    got = feats.float().cpu().numpy()
    if cache_dtype == tok_dtype:
        assert np.array_equal(got, ref_f)
    else:
        assert max_rel_err(got, ref_f) <= TOL_HALF
    assert np.array_equal(obs.cpu().numpy(), ref_o) and np.array_equal(age.cpu().numpy(), ref_a)
