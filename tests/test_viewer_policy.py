"""The live viewer's patch-diff policy (src/viewer.rs): the RGBA u8 scorer with global
lighting compensation, the dense fallback, dilation and encode-bucket padding.

CPU: the oracle against the reference's own tests (src/viewer.rs tests,
crates/bevy_jepa/src/tests.rs).  GPU (marked): the device scorer against the oracle.
Bars: per-pixel arithmetic is rounded as the reference's.  The frame means are sums over
every pixel, which the reference accumulates sequentially in f32 and the device in f64 from
per-block partials: the device means are checked against the exact (f64) means within 1e-6,
and against the oracle (the reference's arithmetic) within the worst-case error of its f32
sum, pixels x 2^-24 x mean |term|; the scores, which subtract the means when compensating,
within that bound plus 1e-5.  The lighting decision agrees exactly away from its boundary."""
import numpy as np
import pytest

import oracle

DEFAULT_PATCH_DIFF_THRESHOLD = np.float32(1.0) - np.float32(0.97)  # src/viewer.rs:19-25


def test_oracle_ignores_uniform_lighting_shift():
    # src/viewer.rs:1391-1403
    grid = oracle.TokenGridShape(1, 4, 4)
    prev = np.full(64 * 64 * 4, 80, np.uint8)
    cur = np.full(64 * 64 * 4, 110, np.uint8)
    scores, st = oracle.patch_diff_scores_from_rgba(prev, cur, 64, 16, grid)
    assert np.all(scores < DEFAULT_PATCH_DIFF_THRESHOLD)
    assert st.compensate_global_lighting == 1


def test_oracle_dilates_direct_hits():
    # src/viewer.rs:1405-1453: adaptive threshold 0.10 with 1-tile dilation around (2, 1)
    grid = oracle.TokenGridShape(1, 4, 4)
    center = 2 * 4 + 1
    scores = np.zeros(16, np.float32)
    scores[center] = 0.5
    cfg = oracle.PatchDiffConfig.adaptive_threshold(0.10, 1, 16, 1).with_dilation(1)
    got = oracle.patch_diff_context_mask_from_scores(scores, grid, cfg)
    assert got.tolist() == [r * 4 + c for r in (1, 2, 3) for c in (0, 1, 2)]
    exact = oracle.patch_diff_context_mask_from_scores(scores, grid, oracle.PatchDiffConfig.adaptive_threshold(0.10, 1, 16, 1))
    assert exact.tolist() == [center]


def test_oracle_dense_cutoff_runs_before_dilation():
    # src/viewer.rs:1455-1481 (and crates/bevy_jepa/src/tests.rs:1868-1910): direct mask ->
    # dense fallback at 0.25 -> 1-tile dilation gives 9 tokens, not the dense grid
    grid = oracle.TokenGridShape(1, 5, 5)
    center = 2 * 5 + 2
    scores = np.zeros(25, np.float32)
    scores[center] = 0.5
    direct = oracle.patch_diff_context_mask_from_scores(scores, grid, oracle.PatchDiffConfig.adaptive_threshold(0.10, 1, 25, 1))
    fallback = oracle.patch_diff_dense_fallback(direct, 25, 0.25)
    write = oracle.dilate_sparse_patch_mask(fallback, grid, 1)
    assert len(write) == 9 and center in write.tolist() and write.tolist() != list(range(25))
    # a mask that reaches the fallback density becomes dense
    assert oracle.patch_diff_dense_fallback(np.arange(7), 25, 0.25).tolist() == list(range(25))


def test_oracle_bucket_preserves_changed_tokens():
    # crates/bevy_jepa/src/tests.rs:1917-1928
    changed = np.arange(103)
    bucketed = oracle.bucket_sparse_mask(changed, 32 * 32, 256)
    assert len(bucketed) == 256
    assert set(changed.tolist()) <= set(bucketed.tolist())
    assert bucketed.tolist() != list(range(256)) or len(bucketed) != 1024


def _frames(seed, S, H, W, shift, changed_frac):
    rng = np.random.default_rng(seed)
    prev = rng.integers(0, 256, size=(S, H, W, 4), dtype=np.uint8)
    cur = prev.astype(np.int32) + shift
    P = 16
    for s in range(S):
        for r in range(H // P):
            for c in range(W // P):
                if rng.uniform() < changed_frac:
                    cur[s, r * P:(r + 1) * P, c * P:(c + 1) * P, :3] = rng.integers(0, 256, size=(P, P, 3))
    return prev, np.clip(cur, 0, 255).astype(np.uint8)


@pytest.mark.gpu
@pytest.mark.parametrize("shift,changed", [(0, 0.1), (25, 0.05), (-40, 0.0), (12, 0.5), (2, 0.3)])
def test_device_rgba_scores_match_oracle(cuda_device, shift, changed):
    import torch

    import burn_jepa_b200 as bj

    S, H, W, P = 3, 128, 192, 16
    prev, cur = _frames(1000 + shift, S, H, W, shift, changed)
    grid = bj.TokenGridShape(1, H // P, W // P)
    dp, dc = torch.from_numpy(prev).to(cuda_device), torch.from_numpy(cur).to(cuda_device)
    got, stats = bj.patch_diff_scores_from_rgba(dp, dc, P, grid, stats=True)
    # without statistics a stream the frame means rule out from compensating takes the
    # unshifted-only pass: the same scores, bit for bit
    plain = bj.patch_diff_scores_from_rgba(dp, dc, P, grid)
    assert torch.equal(plain, got)
    got = got.cpu().numpy()
    for s in range(S):
        ref, st = oracle.patch_diff_scores_from_rgba(prev[s], cur[s], W, P, oracle.TokenGridShape(1, H // P, W // P))
        assert stats[s].compensate_global_lighting == st.compensate_global_lighting
        d = (cur[s, :, :, :3].astype(np.float32) / np.float32(255) - prev[s, :, :, :3].astype(np.float32) / np.float32(255))
        exact = d.astype(np.float64).reshape(-1, 3).mean(axis=0)
        np.testing.assert_allclose(list(stats[s].channel_delta), exact, rtol=0, atol=1e-6)
        bound = H * W * 2.0 ** -24 * float(np.abs(d).mean()) + 1e-7  # worst case of the f32 sequential sum
        np.testing.assert_allclose(list(stats[s].channel_delta), list(st.channel_delta), rtol=0, atol=bound)
        np.testing.assert_allclose(got[s], ref, rtol=0, atol=bound + 1e-5)


@pytest.mark.gpu
def test_device_rgba_uniform_lighting_and_errors(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    prev = torch.full((64, 64, 4), 80, dtype=torch.uint8, device=cuda_device)
    cur = torch.full((64, 64, 4), 110, dtype=torch.uint8, device=cuda_device)
    scores, stats = bj.patch_diff_scores_from_rgba(prev, cur, 16, bj.TokenGridShape(1, 4, 4), stats=True)
    assert bool((scores < float(DEFAULT_PATCH_DIFF_THRESHOLD)).all())
    assert stats[0].compensate_global_lighting == 1
    with pytest.raises(bj.BjfError, match="single-frame grid"):
        bj.patch_diff_scores_from_rgba(prev, cur, 16, bj.TokenGridShape(2, 4, 4))
    with pytest.raises(bj.BjfError, match="width must match the token grid"):
        bj.patch_diff_scores_from_rgba(prev, cur, 16, bj.TokenGridShape(1, 4, 3))
    with pytest.raises(bj.BjfError, match="smaller than the token grid"):
        bj.patch_diff_scores_from_rgba(prev, cur, 16, bj.TokenGridShape(1, 5, 4))


# ---------------------------------------------------------------------------
# Mask policy after the selection: dense fallback -> dilation -> encode buckets
# ---------------------------------------------------------------------------

def test_oracle_bucket_widths_match_reference_prewarm_tests():
    # src/viewer.rs:1342-1376: the default densities (0.10, 0.25, 0.50) and the legacy step
    assert oracle.sparse_mask_bucket_widths(32 * 32, 256, (0.10, 0.25, 0.50)) == [103, 256, 512, 1024]
    assert oracle.sparse_mask_bucket_widths(64 * 64, 256, (0.10, 0.25, 0.50)) == [410, 1024, 2048, 4096]
    # the legacy step gives 768 too; the reference's prewarm list [256, 512, 1024] drops it
    # because 768 tokens reach the 0.75 dense fallback and finalize to the dense mask
    assert oracle.sparse_mask_bucket_widths(32 * 32, 256, ()) == [256, 512, 768, 1024]
    assert len(oracle.patch_diff_dense_fallback(np.arange(768), 1024, 0.75)) == 1024
    assert oracle.sparse_mask_bucket_widths(255, 256, (0.1,)) == []


def test_oracle_bucketed_encode_widens_context():
    # src/viewer.rs:1322-1340: one changed token -> write mask exact, encode mask 103 tokens
    grid = oracle.TokenGridShape(1, 32, 32)
    changed = [15 * 32 + 16]
    write, enc = oracle.viewer_patch_diff_masks(changed, grid, 0.75, 0)
    assert write.tolist() == changed
    assert len(enc) == 103 and changed[0] in enc.tolist()
    # src/viewer.rs:1377-1389: 120 evenly spaced tokens -> the 256 bucket
    mask = np.array([(i * 1023 + 60) // 120 for i in range(120)])
    write, enc = oracle.viewer_patch_diff_masks(mask, grid, 0.75, 0)
    assert write.tolist() == mask.tolist() and len(enc) == 256 and set(mask.tolist()) <= set(enc.tolist())


def test_oracle_masks_from_scores_dense_cutoff_before_dilation():
    # src/viewer.rs:1456-1484 through patch_diff_masks_from_scores
    grid = oracle.TokenGridShape(1, 5, 5)
    scores = np.zeros(25, np.float32)
    scores[12] = 0.5
    cfg = oracle.PatchDiffConfig.adaptive_threshold(0.10, 0, 25, 1).with_dilation(1)
    write, enc = oracle.viewer_patch_diff_masks_from_scores(scores, grid, cfg, 0.25, bucketed=False)
    assert len(write) == 9 and 12 in write.tolist() and enc.tolist() == write.tolist()


def _direct_masks(seed, S, n, densities):
    rng = np.random.default_rng(seed)
    idx = np.zeros((S, n), np.int32)
    cnt = np.zeros(S, np.int32)
    for s in range(S):
        d = densities[s % len(densities)]
        m = int(round(n * d))
        sel = np.sort(rng.choice(n, size=m, replace=False)) if m else np.zeros(0, np.int64)
        idx[s, :m] = sel
        cnt[s] = m
    return idx, cnt


_VIEWER_POLICIES = {
    # name: (grid, dense_fallback_density, dilation, bucketed, bucket_tokens, densities)
    "default": ((1, 32, 32), 0.75, 1, True, 256, (0.10, 0.25, 0.50)),
    "exact": ((1, 32, 32), 0.75, 1, False, 256, (0.10, 0.25, 0.50)),
    "legacy_step": ((1, 32, 48), 0.75, 2, True, 100, ()),
    "legacy_single_width": ((1, 16, 16), 0.75, 0, True, 1, ()),
    "no_fallback": ((1, 40, 40), 1.0, 3, True, 256, (0.05, 0.3, 0.9, 0.3)),
    "fallback_low": ((1, 24, 24), 0.1, 1, True, 256, (0.2, 0.6)),
    "nan_fallback": ((1, 16, 16), float("nan"), 1, True, 256, (0.1, float("nan"), -1.0, 2.0)),
    "small_grid": ((1, 8, 8), 0.75, 1, True, 256, (0.1, 0.25, 0.5)),
    "depth_two": ((2, 20, 20), 0.75, 2, True, 256, (0.1, 0.25, 0.5)),
    "large_grid": ((1, 128, 256), 0.75, 1, True, 256, (0.1, 0.25, 0.5)),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(_VIEWER_POLICIES))
def test_device_viewer_masks_match_oracle(cuda_device, name):
    import torch

    import burn_jepa_b200 as bj

    g, fb, dil, bucketed, bt, dens = _VIEWER_POLICIES[name]
    n = g[0] * g[1] * g[2]
    dens_list = (0.0, 0.002, 0.01, 0.05, 0.09, 0.11, 0.2, 0.3, 0.6, 0.8, 1.0)
    S = len(dens_list)
    idx, cnt = _direct_masks(7 + n, S, n, dens_list)
    policy = bj.ViewerMaskPolicy.new(fb, dil, bucketed, bt, dens)
    d_idx, d_cnt = torch.from_numpy(idx).to(cuda_device), torch.from_numpy(cnt).to(cuda_device)
    wi, wc, ei, ec = (t.cpu().numpy() for t in bj.viewer_patch_diff_masks(d_idx, d_cnt, bj.TokenGridShape(*g), policy))
    og = oracle.TokenGridShape(*g)
    for s in range(S):
        w, e = oracle.viewer_patch_diff_masks(idx[s, :cnt[s]], og, fb, dil, bucketed, bt, dens)
        assert wc[s] == len(w) and wi[s, :wc[s]].tolist() == w.tolist(), (name, s)
        assert ec[s] == len(e) and ei[s, :ec[s]].tolist() == e.tolist(), (name, s)
    # the direct buffers may be the write buffers
    out = (d_idx, d_cnt, torch.empty_like(d_idx), torch.empty_like(d_cnt))
    bj.viewer_patch_diff_masks(d_idx, d_cnt, bj.TokenGridShape(*g), policy, out=out)
    assert np.array_equal(d_cnt.cpu().numpy(), wc) and np.array_equal(out[3].cpu().numpy(), ec)
    for s in range(S):
        assert d_idx[s, :wc[s]].cpu().numpy().tolist() == wi[s, :wc[s]].tolist()
        assert out[2][s, :ec[s]].cpu().numpy().tolist() == ei[s, :ec[s]].tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("threshold,dilation,fallback", [(0.10, 1, 0.25), (0.6, 2, 0.75), (0.95, 1, 0.75), (0.3, 0, 0.5)])
def test_device_viewer_masks_from_scores_match_oracle(cuda_device, threshold, dilation, fallback):
    import torch

    import burn_jepa_b200 as bj

    g = (1, 32, 32)
    n = g[0] * g[1] * g[2]
    S = 6
    rng = np.random.default_rng(int(threshold * 100) + dilation)
    scores = (rng.uniform(0, 1, size=(S, n)) ** np.linspace(1, 12, S)[:, None]).astype(np.float32)
    cfg = bj.PatchDiffConfig.adaptive_threshold(threshold, 4, n, 1).with_dilation(dilation)
    policy = bj.ViewerMaskPolicy.new(fallback, 0)  # the config's dilation applies
    wi, wc, ei, ec = (t.cpu().numpy() for t in bj.viewer_patch_diff_masks_from_scores(
        torch.from_numpy(scores).to(cuda_device), bj.TokenGridShape(*g), cfg, policy))
    ocfg = oracle.PatchDiffConfig.adaptive_threshold(threshold, 4, n, 1).with_dilation(dilation)
    for s in range(S):
        w, e = oracle.viewer_patch_diff_masks_from_scores(scores[s], oracle.TokenGridShape(*g), ocfg, fallback)
        assert wi[s, :wc[s]].tolist() == w.tolist(), s
        assert ei[s, :ec[s]].tolist() == e.tolist(), s


@pytest.mark.gpu
def test_device_viewer_masks_errors(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    idx = torch.zeros((1, 64), dtype=torch.int32, device=cuda_device)
    cnt = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    bad = bj.ViewerMaskPolicy.new()
    bad.bucket_density_count = 33
    with pytest.raises(bj.BjfError, match="bucket densities"):
        bj.viewer_patch_diff_masks(idx, cnt, bj.TokenGridShape(1, 8, 8), bad)
    with pytest.raises(bj.BjfError, match="32768 tokens"):
        big = torch.zeros((1, 2 * 128 * 256), dtype=torch.int32, device=cuda_device)
        bj.viewer_patch_diff_masks(big, cnt, bj.TokenGridShape(2, 128, 256), bj.ViewerMaskPolicy.new())
    neg = bj.ViewerMaskPolicy.new(dilation=-1)
    with pytest.raises(bj.BjfError, match="non-negative"):
        bj.viewer_patch_diff_masks(idx, cnt, bj.TokenGridShape(1, 8, 8), neg)


# ---------------------------------------------------------------------------
# The RGBA mask node: dense fast paths, then scores -> masks
# ---------------------------------------------------------------------------

def _white_block_frames(grid_h, grid_w, P, rows, cols):
    # src/viewer.rs:1579-1593 (fill_rgba_patch): black opaque frame, then white patches
    prev = np.zeros((grid_h * P, grid_w * P, 4), np.uint8)
    prev[..., 3] = 255
    cur = prev.copy()
    for r in rows:
        for c in cols:
            cur[r * P:(r + 1) * P, c * P:(c + 1) * P, :] = 255
    return prev, cur


def test_oracle_sampled_dense_fast_path_uses_direct_density():
    # src/viewer.rs:1486-1527: 16 of 64 patches change -> below the 0.60 fallback, both dilations
    grid = oracle.TokenGridShape(1, 8, 8)
    prev, cur = _white_block_frames(8, 8, 16, range(4), range(4))
    cfg = oracle.PatchDiffConfig.adaptive_threshold(0.10, 1, 64, 64).with_dilation(1)
    assert not oracle.patch_diff_sampled_dense_fast_path_from_rgba(prev, cur, 128, 16, grid, cfg, 0.60)
    assert not oracle.patch_diff_sampled_dense_fast_path_from_rgba(prev, cur, 128, 16, grid, cfg.with_dilation(0), 0.60)
    # 48 of 64 change -> dense; a fallback density of 1.0 never takes the path
    prev, cur = _white_block_frames(8, 8, 16, range(6), range(8))
    assert oracle.patch_diff_sampled_dense_fast_path_from_rgba(prev, cur, 128, 16, grid, cfg, 0.60)
    assert not oracle.patch_diff_sampled_dense_fast_path_from_rgba(prev, cur, 128, 16, grid, cfg, 1.0)
    # a capped context never takes it
    capped = oracle.PatchDiffConfig.adaptive_threshold(0.10, 1, 32, 64)
    assert not oracle.patch_diff_sampled_dense_fast_path_from_rgba(prev, cur, 128, 16, grid, capped, 0.60)
    w, e = oracle.viewer_patch_diff_masks_from_rgba(prev, cur, 128, 16, grid, cfg, 0.60)
    assert w.tolist() == list(range(64)) and e.tolist() == list(range(64))


_RGBA_NODE_CASES = {
    # name: (changed fractions per stream, threshold, dilation, context tokens, fallback density)
    "sparse": ((0.02, 0.05, 0.1), 0.1, 1, 256, 0.75),
    "fast_path": ((0.7, 0.95, 0.3), 0.1, 1, 256, 0.6),
    "capped": ((0.7, 0.2, 0.05), 0.1, 1, 64, 0.6),
    "threshold_zero": ((0.05, 0.0), 0.0, 1, 256, 0.75),
    "no_dilation_exact": ((0.1, 0.4), 0.1, 0, 256, 0.75),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(_RGBA_NODE_CASES))
def test_device_rgba_mask_node_matches_oracle(cuda_device, name):
    import torch

    import burn_jepa_b200 as bj

    fracs, thr, dil, ctx, fb = _RGBA_NODE_CASES[name]
    S, P, gh, gw = len(fracs), 16, 16, 16
    H, W = gh * P, gw * P
    frames = [_frames(300 + 7 * i, 1, H, W, 0, f) for i, f in enumerate(fracs)]
    prev = np.concatenate([f[0] for f in frames])
    cur = np.concatenate([f[1] for f in frames])
    bucketed = name != "no_dilation_exact"
    cfg = bj.PatchDiffConfig.adaptive_threshold(thr, 1, ctx, 1).with_dilation(dil)
    policy = bj.ViewerMaskPolicy.new(fb, 0, bucketed)
    (wi, wc, ei, ec), stats = bj.viewer_patch_diff_masks_from_rgba(
        torch.from_numpy(prev).to(cuda_device), torch.from_numpy(cur).to(cuda_device), P, (1, gh, gw), cfg, policy,
        stats=True)
    wi, wc, ei, ec = (t.cpu().numpy() for t in (wi, wc, ei, ec))
    ocfg = oracle.PatchDiffConfig.adaptive_threshold(thr, 1, ctx, 1).with_dilation(dil)
    og = oracle.TokenGridShape(1, gh, gw)
    for s in range(S):
        w, e = oracle.viewer_patch_diff_masks_from_rgba(prev[s], cur[s], W, P, og, ocfg, fb, bucketed)
        assert wi[s, :wc[s]].tolist() == w.tolist(), (name, s)
        assert ei[s, :ec[s]].tolist() == e.tolist(), (name, s)
        _, st = oracle.patch_diff_scores_from_rgba(prev[s], cur[s], W, P, og)
        assert stats[s].compensate_global_lighting == st.compensate_global_lighting


@pytest.mark.gpu
def test_device_rgba_mask_node_errors(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    prev = torch.zeros((64, 64, 4), dtype=torch.uint8, device=cuda_device)
    cfg = bj.PatchDiffConfig.adaptive_threshold(0.1, 1, 16, 1)
    pol = bj.ViewerMaskPolicy.new()
    with pytest.raises(bj.BjfError, match="single-frame token grid"):
        bj.viewer_patch_diff_masks_from_rgba(prev, prev, 16, (2, 4, 4), cfg, pol)
    with pytest.raises(bj.BjfError, match="frame size must match"):
        bj.viewer_patch_diff_masks_from_rgba(prev, prev, 16, (1, 4, 3), cfg, pol)


# ---------------------------------------------------------------------------
# Refresh state (src/viewer.rs:272-528), the oracle against the reference's own tests
# ---------------------------------------------------------------------------

def _refresh_case(context_density, refresh):
    grid = oracle.TokenGridShape(1, 4, 4)
    cfg = oracle.patch_diff_sparsity_config(context_density, 0.0, 0.10, 0, grid)
    return grid, cfg, dict(refresh)


def test_oracle_subthreshold_refresh_accumulates_slow_motion():
    # src/viewer.rs:1528-1575
    grid, cfg, refresh = _refresh_case(0.25, dict(enabled=True, subthreshold_enabled=True, subthreshold_decay=1.0,
                                                  subthreshold_trigger=1.0, subthreshold_max_density=0.25,
                                                  max_extra_density=0.25))
    slow = 2 * 4 + 1
    scores = np.zeros(16, np.float32)
    scores[0] = 0.09
    scores[slow] = 0.04
    st = oracle.PatchDiffRefreshState()
    assert slow not in st.masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)[0].tolist()
    assert slow not in st.masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)[0].tolist()
    assert slow in st.masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)[0].tolist()
    assert st.residual[slow] == 0.0 and st.age[slow] == 0


def test_oracle_subthreshold_refresh_fills_only_unused_budget():
    # src/viewer.rs:1595-1632
    grid, cfg, refresh = _refresh_case(2.0 / 16.0, dict(enabled=True, subthreshold_enabled=True,
                                                        subthreshold_decay=1.0, subthreshold_trigger=0.5,
                                                        subthreshold_max_density=1.0, max_extra_density=1.0))
    scores = np.full(16, 0.06, np.float32)
    scores[0] = 0.09
    w, _ = oracle.PatchDiffRefreshState().masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)
    assert len(w) == 2


def test_oracle_age_priority_refresh_selects_stale_tokens():
    # src/viewer.rs:1634-1672
    grid, cfg, refresh = _refresh_case(0.5, dict(enabled=True, age_refresh_enabled=True,
                                                 age_refresh_interval_frames=2, age_refresh_max_density=0.25,
                                                 max_extra_density=0.25))
    scores = np.zeros(16, np.float32)
    scores[0] = 0.09
    st = oracle.PatchDiffRefreshState()
    first, _ = st.masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)
    second, _ = st.masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)
    assert len(first) == 1 and len(second) > len(first)


def test_oracle_blue_noise_refresh_is_deterministic():
    # src/viewer.rs:1674-1703
    grid, cfg, refresh = _refresh_case(0.5, dict(enabled=True, blue_noise_enabled=True,
                                                 blue_noise_refresh_density=0.25, max_extra_density=0.25,
                                                 blue_noise_seed=7))
    scores = np.zeros(16, np.float32)
    a, _ = oracle.PatchDiffRefreshState().masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)
    b, _ = oracle.PatchDiffRefreshState().masks_from_scores(scores, grid, cfg, 1.0, refresh, bucketed=False)
    assert a.tolist() == b.tolist() and len(a) > 0
    assert oracle.density_tokens(16, 0.25, "floor", 0.0) == 4
    assert oracle.density_tokens(1000, 0.1234, "ceil", 0.0) == 124
