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
@pytest.mark.parametrize("shift,changed", [(0, 0.1), (25, 0.05), (-40, 0.0), (12, 0.5)])
def test_device_rgba_scores_match_oracle(cuda_device, shift, changed):
    import torch

    import burn_jepa_b200 as bj

    S, H, W, P = 3, 128, 192, 16
    prev, cur = _frames(1000 + shift, S, H, W, shift, changed)
    grid = bj.TokenGridShape(1, H // P, W // P)
    got, stats = bj.patch_diff_scores_from_rgba(torch.from_numpy(prev).to(cuda_device),
                                                torch.from_numpy(cur).to(cuda_device), P, grid, stats=True)
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
