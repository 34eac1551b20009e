"""The seeded synthetic inputs the benchmark and the full-size tests share (CPU)."""
import numpy as np

from burn_jepa_b200 import workloads


def test_multiblock_mask_covers_the_budget_with_whole_temporal_columns():
    depth, height, width, keep = 8, 32, 32, 4096
    a = workloads.multiblock_mask(601, depth, height, width, keep)
    b = workloads.multiblock_mask(601, depth, height, width, keep)
    assert np.array_equal(a, b)  # seeded
    assert len(a) == keep and np.all(np.diff(a) > 0)  # ascending, unique
    assert a.min() >= 0 and a.max() < depth * height * width
    # the blocks span the whole temporal extent: every covered spatial token of frame 0 is
    # covered in the next frames too, except where the budget cuts the last frames
    per_frame = height * width
    frame0 = set((a[a < per_frame]).tolist())
    frame1 = set((a[(a >= per_frame) & (a < 2 * per_frame)] - per_frame).tolist())
    assert frame0 and frame0 == frame1
    assert workloads.multiblock_mask(602, depth, height, width, keep).tolist() != a.tolist()


def test_choose_threshold_sits_in_a_gap():
    scores = np.array([0.0] * 90 + [0.5, 0.51, 0.52, 0.9, 1.0] + [2.0] * 5, np.float32)
    thr = workloads.choose_threshold(scores, 0.10, 1e-3)
    kept = int((scores >= thr).sum())
    assert 0 < thr and kept in (9, 10, 11)
    # no score sits within the relative gap around the threshold
    assert np.all(np.abs(scores[scores > 0] - thr) > 1e-3 * thr)
