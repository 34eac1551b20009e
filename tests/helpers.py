"""Shared fixtures/helpers for the parity tests (test infrastructure)."""
from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def known_answers() -> dict:
    with open(os.path.join(GOLDEN, "reference_known_answers.json")) as f:
        return json.load(f)


def conv3d_cases():
    with open(os.path.join(GOLDEN, "conv3d_cases.json")) as f:
        cases = json.load(f)
    data = np.load(os.path.join(GOLDEN, "conv3d_golden.npz"))
    return [(c, data[c["name"]]) for c in cases]


def changed_patch_video(shape, frame, y0, y1, x0, x1) -> np.ndarray:
    """tests/sparse_pipeline.rs:115-124: zeros with a 1.0 square in one frame."""
    v = np.zeros(shape, dtype=np.float32)
    v[:, :, frame, y0:y1, x0:x1] = 1.0
    return v


def two_frame_changed_patches(shape, patches, patch, frame=1) -> np.ndarray:
    """tests/highres_anyup_pca_pipeline.rs:1468-1494."""
    v = np.zeros(shape, dtype=np.float32)
    for (r, c) in patches:
        v[:, :, frame, r * patch:(r + 1) * patch, c * patch:(c + 1) * patch] = 1.0
    return v


def token_values(token_count, embed_dim, offset) -> np.ndarray:
    """tests/feature_memory.rs:466-472."""
    t = np.arange(token_count, dtype=np.float32)[:, None]
    c = np.arange(embed_dim, dtype=np.float32)[None, :]
    return (offset + t * 10.0 + c).astype(np.float32)


def max_rel_err(got, ref) -> float:
    """Normwise max relative error: max|got - ref| / max|ref|."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / denom)


def conv3d_inputs(case):
    """Regenerates a conv3d golden case's inputs (splitmix64 seeds, bit-identical everywhere)."""
    import sys

    if GOLDEN not in sys.path:
        sys.path.insert(0, GOLDEN)
    from make_golden import conv3d_inputs as gen

    return gen(case)
