"""Writes the golden fixtures the parity tests pin the oracle (and the CUDA path) to.

1. reference_known_answers.json -- the expected values the reference's own tests assert
   for this path, transcribed case by case with the reference file:line of each assertion.
   (The reference is Rust and cannot be built here; its test expectations are the pin.)
2. conv3d_golden.npz -- Conv3d patch-embed outputs from torch ``F.conv3d`` with stride =
   kernel, the op the reference's own cross-framework fixture uses for the patch embed
   (tests/fixtures/vjepa_tiny_parity.py:130-133).  This pins the arithmetic of the
   un-vendored burn_flex_gmm 0.21.2 kernel, which the reference's CUDA tests assert equals
   the dense Conv3d gathered at the selected tokens (tests/sparse_patchify_cuda.rs:45-82).
   Inputs are regenerated from splitmix64 seeds (bit-identical everywhere), so only the
   seeds, shapes and outputs are stored.

Run from the repo root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from burn_jepa_b200 import workloads  # noqa: E402

KNOWN_ANSWERS = {
    "positional_round_trip": {
        "source": "src/positional.rs:97-103",
        "grid": [3, 4, 5], "coords": [2, 3, 4], "index": 59,
    },
    "tiny_config_grid": {
        "source": "src/config.rs:94-128 (tiny_for_tests) and :373-378 (num_patches == 8)",
        "image_size": 32, "patch_size": 16, "num_frames": 4, "tubelet_size": 2, "in_channels": 3,
        "embed_dim": 32, "grid": [2, 2, 2], "num_patches": 8,
    },
    "context_target_masks_tiny": {
        "source": "src/tokens.rs:52-59 from_keep_ratio and :488-495 make_context_target_masks on the tiny grid",
        "dense_len": 8, "keep_ratio": 0.5, "context": [0, 1, 2, 3], "target": [4, 5, 6, 7],
    },
    "mask_sort_dedup_complement": {
        "source": "src/tokens.rs:563-568",
        "indices": [3, 1, 1], "dense_len": 5, "mask": [1, 3], "complement": [0, 2, 4],
    },
    "padded_to_multiple_bucket": {
        "source": "src/tokens.rs:570-580",
        "indices": [7, 1, 3], "dense_len": 10, "multiple": 4, "len": 4, "contains": [1, 3, 7],
        "dense_ordered": False,
    },
    "padded_to_multiple_dense": {
        "source": "src/tokens.rs:582-589",
        "indices": [0, 2, 4, 6, 8], "dense_len": 10, "multiple": 16, "mask": list(range(10)),
    },
    "target_mask_from_context": {
        "source": "src/tokens.rs:591-603",
        "context": [0, 2, 4], "dense_len": 6, "target_tokens": 2, "len": 2,
    },
    "apply_token_mask_gather": {
        "source": "src/tokens.rs:605-622",
        "tokens": list(range(12)), "shape": [1, 6, 2], "indices": [1, 4], "gathered": [2, 3, 8, 9],
    },
    "plan_coords": {
        "source": "src/sparse_patchify.rs:676-693",
        "grid": [2, 3, 4], "mask": [0, 7, 23], "batch": 2,
        "coords": [[0, 0, 0, 0], [0, 0, 1, 3], [0, 1, 2, 3], [1, 0, 0, 0], [1, 0, 1, 3], [1, 1, 2, 3]],
    },
    "patch_diff_changed_patch": {
        "source": "tests/sparse_pipeline.rs:89-136",
        "note": "video [1,3,4,32,32] zeros except frame 1, y,x in 16..32 set to 1.0 for every channel; "
                "SparseJepaPatchDiffSparsityConfig::new(threshold, 1, 2); context mask == [token (0,1,1)]; "
                "target mask has 2 tokens",
        "video_shape": [1, 3, 4, 32, 32], "changed": {"frame": 1, "y0": 16, "y1": 32, "x0": 16, "x1": 32},
        "tubelet_size": 2, "patch_size": 16, "grid": [2, 2, 2],
        "cases": [{"threshold": 0.1, "context": [3]}, {"threshold": 0.0, "context": [3]}],
        "context_tokens": 1, "target_tokens": 2, "target_len": 2,
    },
    "adaptive_changed_patches": {
        "source": "tests/highres_anyup_pca_pipeline.rs:583-604 (helper :1468-1494)",
        "video_shape": [1, 3, 2, 32, 32], "changed_patches": [[0, 1], [1, 0]], "frame": 1,
        "tubelet_size": 2, "patch_size": 16, "grid": [1, 2, 2],
        "config": {"adaptive_threshold": [0.5, 1, 4, 1]}, "context": [1, 2],
    },
    "adaptive_no_cap_above_threshold": {
        "source": "tests/highres_anyup_pca_pipeline.rs:606-624",
        "grid": [1, 2, 3], "scores": [0.9, 0.0, 0.8, 0.7, 0.0, 0.6],
        "config": {"adaptive_threshold": [0.5, 1, 1, 1]}, "context": [0, 2, 3, 5],
    },
    "adaptive_zero_threshold_keeps_all": {
        "source": "tests/highres_anyup_pca_pipeline.rs:626-636",
        "grid": [1, 2, 2], "scores": [0.0, 0.1, 0.2, 0.3],
        "config": {"adaptive_threshold": [0.0, 1, 1, 1]}, "context": [0, 1, 2, 3],
    },
    "adaptive_static_keeps_minimum": {
        "source": "tests/highres_anyup_pca_pipeline.rs:638-653",
        "video_shape": [1, 3, 2, 32, 32], "changed_patches": [], "frame": 1,
        "tubelet_size": 2, "patch_size": 16, "grid": [1, 2, 2],
        "config": {"adaptive_threshold": [0.5, 1, 4, 1]}, "context_len": 1,
    },
    "feature_memory_sequences": {
        "source": "tests/feature_memory.rs:9-65",
        "batch": 1, "grid": [1, 2, 2], "embed_dim": 2,
        "steps": [
            {"tokens": [10.0, 11.0, 20.0, 21.0], "tokens_shape": [1, 2, 2], "indices": [0, 2],
             "features": [10.0, 11.0, 0.0, 0.0, 20.0, 21.0, 0.0, 0.0], "observed": [1.0, 0.0, 1.0, 0.0],
             "age": [0.0, 0.0, 0.0, 0.0], "step": 1, "updated_tokens": 2},
            {"tokens": [30.0, 31.0], "tokens_shape": [1, 1, 2], "indices": [1],
             "features": [10.0, 11.0, 30.0, 31.0, 20.0, 21.0, 0.0, 0.0], "observed": [1.0, 1.0, 1.0, 0.0],
             "age": [1.0, 0.0, 1.0, 0.0], "step": 2},
            {"tokens": [99.0, 98.0], "tokens_shape": [1, 1, 2], "indices": [0],
             "features": [99.0, 98.0, 30.0, 31.0, 20.0, 21.0, 0.0, 0.0], "age": [0.0, 1.0, 2.0, 0.0]},
        ],
    },
    "feature_memory_write_by_index": {
        "source": "tests/feature_memory.rs:67-115",
        "batch": 1, "grid": [1, 3, 3], "embed_dim": 1,
        "steps": [
            {"tokens": [8.0, 0.0, 4.0], "tokens_shape": [1, 3, 1], "indices": [8, 0, 4],
             "features": [0.0, 0.0, 0.0, 0.0, 4.0, 0.0, 0.0, 0.0, 8.0],
             "observed": [1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0]},
            {"tokens": [2.0, 18.0], "tokens_shape": [1, 2, 1], "indices": [2, 8],
             "features": [0.0, 0.0, 2.0, 0.0, 4.0, 0.0, 0.0, 0.0, 18.0],
             "observed": [1.0, 0.0, 1.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0],
             "age": [1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 0.0]},
        ],
    },
    "feature_memory_fill_over_time": {
        "source": "tests/feature_memory.rs:117-143",
        "batch": 1, "grid": [1, 2, 2], "embed_dim": 1,
        "steps": [{"tokens": [float(t + 1)], "tokens_shape": [1, 1, 1], "indices": [t]} for t in range(4)],
        "final_observed": [1.0, 1.0, 1.0, 1.0], "final_features": [1.0, 2.0, 3.0, 4.0],
    },
    "feature_memory_masked_then_encoder_output": {
        "source": "tests/feature_memory.rs:262-298",
        "batch": 1, "grid": [1, 2, 2], "embed_dim": 2,
        "steps": [
            {"tokens": [1.0, 2.0, 7.0, 8.0], "tokens_shape": [1, 2, 2], "indices": [0, 3]},
            {"tokens": [5.0, 6.0], "tokens_shape": [1, 1, 2], "indices": [2],
             "features": [1.0, 2.0, 0.0, 0.0, 5.0, 6.0, 7.0, 8.0]},
        ],
    },
    "feature_memory_high_density_512": {
        "source": "tests/feature_memory.rs:209-260 (token_values helper :466-472)",
        "batch": 1, "grid": [1, 32, 32], "embed_dim": 4, "keep_percent": 98,
        "initial_offset": 1000.0, "update_offset": 2000.0,
        "note": "prime every token densely, then a sparse update of the first keep = ceil(1024*98/100) "
                "tokens; token_values(n, d, off)[t, c] = off + 10 t + c; unwritten rows keep their "
                "primed values; observed all 1; age[0] = age[keep-1] = 0; age[keep] = 1",
        "keep": 1004,
    },
    "feature_memory_shape_errors": {
        "source": "tests/feature_memory.rs:341-377 and src/sparse_feature_memory.rs:127-150",
        "index_shape_mismatch": {"features": [1, 4, 2], "tokens": [1, 1, 2], "indices": [1, 2],
                                 "message_contains": "index dims mismatch"},
        "sparse_len_zero": {"features": [1, 4, 2], "tokens": [1, 0, 2], "indices": [1, 0],
                            "message": "feature memory sparse assignment requires at least one token"},
        "metadata_mismatch": {"features": [1, 4, 2], "observed": [1, 3], "age": [1, 4],
                              "message_contains": "feature memory metadata dims mismatch"},
        "token_dim_mismatch": {"features": [1, 4, 2], "tokens": [1, 1, 3], "indices": [1, 1],
                               "message_contains": "feature memory token dims mismatch"},
    },
    "sparse_positional_encoding": {
        "source": "src/positional.rs:104-111",
        "embed_dim": 10, "grid": [2, 2, 2], "indices": [0, 7], "len": 20,
        "values_at": {"0": 0.0, "3": 1.0},
    },
    "feature_memory_ema": {
        "source": "tests/feature_memory.rs:145-177 (Ema { alpha: 0.25 }: first observation assigned, then blended)",
        "batch": 1, "grid": [1, 1, 2], "embed_dim": 1, "alpha": 0.25,
        "steps": [{"tokens": [8.0], "tokens_shape": [1, 1, 1], "indices": [0]},
                  {"tokens": [12.0], "tokens_shape": [1, 1, 1], "indices": [0], "features": [9.0, 0.0]}],
    },
    "feature_memory_reset_rows": {
        "source": "tests/feature_memory.rs:300-339",
        "batch": 2, "grid": [1, 1, 3], "embed_dim": 1,
        "update": {"tokens": [1.0, 2.0, 3.0, 4.0], "tokens_shape": [2, 2, 1], "indices": [0, 1, 1, 2]},
        "reset": [{"rows": [1], "features": [1.0, 2.0, 0.0, 0.0, 0.0, 0.0], "observed": [1.0, 1.0, 0.0, 0.0, 0.0, 0.0]},
                  {"rows": [0], "features": [0.0] * 6, "observed": [0.0] * 6}],
    },
}

CONV3D_CASES = [
    # VJepaConfig::tiny_for_tests patch embed, uniform[0,1) video, N(0, 0.02^2) weight, zero bias
    {"name": "tiny", "batch": 1, "C": 3, "T": 4, "H": 32, "W": 32, "kt": 2, "P": 16, "D": 32,
     "x_seed": 101, "w_seed": 102, "b_seed": None, "x_kind": "uniform"},
    # the reference CUDA test's input pattern sin(idx) * 0.01 (tests/sparse_patchify_cuda.rs:58-62)
    {"name": "cuda_test_pattern", "batch": 1, "C": 3, "T": 4, "H": 32, "W": 32, "kt": 2, "P": 16, "D": 32,
     "x_seed": None, "w_seed": 202, "b_seed": 203, "x_kind": "sin"},
    # odd geometry: batch 2, tubelet 3, patch 8, non-square grid, D not a power of two
    {"name": "odd", "batch": 2, "C": 2, "T": 6, "H": 24, "W": 40, "kt": 3, "P": 8, "D": 20,
     "x_seed": 301, "w_seed": 302, "b_seed": 303, "x_kind": "uniform"},
]


def conv3d_inputs(case):
    shape = (case["batch"], case["C"], case["T"], case["H"], case["W"])
    if case["x_kind"] == "sin":
        x = (np.sin(np.arange(int(np.prod(shape)), dtype=np.float32)) * np.float32(0.01)).astype(np.float32)
        x = x.reshape(shape)
    else:
        x = workloads.splitmix_uniform(case["x_seed"], shape)
    w = workloads.splitmix_normal(case["w_seed"], (case["D"], case["C"], case["kt"], case["P"], case["P"]), 0.02)
    b = None if case["b_seed"] is None else workloads.splitmix_normal(case["b_seed"], (case["D"],), 0.02)
    return x, w, b


def main():
    with open(os.path.join(HERE, "reference_known_answers.json"), "w") as f:
        json.dump(KNOWN_ANSWERS, f, indent=1)
    import torch
    import torch.nn.functional as F

    arrays = {}
    for case in CONV3D_CASES:
        x, w, b = conv3d_inputs(case)
        y = F.conv3d(torch.from_numpy(x).double(), torch.from_numpy(w).double(),
                     None if b is None else torch.from_numpy(b).double(),
                     stride=(case["kt"], case["P"], case["P"]))
        B, D = y.shape[0], y.shape[1]
        y = y.reshape(B, D, -1).transpose(1, 2).contiguous().float().numpy()  # [B, N, D]
        arrays[case["name"]] = y
    np.savez_compressed(os.path.join(HERE, "conv3d_golden.npz"), **arrays)
    with open(os.path.join(HERE, "conv3d_cases.json"), "w") as f:
        json.dump(CONV3D_CASES, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
