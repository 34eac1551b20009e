"""Split K of the CTA-pair gather-GEMM (few 256-row tiles, plain epilogue, explicit coords):
the tiles run as units over K ranges whose f32 partials a reduce launch adds in a fixed order.
Checked here: the C2 clip shape (511 rows, ViT-L/16, f16) against the oracle, zero rows for
coords outside the grid (no bias), and bit-identical results on repeated calls (the partials'
order never depends on timing)."""
import numpy as np
import pytest

import burn_jepa_b200 as bj
import oracle
from burn_jepa_b200 import workloads
from helpers import max_rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,out,with_bias", [("f16", "f16", True), ("bf16", "f32", True), ("f32", "f32", True),
                                               ("f16", "f32", False)])
def test_split_k_matches_oracle_and_repeats_bit_for_bit(cuda_device, dtype, out, with_bias):
    import torch

    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
    C, T, H, W, kt, P, D, rows = 3, 16, 256, 256, 2, 16, 1024, 511
    grid = oracle.TokenGridShape(T // kt, H // P, W // P)
    rng = np.random.default_rng(77)
    coords = np.stack([np.zeros(rows, np.int64), rng.integers(0, grid.depth, rows),
                       rng.integers(0, grid.height, rows), rng.integers(0, grid.width, rows)], 1).astype(np.int32)
    coords[::50, 3] = grid.width + 1  # outside the grid: a zero row
    x = workloads.splitmix_normal(78, (1, C, T, H, W), 1.0)
    w = workloads.splitmix_normal(79, (D, C, kt, P, P), 0.02)
    b = workloads.splitmix_normal(80, (D,), 0.5) if with_bias else np.zeros(D, np.float32)
    xd = torch.from_numpy(x).to(cuda_device, dt[dtype])
    wd = torch.from_numpy(w).to(cuda_device, dt[dtype])
    cd = torch.from_numpy(coords).to(cuda_device)
    bd = torch.from_numpy(b).to(cuda_device) if with_bias else None
    cfg = bj.PatchifyConfig(C, D, T, H, W, kt, P, P)
    first = bj.sparse_patchify3d_forward(cfg, xd, cd, wd, bd, out_dtype=dt[out])
    again = bj.sparse_patchify3d_forward(cfg, xd, cd, wd, bd, out_dtype=dt[out])
    torch.cuda.synchronize()
    assert not bj.device_error_check()
    assert torch.equal(first, again)
    got = first.float().cpu().numpy()
    assert np.all(got[::50] == 0.0)
    ref = oracle.sparse_patchify3d_forward(oracle.PatchifyConfig(C, D, T, H, W, kt, P, P), xd.float().cpu().numpy(),
                                           coords, wd.float().cpu().numpy(), b)
    assert max_rel_err(got, ref) <= (1e-4 if dtype == "f32" else 1e-2)
