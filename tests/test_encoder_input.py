"""The encoder-input form of the sparse patchify (src/model.rs:690-703): patch embed + bias,
then the token's 3-D sin-cos position embedding (src/positional.rs:42-87), then the
modality embedding, fused into the gather-GEMM epilogue.

Bars: f32 inputs within 1e-4, f16/bf16 within 1e-2 normwise max relative error of the
oracle (which adds the same table in the same order)."""
import numpy as np
import pytest

import oracle
from burn_jepa_b200 import workloads
from helpers import known_answers, max_rel_err

KA = known_answers()


def test_oracle_sparse_positional_encoding_golden():
    c = KA["sparse_positional_encoding"]
    v = oracle.sparse_3d_sincos_pos_embed(c["embed_dim"], oracle.TokenGridShape(*c["grid"]), c["indices"]).ravel()
    assert v.size == c["len"]
    for i, want in c["values_at"].items():
        assert v[int(i)] == want


def test_oracle_encoder_input_adds_table_then_modality():
    cfg = oracle.PatchifyConfig(3, 32, 4, 32, 32, 2, 16, 16)
    x = workloads.splitmix_uniform(1, (1, 3, 4, 32, 32))
    w = workloads.splitmix_normal(2, (32, 3, 2, 16, 16), 0.02)
    b = workloads.splitmix_normal(3, (32,), 0.02)
    grid = oracle.TokenGridShape(2, 2, 2)
    coords = oracle.sparse_patchify_plan_coords(np.array([0, 3, 7]), grid, 1)
    table = oracle.get_3d_sincos_pos_embed(32, grid)
    mod = workloads.splitmix_normal(4, (32,), 0.02)
    plain = oracle.sparse_patchify3d_forward(cfg, x, coords, w, b)
    got = oracle.patchify_encoder_input(cfg, x, coords, w, b, table, mod)
    want = (plain + table[[0, 3, 7]]) + mod[None]
    assert np.array_equal(got, want.astype(np.float32))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,rows_kind,use_pos,use_mod", [
    ("f16", "many", True, True), ("bf16", "many", True, False), ("f16", "few", True, True),
    ("f32", "many", True, True), ("f16", "many", False, True)])
def test_device_encoder_input_matches_oracle(cuda_device, dtype, rows_kind, use_pos, use_mod):
    import torch

    import burn_jepa_b200 as bj

    dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dtype]
    B, C, T, H, W, kt, P, D = 2, 3, 4, 256, 256, 2, 16, 256
    grid = oracle.TokenGridShape(T // kt, H // P, W // P)
    n = len(grid)
    rng = np.random.default_rng(5)
    m = 300 if rows_kind == "many" else 40   # > 128 rows: CTA-pair kernel; <= 128: one-SM kernel
    rows = np.stack([np.sort(rng.choice(n, m // B, replace=False)) for _ in range(B)])
    coords = np.concatenate([oracle.sparse_patchify_plan_coords(rows[b], grid, 1) + np.array([b, 0, 0, 0], np.int32)
                             for b in range(B)])
    x = workloads.splitmix_uniform(11, (B, C, T, H, W))
    w = workloads.splitmix_normal(12, (D, C, kt, P, P), 0.02)
    bias = workloads.splitmix_normal(13, (D,), 0.02)
    table = oracle.get_3d_sincos_pos_embed(D, grid) if use_pos else None
    mod = workloads.splitmix_normal(14, (D,), 0.02) if use_mod else None
    xd = torch.from_numpy(x).to(cuda_device).to(dt)
    wd = torch.from_numpy(w).to(cuda_device).to(dt)
    cfg = bj.PatchifyConfig(C, D, T, H, W, kt, P, P)
    out = bj.sparse_patchify3d_forward_encoder_input(
        cfg, xd, torch.from_numpy(coords).to(cuda_device), wd, torch.from_numpy(bias).to(cuda_device),
        None if table is None else torch.from_numpy(table).to(cuda_device),
        None if mod is None else torch.from_numpy(mod).to(cuda_device), out_dtype=torch.float32).cpu().numpy()
    ref = oracle.patchify_encoder_input(oracle.PatchifyConfig(C, D, T, H, W, kt, P, P), xd.float().cpu().numpy(),
                                        coords, wd.float().cpu().numpy(), bias, table, mod)
    assert max_rel_err(out, ref) <= (1e-4 if dtype == "f32" else 1e-2)
