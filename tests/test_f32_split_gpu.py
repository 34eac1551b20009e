"""f32 operands on the tensor cores: the error-compensated bf16 split of the gather-GEMM.

The reference's CUDA lane is f32 (RawCudaBackend = CubeBackend<CudaRuntime, f32, i32, u8>,
src/sparse_feature_memory.rs:273-275).  Here f32 inputs and weights are split as
x = hi + lo (hi = bf16(x), lo = bf16(x - hi)) and three bf16 products per term run on the
tcgen05 tensor cores with f32 accumulation; the dropped terms are below 3 * 2^-16 |a w| per
product.  Bars: normwise max relative error 1e-4 against the oracle (the f32 bar), and per
element |got - ref| <= 2^-13 * sum_k |a_k w_k| (the split's bound with room for the f32
accumulation order).  The no-alloc step keeps f32 on the SIMT kernel (the split needs
scratch); both forms are checked against the oracle and against each other's masks.
"""
import ctypes

import numpy as np
import pytest

import burn_jepa_b200 as bj
import oracle
from burn_jepa_b200 import _abi, workloads
from helpers import max_rel_err

pytestmark = pytest.mark.gpu


def _coords(rng, B, grid, rows, invalid=0):
    c = np.stack([rng.integers(0, B, rows), rng.integers(0, grid.depth, rows), rng.integers(0, grid.height, rows),
                  rng.integers(0, grid.width, rows)], axis=1).astype(np.int32)
    if invalid:  # rows outside the grid project to the bias alone
        c[rng.choice(rows, invalid, replace=False), 2] = grid.height + 3
    return c


@pytest.mark.parametrize("B,T,H,W,D,rows,dist", [
    (2, 4, 256, 256, 1024, 2000, "normal"),    # ViT-L width, many pair tiles, a partial last tile
    (1, 16, 128, 128, 1408, 700, "uniform"),   # ViT-g width (six 256-column tiles, one half-padded)
    (3, 2, 64, 96, 256, 129, "normal"),        # one row beyond a single 128-row tile
    (1, 2, 64, 64, 96, 37, "wide"),            # the one-SM kernel; values over eight binades
])
def test_f32_patchify_on_tensor_cores_matches_oracle(cuda_device, B, T, H, W, D, rows, dist):
    import torch

    C, kt, P = 3, 2, 16
    grid = oracle.TokenGridShape(T // kt, H // P, W // P)
    rng = np.random.default_rng(rows + D)
    if dist == "uniform":
        x = workloads.splitmix_uniform(rows, (B, C, T, H, W))
    else:
        x = workloads.splitmix_normal(rows, (B, C, T, H, W), 1.0)
        if dist == "wide":
            x = (x * np.exp2(rng.integers(-4, 4, size=x.shape))).astype(np.float32)
    w = workloads.splitmix_normal(D + 7, (D, C, kt, P, P), 0.02)
    b = workloads.splitmix_normal(D + 8, (D,), 0.02)
    coords = _coords(rng, B, grid, rows, invalid=min(5, rows // 7))
    cfg = bj.PatchifyConfig(C, D, T, H, W, kt, P, P)
    t = lambda a: torch.from_numpy(a).to(cuda_device)  # noqa: E731
    out = bj.sparse_patchify3d_forward(cfg, t(x), t(coords), t(w), t(b), out_dtype=torch.float32)
    got = out.cpu().numpy()
    assert not bj.device_error_check()
    ocfg = oracle.PatchifyConfig(C, D, T, H, W, kt, P, P)
    ref = oracle.sparse_patchify3d_forward(ocfg, x, coords, w, b)
    assert max_rel_err(got, ref) <= 1e-4
    mag = oracle.sparse_patchify3d_forward(ocfg, np.abs(x), coords, np.abs(w), np.zeros(D, np.float32))
    assert np.all(np.abs(got.astype(np.float64) - ref) <= 2.0 ** -13 * mag + 1e-7)


def test_f32_encoder_input_on_tensor_cores(cuda_device):
    import torch

    B, C, T, H, W, kt, P, D = 2, 3, 4, 128, 128, 2, 16, 1024
    grid = oracle.TokenGridShape(T // kt, H // P, W // P)
    rng = np.random.default_rng(3)
    coords = _coords(rng, B, grid, 500)
    x = workloads.splitmix_normal(21, (B, C, T, H, W), 1.0)
    w = workloads.splitmix_normal(22, (D, C, kt, P, P), 0.02)
    bias = workloads.splitmix_normal(23, (D,), 0.02)
    table = oracle.get_3d_sincos_pos_embed(D, grid)
    mod = workloads.splitmix_normal(24, (D,), 0.02)
    t = lambda a: torch.from_numpy(a).to(cuda_device)  # noqa: E731
    cfg = bj.PatchifyConfig(C, D, T, H, W, kt, P, P)
    out = bj.sparse_patchify3d_forward_encoder_input(cfg, t(x), t(coords), t(w), t(bias), t(table), t(mod),
                                                     out_dtype=torch.float32).cpu().numpy()
    ref = oracle.patchify_encoder_input(oracle.PatchifyConfig(C, D, T, H, W, kt, P, P), x, coords, w, bias, table,
                                        mod)
    assert max_rel_err(out, ref) <= 1e-4


def test_f32_front_end_step_split_and_no_alloc_match_oracle(cuda_device):
    """The fused step on f32 video and weight: the workspace step (tensor cores, split) and the
    no-alloc step (SIMT) give identical masks, and each cache's written rows match the oracle."""
    import torch

    S, C, T, H, W, KT, P, D = 3, 3, 2, 256, 256, 2, 16, 512
    n = (T // KT) * (H // P) * (W // P)
    video = workloads.rect_perturbation_clips(1301, S, C, T, H, W, 0.3)
    weight = workloads.splitmix_normal(1302, (D, C, KT, P, P), 0.02)
    bias = workloads.splitmix_normal(1303, (D,), 0.02)
    cache0 = workloads.splitmix_normal(1304, (S, n, D), 1.0)
    vd = torch.from_numpy(video).to(cuda_device)
    sc = bj.patch_diff_token_scores(vd.unsqueeze(1), KT, P).cpu().numpy().ravel()
    thr = workloads.choose_threshold(sc, 0.25)
    mask = bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
    wd = torch.from_numpy(weight).to(cuda_device)
    bd = torch.from_numpy(bias).to(cuda_device)

    fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, mask, torch.float32, torch.float32, cuda_device)
    c1 = torch.from_numpy(cache0).to(cuda_device)
    o1 = torch.zeros((S, n), device=cuda_device)
    a1 = torch.zeros((S, n), device=cuda_device)
    counts1 = fe.step(vd, wd, bd, c1, o1, a1, age_observed=False).clone()
    torch.cuda.synchronize()

    desc = bj.FrontEndDesc(S, C, T, H, W, KT, P, D, _abi.DTYPE_F32, _abi.DTYPE_F32, _abi.DTYPE_F32, mask)
    c2 = torch.from_numpy(cache0).to(cuda_device)
    o2 = torch.zeros((S, n), device=cuda_device)
    a2 = torch.zeros((S, n), device=cuda_device)
    counts2 = torch.zeros((S,), dtype=torch.int32, device=cuda_device)
    p = lambda v: ctypes.c_void_p(v.data_ptr())  # noqa: E731
    rc = bj.load().bjf_front_end_step_no_alloc(ctypes.byref(desc), p(vd), p(wd), p(bd), p(c2), p(o2), p(a2), 0,
                                              p(counts2), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, bj.last_error()
    torch.cuda.synchronize()
    assert not bj.device_error_check()
    assert torch.equal(counts1, counts2) and torch.equal(o1, o2) and torch.equal(a1, a2)

    cfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    ocfg = oracle.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
    cache = cache0.copy()
    obs = np.zeros((S, n), np.float32)
    age = np.zeros((S, n), np.float32)
    counts = oracle.front_end_streams(video, cfg, ocfg, weight, bias, cache, obs, age, age_observed=False)
    assert counts1.cpu().numpy().tolist() == counts.tolist() and np.array_equal(o1.cpu().numpy(), obs)
    written = obs > 0
    assert int(written.sum()) > 0
    for got in (c1, c2):
        g = got.cpu().numpy()
        assert np.array_equal(g[~written], cache[~written])
        assert max_rel_err(g[written], cache[written]) <= 1e-4
