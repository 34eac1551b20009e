"""Parity at the benchmark workloads' full sizes, through properties that do not need the
oracle to process the whole workload.

- Live streams: 32 streams x [3, 2, 1024, 1024] f16, D = 1024, f16 caches [4096, 1024] (the
  fused step the bench times).  The threshold sits in a gap of every stream's oracle scores,
  so the masks must equal the oracle's exactly: observed = 1 exactly on the oracle's tokens,
  age stays 0, every cache row outside the mask is bit-for-bit untouched, the step's counts
  are the mask sizes, and sampled written rows equal the oracle's patch embed within the half
  tolerance (normwise 1e-2).
- ViT-g batch: 32 clips [3, 16, 512, 512] bf16, one multiblock mask of 4096 of the 8192
  tokens shared by the batch (131 072 rows), D = 1408 (BN = 176 tiles): sampled rows from four
  clips against the oracle (normwise 1e-2), and doubling the weight and bias doubles every one
  of the 131 072 x 1408 outputs exactly (products and f32 sums scale by two without rounding).
"""
import numpy as np
import pytest

import burn_jepa_b200 as bj
import oracle
from burn_jepa_b200 import workloads
from helpers import max_rel_err

pytestmark = pytest.mark.gpu

TOL_HALF = 1e-2


def test_live_streams_full_size_step(cuda_device):
    import torch

    S, C, T, H, W, KT, P, D = 32, 3, 2, 1024, 1024, 2, 16, 1024
    grid = oracle.TokenGridShape(T // KT, H // P, W // P)
    n = len(grid)
    vd = workloads.rect_perturbation_clips_torch(501, S, C, T, H, W, 0.1, cuda_device, torch.float16)
    w = workloads.splitmix_normal(502, (D, C, KT, P, P), 0.02)
    b = workloads.splitmix_normal(503, (D,), 0.02)
    wd = torch.from_numpy(w).to(cuda_device, torch.float16)
    bd = torch.from_numpy(b).to(cuda_device)
    w_exact = wd.float().cpu().numpy()

    scores = np.stack([oracle.patch_diff_token_scores(vd[s:s + 1].float().cpu().numpy(), KT, P) for s in range(S)])
    thr = workloads.choose_threshold(scores, 0.1)
    ocfg = oracle.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
    masks = [oracle.patch_diff_context_mask_from_scores(scores[s], grid, ocfg) for s in range(S)]

    caches = torch.from_numpy(workloads.splitmix_normal(504, (S, n, D), 1.0)).to(cuda_device, torch.float16)
    cache0 = caches.clone()
    observed = torch.zeros((S, n), device=cuda_device)
    age = torch.zeros((S, n), device=cuda_device)
    fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1), torch.float16,
                     torch.float16, cuda_device)
    counts = fe.step(vd, wd, bd, caches, observed, age, age_observed=False).cpu().numpy()
    torch.cuda.synchronize()
    assert not bj.device_error_check()

    want = np.zeros((S, n), np.float32)
    for s in range(S):
        want[s, masks[s]] = 1.0
    assert counts.tolist() == [len(m) for m in masks]
    assert np.array_equal(observed.cpu().numpy(), want)
    assert not bool(age.any())
    changed = (caches != cache0).any(dim=2).cpu().numpy()
    assert np.array_equal(changed, want > 0)

    rng = np.random.default_rng(505)
    cfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    for s in (0, 9, 22, 31):
        toks = np.sort(rng.choice(masks[s], size=min(32, len(masks[s])), replace=False))
        coords = np.array([[0, *oracle.token_index_to_coords(int(t), grid)] for t in toks], np.int32)
        ref = oracle.sparse_patchify3d_forward(cfg, vd[s:s + 1].float().cpu().numpy(), coords, w_exact, b)
        got = caches[s, torch.from_numpy(toks).to(cuda_device)].float().cpu().numpy()
        assert max_rel_err(got, ref) <= TOL_HALF, s


def test_vitg_batch_full_size_patchify(cuda_device):
    import torch

    B, C, T, H, W, KT, P, D = 32, 3, 16, 512, 512, 2, 16, 1408
    grid = oracle.TokenGridShape(T // KT, H // P, W // P)
    mask = workloads.multiblock_mask(601, grid.depth, grid.height, grid.width, len(grid) // 2)
    assert len(mask) == 4096
    g = torch.Generator(device=cuda_device).manual_seed(602)
    video = torch.empty((B, C, T, H, W), dtype=torch.bfloat16, device=cuda_device)
    for i in range(B):
        video[i] = ((torch.rand((C, T, H, W), generator=g, device=cuda_device) - 0.45) / 0.225).to(torch.bfloat16)
    w = workloads.splitmix_normal(603, (D, C, KT, P, P), 0.02)
    b = workloads.splitmix_normal(604, (D,), 0.02)
    wd = torch.from_numpy(w).to(cuda_device, torch.bfloat16)
    bd = torch.from_numpy(b).to(cuda_device)
    coords, total = bj.sparse_patchify_plan_coords(torch.from_numpy(mask.astype(np.int32)).to(cuda_device),
                                                   (grid.depth, grid.height, grid.width), batch=B)
    rows = int(total.item())
    assert rows == B * len(mask)
    cfg = bj.PatchifyConfig(C, D, T, H, W, KT, P, P)
    out = bj.sparse_patchify3d_forward(cfg, video, coords[:rows], wd, bd)
    out2 = bj.sparse_patchify3d_forward(cfg, video, coords[:rows], wd * 2, bd * 2)
    torch.cuda.synchronize()
    assert not bj.device_error_check()
    assert bool(torch.equal(out2, out * 2))

    ref_coords = oracle.sparse_patchify_plan_coords(mask, grid, B)
    assert np.array_equal(coords[:rows].cpu().numpy(), ref_coords)
    ocfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    w_exact = wd.float().cpu().numpy()
    rng = np.random.default_rng(605)
    for clip in (0, 7, 19, 31):
        sel = np.sort(rng.choice(len(mask), size=64, replace=False)) + clip * len(mask)
        c = ref_coords[sel].copy()
        c[:, 0] = 0
        ref = oracle.sparse_patchify3d_forward(ocfg, video[clip:clip + 1].float().cpu().numpy(), c, w_exact, b)
        got = out[torch.from_numpy(sel).to(cuda_device)].cpu().numpy()
        assert max_rel_err(got, ref) <= TOL_HALF, clip
