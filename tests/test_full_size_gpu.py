"""Parity at the benchmark workloads' full sizes.

- Live streams: 32 streams x [3, 2, 1024, 1024] f16, D = 1024, f16 caches [4096, 1024] (the
  fused step the bench times).  The threshold sits in a gap of every stream's oracle scores,
  so the masks must equal the oracle's exactly: observed = 1 exactly on the oracle's tokens,
  age stays 0, every cache row outside the mask is bit-for-bit untouched, the step's counts
  are the mask sizes, and EVERY written row (about 13 000, so every 256-row pair tile, every
  stream boundary inside a tile and the last partial tile) equals the oracle's patch embed
  within the half tolerance (normwise 1e-2 per stream).
- ViT-g batch: 32 clips [3, 16, 512, 512] bf16, one multiblock mask of 4096 of the 8192
  tokens shared by the batch (131 072 rows), D = 1408 (six 240-column tiles): every row of
  four whole clips (16 384 rows, every column tile and its tail) against the oracle (normwise
  1e-2), and doubling the weight and bias doubles every one of the 131 072 x 1408 outputs
  exactly (products and f32 sums scale by two without rounding).
- ViT-L clip (config C2): one clip [1, 3, 16, 256, 256] f16, grid 8 x 16 x 16 = 2048 tokens,
  D = 1024, a gap threshold keeping about 25 %: through the fused step (masks exact, every
  written row within 1e-2) and through bjf_sparse_patchify3d_forward on the oracle's plan
  (every row within 1e-2).  This is the small-M case: about 512 rows, two pair tiles.
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

    cfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    for s in range(S):
        toks = np.asarray(masks[s], dtype=np.int64)
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
    for clip in (0, 7, 19, 31):
        sel = np.arange(len(mask)) + clip * len(mask)
        c = ref_coords[sel].copy()
        c[:, 0] = 0
        ref = oracle.sparse_patchify3d_forward(ocfg, video[clip:clip + 1].float().cpu().numpy(), c, w_exact, b)
        got = out[torch.from_numpy(sel).to(cuda_device)].float().cpu().numpy()
        assert max_rel_err(got, ref) <= TOL_HALF, clip


def test_vitl_clip_full_size_c2(cuda_device):
    import torch

    S, C, T, H, W, KT, P, D = 1, 3, 16, 256, 256, 2, 16, 1024
    grid = oracle.TokenGridShape(T // KT, H // P, W // P)
    n = len(grid)
    assert n == 2048
    video = workloads.rect_perturbation_clips(701, S, C, T, H, W, 0.25)
    vd = torch.from_numpy(video).to(cuda_device, torch.float16)
    v_exact = vd.float().cpu().numpy()
    w = workloads.splitmix_normal(702, (D, C, KT, P, P), 0.02)
    b = workloads.splitmix_normal(703, (D,), 0.02)
    wd = torch.from_numpy(w).to(cuda_device, torch.float16)
    bd = torch.from_numpy(b).to(cuda_device)
    w_exact = wd.float().cpu().numpy()

    scores = oracle.patch_diff_token_scores(v_exact, KT, P)
    thr = workloads.choose_threshold(scores, 0.25)
    ocfg = oracle.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
    mask = oracle.patch_diff_context_mask_from_scores(scores, grid, ocfg)
    assert 0.15 * n < len(mask) < 0.35 * n
    coords = oracle.sparse_patchify_plan_coords(mask, grid, 1)
    cfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    ref = oracle.sparse_patchify3d_forward(cfg, v_exact, coords, w_exact, b)

    # the fused step (mask -> plan -> patchify -> cache write)
    caches = torch.from_numpy(workloads.splitmix_normal(704, (S, n, D), 1.0)).to(cuda_device, torch.float16)
    cache0 = caches.clone()
    observed = torch.zeros((S, n), device=cuda_device)
    age = torch.zeros((S, n), device=cuda_device)
    fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1), torch.float16,
                     torch.float16, cuda_device)
    counts = fe.step(vd, wd, bd, caches, observed, age, age_observed=False).cpu().numpy()
    torch.cuda.synchronize()
    assert not bj.device_error_check()
    want = np.zeros((S, n), np.float32)
    want[0, mask] = 1.0
    assert counts.tolist() == [len(mask)]
    assert np.array_equal(observed.cpu().numpy(), want)
    changed = (caches != cache0).any(dim=2).cpu().numpy()
    assert np.array_equal(changed, want > 0)
    got = caches[0, torch.from_numpy(np.asarray(mask, np.int64)).to(cuda_device)].float().cpu().numpy()
    assert max_rel_err(got, ref) <= TOL_HALF

    # the standalone patchify API on the oracle's plan, f16 and f32 outputs
    cd = torch.from_numpy(coords.astype(np.int32)).to(cuda_device)
    pcfg = bj.PatchifyConfig(C, D, T, H, W, KT, P, P)
    for out_dtype in (torch.float32, torch.float16):
        out = bj.sparse_patchify3d_forward(pcfg, vd, cd, wd, bd, out_dtype=out_dtype)
        torch.cuda.synchronize()
        assert not bj.device_error_check()
        assert max_rel_err(out.float().cpu().numpy(), ref) <= TOL_HALF, out_dtype
