"""Fused front-end step (bjf_front_end_step) against the oracle's per-stream composition
(patch_diff_context_mask -> plan -> sparse patchify -> AssignLatest cache write, which the
device runs as three kernels: scores, selection, gather-GEMM with the row plan) over
several steps: masks and cache slots bit-exact, written rows within the f16 tolerance,
untouched rows unchanged, observed/age exact."""
import numpy as np
import pytest

import burn_jepa_b200 as bj
import oracle
from burn_jepa_b200 import workloads
from helpers import max_rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_timeouts(cuda_device):
    yield
    assert not bj.device_error_check(), "a kernel reported a bounded-wait timeout"


@pytest.mark.parametrize("S,H,W,D,cache_dt,video_dt", [
    (3, 128, 128, 256, "f16", "f16"),
    (2, 64, 96, 1024, "f16", "bf16"),
    (2, 64, 64, 1408, "bf16", "bf16"),
    (2, 64, 64, 96, "f32", "f32"),
])
def test_front_end_steps_match_oracle(cuda_device, S, H, W, D, cache_dt, video_dt):
    import torch

    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
    C, T, KT, P = 3, 2, 2, 16
    n = (T // KT) * (H // P) * (W // P)
    weight = workloads.splitmix_normal(21, (D, C, KT, P, P), 0.02)
    bias = workloads.splitmix_normal(22, (D,), 0.02)
    wd = torch.from_numpy(weight).to(cuda_device, dt[video_dt])
    bd = torch.from_numpy(bias).to(cuda_device)
    cache0 = workloads.splitmix_normal(23, (S, n, D), 1.0)
    caches = torch.from_numpy(cache0).to(cuda_device, dt[cache_dt])
    observed = torch.zeros((S, n), device=cuda_device)
    age = torch.zeros((S, n), device=cuda_device)

    ref_cache = caches.float().cpu().numpy()
    ref_obs = np.zeros((S, n), np.float32)
    ref_age = np.zeros((S, n), np.float32)
    w_exact = wd.float().cpu().numpy()
    ocfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    fe = None
    for step in range(3):
        video = workloads.rect_perturbation_clips(100 + step, S, C, T, H, W, area_fraction=0.2)
        vd = torch.from_numpy(video).to(cuda_device, dt[video_dt])
        xs = vd.float().cpu().numpy()
        thr = workloads.choose_threshold(oracle.patch_diff_token_scores(xs[0:1], KT, P), 0.2)
        mask = bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
        fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, mask, dt[video_dt], dt[cache_dt], cuda_device)
        counts = fe.step(vd, wd, bd, caches, observed, age, age_observed=step > 0).cpu().numpy()
        omask = oracle.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
        for s in range(S):
            idx = oracle.patch_diff_context_mask_from_video(xs[s:s + 1], KT, P, oracle.TokenGridShape(T // KT, H // P, W // P), omask)
            assert counts[s] == len(idx), (step, s)
            coords = oracle.sparse_patchify_plan_coords(idx, oracle.TokenGridShape(T // KT, H // P, W // P), 1)
            feats = oracle.sparse_patchify3d_forward(ocfg, xs[s:s + 1], coords, w_exact, bias)
            rc, ro, ra = ref_cache[s:s + 1], ref_obs[s:s + 1], ref_age[s:s + 1]
            oracle.feature_memory_assign_latest(rc, ro, ra, feats[None], idx.astype(np.int32)[None],
                                                age_observed=step > 0)
        got = caches.float().cpu().numpy()
        assert np.array_equal(observed.cpu().numpy(), ref_obs)
        assert np.array_equal(age.cpu().numpy(), ref_age)
        written = ref_obs.astype(bool) if step == 0 else None
        tol = 1e-2 if cache_dt != "f32" or video_dt != "f32" else 1e-4
        assert max_rel_err(got, ref_cache) <= tol
        if written is not None:
            # rows never written keep their exact pre-filled values
            assert np.array_equal(got[~written], caches.new_tensor(cache0).to(dt[cache_dt]).float().cpu().numpy()[~written])
        ref_cache = got.copy()  # carry the device's rounding forward; exactness is checked per step


def _oracle_front_end(xs, weight, bias, ocfg, grid, omask, ref_cache, ref_obs, ref_age, age_observed):
    counts = []
    for s in range(xs.shape[0]):
        idx = oracle.patch_diff_context_mask_from_video(xs[s:s + 1], ocfg.tubelet_size, ocfg.patch_h, grid, omask)
        counts.append(len(idx))
        coords = oracle.sparse_patchify_plan_coords(idx, grid, 1)
        feats = oracle.sparse_patchify3d_forward(ocfg, xs[s:s + 1], coords, weight, bias)
        oracle.feature_memory_assign_latest(ref_cache[s:s + 1], ref_obs[s:s + 1], ref_age[s:s + 1], feats[None],
                                            idx.astype(np.int32)[None], age_observed=age_observed)
    return np.array(counts)


@pytest.mark.parametrize("name,S,T,H,W,D,mask_kind", [
    ("dilated_cap", 3, 2, 128, 128, 256, "dilated"),      # dilated selection: a launch of its own
    ("topk_fill", 3, 2, 128, 128, 256, "topk"),           # threshold 0, fill to the budget: radix select
    ("many_streams", 70, 2, 32, 48, 128, "adaptive"),     # 70 streams, some static: binary search of offsets
    ("depth_two", 2, 4, 64, 64, 256, "adaptive"),         # two tubelets per clip
    ("one_stream", 1, 2, 256, 256, 512, "adaptive"),
    ("fill_ties", 4, 2, 128, 128, 256, "fill"),            # fill to half the grid: ties among zero scores
])
def test_front_end_mask_policies_match_oracle(cuda_device, name, S, T, H, W, D, mask_kind):
    import torch

    C, KT, P = 3, 2, 16
    grid_t = (T // KT, H // P, W // P)
    n = grid_t[0] * grid_t[1] * grid_t[2]
    grid = oracle.TokenGridShape(*grid_t)
    weight = workloads.splitmix_normal(31, (D, C, KT, P, P), 0.02)
    bias = workloads.splitmix_normal(32, (D,), 0.02)
    wd = torch.from_numpy(weight).to(cuda_device, torch.float16)
    bd = torch.from_numpy(bias).to(cuda_device)
    caches = torch.zeros((S, n, D), device=cuda_device, dtype=torch.float16)
    observed = torch.zeros((S, n), device=cuda_device)
    age = torch.zeros((S, n), device=cuda_device)
    ref_cache = np.zeros((S, n, D), np.float32)
    ref_obs = np.zeros((S, n), np.float32)
    ref_age = np.zeros((S, n), np.float32)
    ocfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    for step in range(2):
        video = workloads.rect_perturbation_clips(300 + step, S, C, T, H, W, area_fraction=0.15)
        if name == "many_streams":
            video[::7, :, 1:] = video[::7, :, :1]  # every 7th stream static: no change, fill to 1 token
        vd = torch.from_numpy(video).to(cuda_device, torch.float16)
        xs = vd.float().cpu().numpy()
        thr = workloads.choose_threshold(oracle.patch_diff_token_scores(xs[1:2], KT, P), 0.15)
        if mask_kind == "dilated":
            args = (thr, max(2, n // 6), 1)
            mask, omask = bj.PatchDiffConfig.new(*args).with_dilation(1), oracle.PatchDiffConfig.new(*args).with_dilation(1)
        elif mask_kind == "fill":
            args = (thr, n // 2, n, 1)
            mask, omask = bj.PatchDiffConfig.adaptive_threshold(*args), oracle.PatchDiffConfig.adaptive_threshold(*args)
        elif mask_kind == "topk":
            args = (0.0, max(2, n // 5), 1)
            mask, omask = bj.PatchDiffConfig.new(*args), oracle.PatchDiffConfig.new(*args)
        else:
            args = (thr, 1, n, 1)
            mask, omask = bj.PatchDiffConfig.adaptive_threshold(*args), oracle.PatchDiffConfig.adaptive_threshold(*args)
        fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, mask, torch.float16, torch.float16, cuda_device)
        counts = fe.step(vd, wd, bd, caches, observed, age, age_observed=step > 0).cpu().numpy()
        want = _oracle_front_end(xs, wd.float().cpu().numpy(), bias, ocfg, grid, omask, ref_cache, ref_obs, ref_age,
                                 step > 0)
        assert np.array_equal(counts, want), name
        assert np.array_equal(observed.cpu().numpy(), ref_obs)
        assert np.array_equal(age.cpu().numpy(), ref_age)
        got = caches.float().cpu().numpy()
        assert max_rel_err(got, ref_cache) <= 1e-2
        ref_cache = got.copy()


def test_front_end_reused_workspace_matches_oracle(cuda_device):
    """One FrontEnd (one workspace) over five steps with changing masks: whatever the step keeps
    in its workspace between steps, every step must match the oracle."""
    import torch

    S, C, T, H, W, KT, P, D = 5, 3, 2, 96, 128, 2, 16, 128
    grid_t = (T // KT, H // P, W // P)
    n = grid_t[0] * grid_t[1] * grid_t[2]
    grid = oracle.TokenGridShape(*grid_t)
    weight = workloads.splitmix_normal(41, (D, C, KT, P, P), 0.02)
    bias = workloads.splitmix_normal(42, (D,), 0.02)
    wd = torch.from_numpy(weight).to(cuda_device, torch.float16)
    bd = torch.from_numpy(bias).to(cuda_device)
    videos = [workloads.rect_perturbation_clips(500 + k, S, C, T, H, W, area_fraction=0.1 + 0.05 * k) for k in range(5)]
    xs_all = [torch.from_numpy(v).to(torch.float16).float().numpy() for v in videos]
    all_scores = np.concatenate([oracle.patch_diff_token_scores(x[s:s + 1], KT, P) for x in xs_all for s in range(S)])
    thr = workloads.choose_threshold(all_scores, 0.15)
    args = (thr, 3, n, 1)
    fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, bj.PatchDiffConfig.adaptive_threshold(*args), torch.float16,
                     torch.float16, cuda_device)
    omask = oracle.PatchDiffConfig.adaptive_threshold(*args)
    caches = torch.zeros((S, n, D), device=cuda_device, dtype=torch.float16)
    observed = torch.zeros((S, n), device=cuda_device)
    age = torch.zeros((S, n), device=cuda_device)
    ref_cache = np.zeros((S, n, D), np.float32)
    ref_obs = np.zeros((S, n), np.float32)
    ref_age = np.zeros((S, n), np.float32)
    ocfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    for step in range(5):
        vd = torch.from_numpy(videos[step]).to(cuda_device, torch.float16)
        counts = fe.step(vd, wd, bd, caches, observed, age, age_observed=step > 0).cpu().numpy()
        want = _oracle_front_end(xs_all[step], wd.float().cpu().numpy(), bias, ocfg, grid, omask, ref_cache, ref_obs,
                                 ref_age, step > 0)
        assert np.array_equal(counts, want), step
        assert np.array_equal(observed.cpu().numpy(), ref_obs), step
        assert np.array_equal(age.cpu().numpy(), ref_age), step
        got = caches.float().cpu().numpy()
        assert max_rel_err(got, ref_cache) <= 1e-2, step
        ref_cache = got.copy()
    assert not bj.device_error_check()


@pytest.mark.parametrize("ring_slots,D,video_dt", [(3, 1024, "f16"), (2, 256, "bf16"), (3, 512, "f32")])
def test_ring_step_equals_the_contiguous_step(cuda_device, ring_slots, D, video_dt):
    """bjf_front_end_step_ring on a frame ring (a live stream that copies only its new frame per
    step) equals bjf_front_end_step on the same two frames stored as a contiguous clip, bit for
    bit, over a sequence of frames that wraps the ring (so for some steps the newer frame sits
    in a lower slot than the older one)."""
    import torch

    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[video_dt]
    S, C, H, W, P = 4, 3, 256, 256, 16
    n = (H // P) * (W // P)
    frames = [torch.from_numpy(workloads.rect_perturbation_clips(300 + f, S, C, 2, H, W, 0.25)[:, :, 0]).to(
        cuda_device, dt) for f in range(5)]  # [S, C, H, W] each
    wd = torch.from_numpy(workloads.splitmix_normal(31, (D, C, 2, P, P), 0.02)).to(cuda_device, dt)
    bd = torch.from_numpy(workloads.splitmix_normal(32, (D,), 0.02)).to(cuda_device)
    cache0 = torch.from_numpy(workloads.splitmix_normal(33, (S, n, D), 1.0)).to(cuda_device, torch.float16)
    clip01 = torch.stack([frames[0], frames[1]], dim=2)
    thr = workloads.choose_threshold(bj.patch_diff_token_scores(clip01.unsqueeze(1), 2, P).cpu().numpy(), 0.25)
    mask = bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
    fe_ring = bj.FrontEnd(S, C, 2, H, W, 2, P, D, mask, dt, torch.float16, cuda_device)
    fe_clip = bj.FrontEnd(S, C, 2, H, W, 2, P, D, mask, dt, torch.float16, cuda_device)
    state = {k: (cache0.clone(), torch.zeros((S, n), device=cuda_device), torch.zeros((S, n), device=cuda_device))
             for k in ("ring", "clip")}
    ring = torch.zeros((S, C, ring_slots, H, W), dtype=dt, device=cuda_device)
    ring[:, :, 0] = frames[0]
    for f in range(1, 5):
        prev_slot, cur_slot = (f - 1) % ring_slots, f % ring_slots
        ring[:, :, cur_slot] = frames[f]  # only the new frame is written
        c_ring = fe_ring.step_ring(ring, prev_slot, cur_slot, wd, bd, *state["ring"], age_observed=f > 1).clone()
        clip = torch.stack([frames[f - 1], frames[f]], dim=2).contiguous()
        c_clip = fe_clip.step(clip, wd, bd, *state["clip"], age_observed=f > 1).clone()
        torch.cuda.synchronize()
        assert torch.equal(c_ring, c_clip), f"frame {f}: counts"
        assert int(c_ring.sum()) > 0
        for a, b in zip(state["ring"], state["clip"]):
            assert torch.equal(a, b), f"frame {f}"


@pytest.mark.gpu
def test_frame_ring_upload_writes_only_its_slot_and_streams(cuda_device):
    """bjf_frame_ring_upload copies streams [b, e) of a host frame into one ring slot; every
    other slot and stream of the ring is left as it was."""
    import torch

    import burn_jepa_b200 as bj

    S, C, H, W, R = 5, 3, 64, 48, 3
    mask = bj.PatchDiffConfig.adaptive_threshold(0.1, 1, (H // 16) * (W // 16), 1)
    fe = bj.FrontEnd(S, C, 2, H, W, 2, 16, 64, mask, torch.float16, torch.float16, cuda_device)
    ring = torch.randn((S, C, R, H, W), device=cuda_device).to(torch.float16)
    before = ring.clone()
    frame = torch.randn((S, C, H, W)).to(torch.float16).pin_memory()
    fe.upload_frame(frame, ring, 1, streams=(1, 4))
    torch.cuda.synchronize()
    want = before.clone()
    want[1:4, :, 1] = frame[1:4].to(cuda_device)
    assert torch.equal(ring, want)
    fe.upload_frame(frame, ring, 2)
    torch.cuda.synchronize()
    want[:, :, 2] = frame.to(cuda_device)
    assert torch.equal(ring, want)
