"""The patch-diff refresh state on the device (PatchDiffRefreshState, src/viewer.rs:275-528).

The state of S streams (residual f32 [S, N], age u32 [S, N], frame index u64 [S]) lives in
device memory and advances one frame inside the viewer mask launch.  These tests drive it
frame after frame against the oracle's PatchDiffRefreshState on the same scores: every
frame's write and encode masks must be identical, and so must the whole state -- residuals
bit for bit (both sides evaluate the reference's f32 products, quotient and sum with IEEE
rounding and no contraction), ages and frame indices exactly.  The cases cover each stage
alone and all three together, more candidates than budget (the device's radix select), a
full context budget (no refresh, residuals still updated), the dense fallback, dilation and
encode buckets around the refresh, saturated ages and frame indices, the largest grid, the
RGBA mask node with its state, and observe_write_mask.
"""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

U32_MAX = 0xFFFFFFFF
U64_MAX = 0xFFFFFFFFFFFFFFFF


def _refresh(**kw):
    import burn_jepa_b200 as bj

    return bj.PatchDiffRefreshConfig.from_fields(**kw)


def _check_state(dev_state, ostates, where):
    res = dev_state.subthreshold_residual()
    age = dev_state.age_frames()
    frame = dev_state.frame_index()
    for s, o in enumerate(ostates):
        assert int(frame[s]) == o.frame_index, (where, s, "frame index")
        assert np.array_equal(age[s], o.age), (where, s, "ages")
        assert np.array_equal(res[s].view(np.uint32), o.residual.view(np.uint32)), (where, s, "residuals")


def _slow_motion_scores(rng, S, n, frames, threshold):
    """Per stream: a slowly drifting field mostly below the threshold, a few tokens above it
    every frame, and some frames with no motion at all."""
    base = rng.uniform(0.0, 0.9 * threshold, size=(S, n)).astype(np.float32)
    out = []
    for f in range(frames):
        sc = base * rng.uniform(0.6, 1.2, size=(S, n)).astype(np.float32)
        hot = rng.uniform(size=(S, n)) < 0.03
        sc[hot] = rng.uniform(threshold, 1.0, size=int(hot.sum())).astype(np.float32)
        if f % 5 == 3:
            sc[S - 1] = 0.0  # a still frame: the selection keeps its minimum only
        out.append(sc.astype(np.float32))
    return out


_CASES = {
    # name: (grid, streams, frames, context density, dilation, fallback, bucketed, refresh fields)
    "subthreshold": ((1, 24, 32), 3, 8, 0.3, 0, 1.0, False,
                     dict(enabled=True, subthreshold_enabled=True, subthreshold_decay=0.9, subthreshold_trigger=0.8,
                          subthreshold_max_density=0.05, max_extra_density=0.08)),
    "age": ((1, 24, 32), 3, 9, 0.3, 0, 1.0, False,
            dict(enabled=True, age_refresh_enabled=True, age_refresh_interval_frames=3, age_refresh_max_density=0.03,
                 max_extra_density=0.08)),
    "blue_noise": ((1, 24, 32), 3, 6, 0.3, 0, 1.0, False,
                   dict(enabled=True, blue_noise_enabled=True, blue_noise_refresh_density=0.04, blue_noise_seed=7,
                        max_extra_density=0.08)),
    "all_stages": ((1, 32, 32), 4, 12, 0.25, 1, 0.75, True,
                   dict(enabled=True, subthreshold_enabled=True, subthreshold_decay=0.95, subthreshold_gain=1.5,
                        subthreshold_trigger=1.0, subthreshold_max_density=0.03, age_refresh_enabled=True,
                        age_refresh_interval_frames=4, age_refresh_max_density=0.02, blue_noise_enabled=True,
                        blue_noise_refresh_density=0.02, max_extra_density=0.06)),
    "budget_full": ((1, 16, 32), 2, 5, 0.02, 0, 1.0, True,  # the selection fills the context but on still frames
                    dict(enabled=True, subthreshold_enabled=True, subthreshold_decay=0.9, subthreshold_trigger=0.5,
                         blue_noise_enabled=True, blue_noise_refresh_density=0.5, max_extra_density=0.5)),
    "dense_fallback": ((1, 16, 16), 2, 5, 1.0, 1, 0.02, True,  # every frame but the still one is every token
                       dict(enabled=True, age_refresh_enabled=True, age_refresh_interval_frames=1,
                            age_refresh_max_density=0.1, max_extra_density=0.1)),
    "disabled": ((1, 24, 24), 2, 4, 0.3, 1, 0.75, True, dict()),
    "depth_two": ((2, 12, 20), 2, 6, 0.3, 1, 1.0, True,
                  dict(enabled=True, subthreshold_enabled=True, subthreshold_trigger=0.7, subthreshold_max_density=0.04,
                       blue_noise_enabled=True, blue_noise_refresh_density=0.02, max_extra_density=0.06)),
    "largest_grid": ((1, 128, 256), 2, 3, 0.2, 0, 1.0, True,  # no dilation: room left in the context
                     dict(enabled=True, subthreshold_enabled=True, subthreshold_trigger=0.6,
                          subthreshold_max_density=0.01, age_refresh_enabled=True, age_refresh_interval_frames=2,
                          age_refresh_max_density=0.005, blue_noise_enabled=True, blue_noise_refresh_density=0.003,
                          max_extra_density=0.02)),
}


@pytest.mark.parametrize("name", sorted(_CASES))
def test_refresh_masks_and_state_match_oracle_frame_by_frame(cuda_device, name):
    import torch

    import burn_jepa_b200 as bj

    g, S, frames, ctx_density, dil, fb, bucketed, fields = _CASES[name]
    grid = oracle.TokenGridShape(*g)
    n = len(grid)
    thr = 0.1
    ocfg = oracle.patch_diff_sparsity_config(ctx_density, 0.0, thr, dil, grid)
    cfg = bj.PatchDiffConfig.adaptive_threshold(thr, ocfg.min_context_tokens, ocfg.context_tokens,
                                                ocfg.target_tokens).with_dilation(dil)
    policy = bj.ViewerMaskPolicy.new(fb, 0, bucketed)
    refresh = _refresh(**fields)
    state = bj.PatchDiffRefreshState(S)
    ostates = [oracle.PatchDiffRefreshState() for _ in range(S)]
    rng = np.random.default_rng(sum(map(ord, name)))
    ranked = 0
    for f, sc in enumerate(_slow_motion_scores(rng, S, n, frames, thr)):
        wi, wc, ei, ec = (t.cpu().numpy() for t in state.masks_from_scores(
            torch.from_numpy(sc).to(cuda_device), bj.TokenGridShape(*g), cfg, policy, refresh))
        for s in range(S):
            w, e = ostates[s].masks_from_scores(sc[s], grid, ocfg, fb, fields, bucketed)
            assert wi[s, :wc[s]].tolist() == w.tolist(), (name, f, s, "write mask")
            assert ei[s, :ec[s]].tolist() == e.tolist(), (name, f, s, "encode mask")
            base, _ = oracle.viewer_patch_diff_masks_from_scores(sc[s], grid, ocfg, fb, bucketed)
            ranked += len(w) - len(base)
        _check_state(state, ostates, (name, f))
    if name in ("subthreshold", "age", "blue_noise", "all_stages", "largest_grid", "depth_two"):
        assert ranked > 0, "the case never added a refresh token"
    if name == "disabled":
        assert ranked == 0


def test_refresh_saturated_ages_and_frame_index(cuda_device):
    """Ages at u32::MAX stay there (and many of them round to one f32 priority, so the refresh
    rank decides); a frame index at u64::MAX stays there and still seeds the rank."""
    import torch

    import burn_jepa_b200 as bj

    g, S = (1, 16, 32), 2
    grid = oracle.TokenGridShape(*g)
    n = len(grid)
    ocfg = oracle.patch_diff_sparsity_config(0.3, 0.0, 0.1, 0, grid)
    cfg = bj.PatchDiffConfig.adaptive_threshold(0.1, ocfg.min_context_tokens, ocfg.context_tokens,
                                                ocfg.target_tokens)
    policy = bj.ViewerMaskPolicy.new(1.0, 0, False)
    fields = dict(enabled=True, age_refresh_enabled=True, age_refresh_interval_frames=1 << 40,
                  age_refresh_max_density=0.05, max_extra_density=0.1)
    refresh = _refresh(**fields)
    state = bj.PatchDiffRefreshState(S)
    rng = np.random.default_rng(5)
    sc0 = np.zeros((S, n), np.float32)
    state.masks_from_scores(torch.from_numpy(sc0).to(cuda_device), bj.TokenGridShape(*g), cfg, policy, refresh)
    ages = rng.integers(U32_MAX - 600, U32_MAX + 1, size=(S, n), dtype=np.uint64).astype(np.uint32)
    ages[:, ::7] = U32_MAX
    ostates = []
    for s in range(S):
        o = oracle.PatchDiffRefreshState()
        o.dense_len, o.frame_index = n, (U64_MAX - 1 if s == 0 else 12345)
        o.residual = np.zeros(n, np.float32)
        o.age = ages[s].copy()
        ostates.append(o)
    state.age.copy_(torch.from_numpy(ages.view(np.int32)).to(cuda_device))
    frames = np.array([o.frame_index for o in ostates], dtype=np.uint64).view(np.int64)
    state.frame.copy_(torch.from_numpy(frames).to(cuda_device))
    for f in range(3):
        sc = rng.uniform(0, 0.05, size=(S, n)).astype(np.float32)
        sc[:, f] = 0.5
        wi, wc, _, _ = (t.cpu().numpy() for t in state.masks_from_scores(
            torch.from_numpy(sc).to(cuda_device), bj.TokenGridShape(*g), cfg, policy, refresh))
        for s in range(S):
            w, _ = ostates[s].masks_from_scores(sc[s], grid, ocfg, 1.0, fields, False)
            assert wi[s, :wc[s]].tolist() == w.tolist(), (f, s)
            assert len(w) > 1
        _check_state(state, ostates, f)
    assert int(state.frame_index()[0]) == U64_MAX


def test_refresh_state_starts_over_on_a_new_grid(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    fields = dict(enabled=True, blue_noise_enabled=True, blue_noise_refresh_density=0.05, max_extra_density=0.05)
    refresh = _refresh(**fields)
    state = bj.PatchDiffRefreshState(1)
    o = oracle.PatchDiffRefreshState()
    for g in ((1, 16, 16), (1, 16, 16), (1, 8, 32), (1, 16, 16)):
        grid = oracle.TokenGridShape(*g)
        n = len(grid)
        ocfg = oracle.patch_diff_sparsity_config(0.3, 0.0, 0.1, 0, grid)
        cfg = bj.PatchDiffConfig.adaptive_threshold(0.1, ocfg.min_context_tokens, ocfg.context_tokens,
                                                    ocfg.target_tokens)
        sc = np.zeros((1, n), np.float32)
        sc[0, 3] = 0.5
        wi, wc, _, _ = (t.cpu().numpy() for t in state.masks_from_scores(
            torch.from_numpy(sc).to(cuda_device), bj.TokenGridShape(*g), cfg, bj.ViewerMaskPolicy.new(1.0, 0, False),
            refresh))
        w, _ = o.masks_from_scores(sc[0], grid, ocfg, 1.0, fields, False)
        assert wi[0, :wc[0]].tolist() == w.tolist(), g
        _check_state(state, [o], g)


def test_refresh_reference_cases_on_the_device(cuda_device):
    """The reference's refresh tests (src/viewer.rs:1528-1703) through the device state."""
    import torch

    import burn_jepa_b200 as bj

    g = (1, 4, 4)
    grid = bj.TokenGridShape(*g)
    policy = bj.ViewerMaskPolicy.new(1.0, 0, False)

    def run(state, ctx_density, fields, scores):
        ocfg = oracle.patch_diff_sparsity_config(ctx_density, 0.0, 0.10, 0, oracle.TokenGridShape(*g))
        cfg = bj.PatchDiffConfig.adaptive_threshold(0.10, ocfg.min_context_tokens, ocfg.context_tokens,
                                                    ocfg.target_tokens)
        wi, wc, _, _ = state.masks_from_scores(torch.from_numpy(scores[None]).to(cuda_device), grid, cfg, policy,
                                               _refresh(**fields))
        return wi[0, :int(wc[0])].cpu().numpy().tolist()

    slow = 2 * 4 + 1
    sub = dict(enabled=True, subthreshold_enabled=True, subthreshold_decay=1.0, subthreshold_trigger=1.0,
               subthreshold_max_density=0.25, max_extra_density=0.25)
    scores = np.zeros(16, np.float32)
    scores[0], scores[slow] = 0.09, 0.04
    st = bj.PatchDiffRefreshState(1)
    assert slow not in run(st, 0.25, sub, scores)
    assert slow not in run(st, 0.25, sub, scores)
    assert slow in run(st, 0.25, sub, scores)
    assert st.subthreshold_residual()[0, slow] == 0.0 and st.age_frames()[0, slow] == 0

    budget = dict(enabled=True, subthreshold_enabled=True, subthreshold_decay=1.0, subthreshold_trigger=0.5,
                  subthreshold_max_density=1.0, max_extra_density=1.0)
    scores = np.full(16, 0.06, np.float32)
    scores[0] = 0.09
    assert len(run(bj.PatchDiffRefreshState(1), 2.0 / 16.0, budget, scores)) == 2

    age = dict(enabled=True, age_refresh_enabled=True, age_refresh_interval_frames=2, age_refresh_max_density=0.25,
               max_extra_density=0.25)
    scores = np.zeros(16, np.float32)
    scores[0] = 0.09
    st = bj.PatchDiffRefreshState(1)
    first = run(st, 0.5, age, scores)
    assert len(first) == 1 and len(run(st, 0.5, age, scores)) > len(first)

    blue = dict(enabled=True, blue_noise_enabled=True, blue_noise_refresh_density=0.25, max_extra_density=0.25,
                blue_noise_seed=7)
    zeros = np.zeros(16, np.float32)
    a = run(bj.PatchDiffRefreshState(1), 0.5, blue, zeros)
    b = run(bj.PatchDiffRefreshState(1), 0.5, blue, zeros)
    assert a == b and len(a) > 0


def test_refresh_observe_matches_oracle(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    g, S = (1, 20, 20), 3
    n = g[0] * g[1] * g[2]
    rng = np.random.default_rng(11)
    state = bj.PatchDiffRefreshState(S)
    ostates = [oracle.PatchDiffRefreshState() for _ in range(S)]
    for f in range(4):
        idx = np.zeros((S, n), np.int32)
        cnt = np.zeros(S, np.int32)
        for s in range(S):
            m = int(rng.integers(0, n // 3))
            sel = np.sort(rng.choice(n, size=m, replace=False))
            idx[s, :m], cnt[s] = sel, m
            ostates[s].observe_write_mask(sel, n)
        state.observe_write_mask(torch.from_numpy(idx).to(cuda_device), torch.from_numpy(cnt).to(cuda_device),
                                 bj.TokenGridShape(*g))
        _check_state(state, ostates, f)


def _rgba_frames(seed, S, H, W, changed_frac, slow_level):
    """prev / current RGBA frames: some patches replaced, every other patch nudged by a small
    per-patch offset (slow motion below the threshold)."""
    rng = np.random.default_rng(seed)
    prev = rng.integers(40, 216, size=(S, H, W, 4), dtype=np.uint8)
    cur = prev.astype(np.int32)
    P = 16
    for s in range(S):
        for r in range(H // P):
            for c in range(W // P):
                if rng.uniform() < changed_frac:
                    cur[s, r * P:(r + 1) * P, c * P:(c + 1) * P, :3] = rng.integers(0, 256, size=(P, P, 3))
                else:  # either sign, so the frame shows no uniform lighting shift
                    cur[s, r * P:(r + 1) * P, c * P:(c + 1) * P, :3] += int(rng.integers(-slow_level, slow_level + 1))
    return prev, np.clip(cur, 0, 255).astype(np.uint8)


def test_refresh_rgba_mask_node_matches_oracle(cuda_device):
    """The RGBA mask node with its state over several frames, a dense shortcut among them
    (observe_write_mask of every token).  Masks and ages exactly; residuals to f32 rounding of
    the scores (the device's frame sums are f64, the reference's f32)."""
    import torch

    import burn_jepa_b200 as bj

    S, P, gh, gw = 2, 16, 16, 16
    H, W = gh * P, gw * P
    g = (1, gh, gw)
    grid = oracle.TokenGridShape(*g)
    ocfg = oracle.patch_diff_sparsity_config(1.0, 0.0, 0.06, 1, grid)  # full context: the shortcuts apply
    cfg = bj.PatchDiffConfig.adaptive_threshold(0.06, ocfg.min_context_tokens, ocfg.context_tokens,
                                                ocfg.target_tokens).with_dilation(1)
    fb = 0.6
    policy = bj.ViewerMaskPolicy.new(fb, 0, True)
    fields = dict(enabled=True, subthreshold_enabled=True, subthreshold_trigger=0.9, subthreshold_max_density=0.05,
                  age_refresh_enabled=True, age_refresh_interval_frames=3, age_refresh_max_density=0.02,
                  max_extra_density=0.06)
    refresh = _refresh(**fields)
    state = bj.PatchDiffRefreshState(S)
    ostates = [oracle.PatchDiffRefreshState() for _ in range(S)]
    for f, frac in enumerate((0.04, 0.02, 0.9, 0.03, 0.05, 0.01)):  # frame 2 takes the sampled dense shortcut
        prev, cur = _rgba_frames(700 + f, S, H, W, frac, 12)
        wi, wc, ei, ec = (t.cpu().numpy() for t in state.masks_from_rgba(
            torch.from_numpy(prev).to(cuda_device), torch.from_numpy(cur).to(cuda_device), P, g, cfg, policy,
            refresh))
        for s in range(S):
            w, e = oracle.viewer_patch_diff_refresh_masks_from_rgba(ostates[s], prev[s], cur[s], W, P, grid, ocfg, fb,
                                                                    fields, True)
            assert wi[s, :wc[s]].tolist() == w.tolist(), (f, s)
            assert ei[s, :ec[s]].tolist() == e.tolist(), (f, s)
            if f == 2:
                assert len(w) == len(grid)
        age, frame = state.age_frames(), state.frame_index()
        res = state.subthreshold_residual()
        for s, o in enumerate(ostates):
            assert int(frame[s]) == o.frame_index and np.array_equal(age[s], o.age), (f, s)
            np.testing.assert_allclose(res[s], o.residual, rtol=1e-5, atol=1e-6)


def test_refresh_entry_errors(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    lib = bj.load()
    sc = torch.zeros((1, 16), device=cuda_device)
    out = [torch.zeros((1, 16), dtype=torch.int32, device=cuda_device), torch.zeros(1, dtype=torch.int32,
                                                                                     device=cuda_device)] * 2
    cfg = bj.PatchDiffConfig.adaptive_threshold(0.1, 1, 16, 1)
    pol = bj.ViewerMaskPolicy.new()
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    dims = bj._abi.dims(1, 4, 4)
    missing = bj._abi.PatchDiffRefreshState(None, None, None)
    rc = lib.bjf_viewer_patch_diff_refresh_masks_from_scores(p(sc), 1, dims, ctypes.byref(cfg), ctypes.byref(pol),
                                                             ctypes.byref(_refresh()), ctypes.byref(missing),
                                                             *[p(t) for t in out], None)
    assert rc == bj._abi.BJF_ERR_INVALID_ARGUMENT and "refresh state buffers" in bj.last_error()
    rc = lib.bjf_viewer_patch_diff_refresh_masks_from_scores(p(sc), 1, dims, ctypes.byref(cfg), ctypes.byref(pol),
                                                             None, ctypes.byref(missing), *[p(t) for t in out], None)
    assert rc == bj._abi.BJF_ERR_INVALID_ARGUMENT and "refresh config" in bj.last_error()
