"""bjf_front_end_step_no_alloc: the front-end step for callers that cannot allocate device
memory (their device memory belongs to a framework allocator, or their frame loop forbids
allocation after start-up).  Its scratch is a fixed 4 MiB array inside the library instead of
a caller workspace.

The GPU tests call it through the C ABI twice in a row (the second call ages the cache and
reuses the scratch the first call left behind) and check every output against the
workspace entry point bjf_front_end_step run on identical inputs: the two run the same
kernels on the same inputs, so counts, caches and metadata must be bit-identical.  One call
is also checked against the oracle directly, the bench shape (32 streams x 4096 tokens, close
to the limit) runs once, and a bounded-wait timeout inside the step reaches the caller through
bjf_device_error_check.  They run alone in a fresh process as well as after the rest of the
suite (the first call on a device does the set-up).  This file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

import burn_jepa_b200 as bj
import oracle
from burn_jepa_b200 import _abi, workloads
from helpers import max_rel_err

LIMIT = 4 << 20  # bytes of the fixed scratch array


def _desc(S, H, W, D, thr, n, T=2):
    mask = bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
    return bj.FrontEndDesc(S, 3, T, H, W, 2, 16, D, _abi.DTYPE_F16, _abi.DTYPE_F16, _abi.DTYPE_F16, mask)


def _carve_bytes(S, N):
    """The scratch carve: a 256-byte flag, then scores, indices and counts, each 256-aligned."""
    up = lambda v: (v + 255) // 256 * 256  # noqa: E731
    off = 256
    off = up(off + 4 * S * N)
    off = up(off + 4 * S * N)
    return up(off + 4 * S)


def _call_null_buffers(S, H, W):
    d = _desc(S, H, W, 1024, 0.05, (H // 16) * (W // 16))
    return bj.load().bjf_front_end_step_no_alloc(ctypes.byref(d), None, None, None, None, None, None, 0, None,
                                                 None)


def test_no_alloc_rejects_steps_beyond_its_scratch():
    # 160 streams x 4096 tokens needs more than the fixed 4 MiB: refused before any launch
    d = _desc(160, 1024, 1024, 1024, 0.05, 4096)
    rc = bj.load().bjf_front_end_step_no_alloc(ctypes.byref(d), 16, 16, None, 16, 16, 16, 0, None, None)
    assert rc == _abi.BJF_ERR_UNSUPPORTED
    assert "above the fixed 4194304-byte limit" in bj.last_error()


@pytest.mark.parametrize("H,W", [(1024, 1024), (512, 256), (256, 256)])
def test_no_alloc_limit_matches_the_carve(H, W):
    """The largest accepted stream count for a grid is the largest whose carve fits the 4 MiB:
    it passes the size check (and then stops at the null buffers, before any device call),
    one stream more is refused as unsupported."""
    n = (H // 16) * (W // 16)
    s_max = max(s for s in range(1, 4097) if _carve_bytes(s, n) <= LIMIT)
    assert _carve_bytes(s_max + 1, n) > LIMIT
    assert _call_null_buffers(s_max, H, W) == _abi.BJF_ERR_INVALID_ARGUMENT
    assert "must not be null" in bj.last_error()
    assert _call_null_buffers(s_max + 1, H, W) == _abi.BJF_ERR_UNSUPPORTED
    if n == 4096:
        assert s_max == 127  # the bench's 32 streams x 4096 tokens fit with room to spare


def _run_pair(dev, S, H, W, D, density, seed, calls=2):
    """Runs the workspace step and the no-alloc step on identical inputs, `calls` frames in a
    row; returns both results and the inputs."""
    import torch

    C, T, KT, P = 3, 2, 2, 16
    n = (T // KT) * (H // P) * (W // P)
    videos = [workloads.rect_perturbation_clips_torch(seed + i, S, C, T, H, W, density, dev, torch.float16)
              for i in range(calls)]
    weight = torch.from_numpy(workloads.splitmix_normal(seed + 31, (D, C, KT, P, P), 0.02)).to(dev, torch.float16)
    bias = torch.from_numpy(workloads.splitmix_normal(seed + 32, (D,), 0.02)).to(dev)
    cache0 = torch.from_numpy(workloads.splitmix_normal(seed + 33, (S, n, D), 1.0)).to(dev, torch.float16)
    # a threshold in a gap of every stream's scores, so any f32 summation order keeps the same tokens
    scores = bj.patch_diff_token_scores(videos[0].unsqueeze(1), KT, P).cpu().numpy().ravel()
    thr = workloads.choose_threshold(scores, density)
    desc = _desc(S, H, W, D, thr, n)

    fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, desc.mask, torch.float16, torch.float16, dev)
    ref = dict(cache=cache0.clone(), obs=torch.zeros((S, n), device=dev), age=torch.zeros((S, n), device=dev),
               counts=[])
    for i in range(calls):
        ref["counts"].append(fe.step(videos[i], weight, bias, ref["cache"], ref["obs"], ref["age"],
                                     age_observed=i > 0).clone())

    got = dict(cache=cache0.clone(), obs=torch.zeros((S, n), device=dev), age=torch.zeros((S, n), device=dev),
               counts=[])
    counts = torch.zeros((S,), dtype=torch.int32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    lib = bj.load()
    for i in range(calls):
        rc = lib.bjf_front_end_step_no_alloc(ctypes.byref(desc), p(videos[i]), p(weight), p(bias), p(got["cache"]),
                                             p(got["obs"]), p(got["age"]), int(i > 0), p(counts), stream)
        assert rc == 0, bj.last_error()
        torch.cuda.synchronize()
        got["counts"].append(counts.clone())
    assert not bj.device_error_check()
    return ref, got, dict(videos=videos, weight=weight, bias=bias, cache0=cache0, thr=thr, n=n)


@pytest.mark.gpu
def test_no_alloc_step_matches_workspace_step_twice(cuda_device):
    import torch

    ref, got, _ = _run_pair(cuda_device, 4, 256, 256, 1024, 0.2, 900)
    for i in range(2):
        assert torch.equal(got["counts"][i], ref["counts"][i]), f"call {i}: active counts differ"
    assert torch.equal(got["cache"], ref["cache"])
    assert torch.equal(got["obs"], ref["obs"]) and torch.equal(got["age"], ref["age"])
    assert int(ref["counts"][1].sum()) > 0 and float(got["age"].max()) >= 1.0


@pytest.mark.gpu
def test_no_alloc_step_matches_the_oracle(cuda_device):
    """One no-alloc call against the oracle's front end: masks (observed, counts) exactly,
    every written cache row within the half-precision tolerance, untouched rows bit for bit."""
    import torch

    S, H, W, D = 3, 256, 256, 256
    ref, got, inp = _run_pair(cuda_device, S, H, W, D, 0.25, 940, calls=1)
    n = inp["n"]
    grid = oracle.TokenGridShape(1, H // 16, W // 16)
    cfg = oracle.PatchifyConfig(3, D, 2, H, W, 2, 16, 16)
    v = inp["videos"][0].float().cpu().numpy()
    w = inp["weight"].float().cpu().numpy()
    b = inp["bias"].cpu().numpy()
    ocfg = oracle.PatchDiffConfig.adaptive_threshold(inp["thr"], 1, n, 1)
    cache = inp["cache0"].float().cpu().numpy().copy()
    obs = np.zeros((S, n), np.float32)
    age = np.zeros((S, n), np.float32)
    counts = oracle.front_end_streams(v, cfg, ocfg, w, b, cache, obs, age, age_observed=False)
    assert got["counts"][0].cpu().numpy().tolist() == counts.tolist()
    assert np.array_equal(got["obs"].cpu().numpy(), obs)
    written = obs > 0
    gc = got["cache"].float().cpu().numpy()
    assert np.array_equal(gc[~written], cache[~written])
    assert max_rel_err(gc[written], cache[written]) <= 1e-2
    assert int(written.sum()) > 0 and len(grid) == n


@pytest.mark.gpu
def test_no_alloc_step_at_the_bench_shape(cuda_device):
    """32 streams x [3, 2, 1024, 1024], D = 1024 (3.2 MiB of the 4 MiB scratch): identical to
    the workspace step."""
    import torch

    ref, got, _ = _run_pair(cuda_device, 32, 1024, 1024, 1024, 0.1, 960, calls=1)
    assert torch.equal(got["counts"][0], ref["counts"][0])
    assert torch.equal(got["cache"], ref["cache"])
    assert torch.equal(got["obs"], ref["obs"]) and torch.equal(got["age"], ref["age"])


@pytest.mark.gpu
def test_no_alloc_step_timeout_reaches_the_caller(cuda_device):
    """A bounded wait that runs out inside the no-alloc step's GEMM is reported by
    bjf_device_error_check (the flag lives in the fixed scratch), stays set across a later
    call until it is read, and is cleared by the read; the step then runs normally again."""
    import torch

    S, H, W, D = 1, 128, 128, 256  # 64 tokens: the single-CTA tensor-core kernel
    n = (H // 16) * (W // 16)
    dev = cuda_device
    video = workloads.rect_perturbation_clips_torch(980, S, 3, 2, H, W, 0.3, dev, torch.float16)
    weight = torch.from_numpy(workloads.splitmix_normal(981, (D, 3, 2, 16, 16), 0.02)).to(dev, torch.float16)
    cache = torch.zeros((S, n, D), dtype=torch.float16, device=dev)
    obs = torch.zeros((S, n), device=dev)
    age = torch.zeros((S, n), device=dev)
    desc = _desc(S, H, W, D, 1e-4, n)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    lib = bj.load()

    def call():
        rc = lib.bjf_front_end_step_no_alloc(ctypes.byref(desc), p(video), p(weight), None, p(cache), p(obs),
                                             p(age), 0, None, stream)
        assert rc == 0, bj.last_error()

    assert not bj.device_error_check()
    try:
        bj.set_bounded_wait(1_000_000, stall=True)  # 1 ms, and a wait nothing completes
        call()
        torch.cuda.synchronize()
    finally:
        bj.set_bounded_wait(0, stall=False)
    call()  # a normal call does not wipe the earlier timeout
    assert bj.device_error_check()
    assert not bj.device_error_check()  # read once, cleared
    call()
    torch.cuda.synchronize()
    assert not bj.device_error_check()
    assert int((obs > 0).sum()) > 0 and bool(cache.abs().sum() > 0)
