"""bjf_front_end_step_no_alloc: the front-end step for callers that cannot allocate device
memory (their device memory belongs to a framework allocator, or their frame loop forbids
allocation after start-up).  Its scratch is a fixed 4 MiB array inside the library instead of
a caller workspace.

The GPU test calls it through the C ABI twice in a row (the second call ages the cache and
reuses the scratch the first call left behind) and checks every output against the
workspace entry point bjf_front_end_step run on identical inputs.  It runs alone in a fresh
process as well as after the rest of the suite (the first call on a device does the
set-up).  This file is named to be collected last."""
import ctypes

import numpy as np
import pytest

import burn_jepa_b200 as bj
from burn_jepa_b200 import _abi, workloads
from helpers import max_rel_err


def _desc(S, H, W, D, thr, n):
    mask = bj.PatchDiffConfig.adaptive_threshold(thr, 1, n, 1)
    return bj.FrontEndDesc(S, 3, 2, H, W, 2, 16, D, _abi.DTYPE_F16, _abi.DTYPE_F16, _abi.DTYPE_F16, mask)


def test_no_alloc_rejects_steps_beyond_its_scratch():
    # 160 streams x 4096 tokens needs more than the fixed 4 MiB: refused before any launch
    d = _desc(160, 1024, 1024, 1024, 0.05, 4096)
    rc = bj.load().bjf_front_end_step_no_alloc(ctypes.byref(d), 16, 16, None, 16, 16, 16, 0, None, None)
    assert rc == _abi.BJF_ERR_UNSUPPORTED
    assert "above the fixed 4194304-byte limit" in bj.last_error()


@pytest.mark.gpu
def test_no_alloc_step_matches_workspace_step_twice(cuda_device):
    import torch

    S, C, T, H, W, KT, P, D = 4, 3, 2, 256, 256, 2, 16, 1024
    n = (T // KT) * (H // P) * (W // P)
    dev = cuda_device
    videos = [torch.from_numpy(workloads.rect_perturbation_clips(900 + i, S, C, T, H, W, 0.2)).to(dev, torch.float16)
              for i in range(2)]
    weight = torch.from_numpy(workloads.splitmix_normal(31, (D, C, KT, P, P), 0.02)).to(dev, torch.float16)
    bias = torch.from_numpy(workloads.splitmix_normal(32, (D,), 0.02)).to(dev)
    cache0 = torch.from_numpy(workloads.splitmix_normal(33, (S, n, D), 1.0)).to(dev, torch.float16)
    scores = bj.patch_diff_token_scores(videos[0][:1].unsqueeze(1), KT, P).cpu().numpy().ravel()
    thr = workloads.choose_threshold(scores, 0.2)
    desc = _desc(S, H, W, D, thr, n)

    # reference run: the workspace entry point
    fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, desc.mask, torch.float16, torch.float16, dev)
    ref_cache, ref_obs, ref_age = cache0.clone(), torch.zeros((S, n), device=dev), torch.zeros((S, n), device=dev)
    ref_counts = []
    for i in range(2):
        ref_counts.append(fe.step(videos[i], weight, bias, ref_cache, ref_obs, ref_age, age_observed=i > 0).clone())

    # the no-allocation entry point on identical inputs, two calls in a row
    cache, obs, age = cache0.clone(), torch.zeros((S, n), device=dev), torch.zeros((S, n), device=dev)
    counts = torch.zeros((S,), dtype=torch.int32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    lib = bj.load()
    for i in range(2):
        rc = lib.bjf_front_end_step_no_alloc(ctypes.byref(desc), p(videos[i]), p(weight), p(bias), p(cache), p(obs),
                                             p(age), int(i > 0), p(counts), stream)
        assert rc == 0, bj.last_error()
        torch.cuda.synchronize()
        assert torch.equal(counts, ref_counts[i]), f"call {i}: active counts differ"
    assert max_rel_err(cache.float().cpu().numpy(), ref_cache.float().cpu().numpy()) <= 1e-2
    assert torch.equal(obs, ref_obs) and torch.equal(age, ref_age)
    assert int(ref_counts[1].sum()) > 0 and float(age.max()) >= 1.0
