"""The gather-GEMM's give-up path, exercised without faulting or hanging anything.

Every pipeline wait in the tensor-core kernels is bounded in time; on expiry the kernel sets a
device flag, drains its own copies, lets its issued MMAs retire, frees TMEM and returns.  Here
bjf_set_bounded_wait shortens the limit to 1 ms and makes the single-CTA kernel's MMA thread
wait on a barrier that nothing completes (a flag nothing sets), so that wait runs out on a
normal launch.  The host must then see the flag through bjf_device_error_check (once: the read
clears it), the context must stay usable, and the next normal launch must match the oracle.
"""
import numpy as np
import pytest

import burn_jepa_b200 as bj
import oracle
from burn_jepa_b200 import workloads
from helpers import max_rel_err


def _case(dev):
    import torch

    C, T, H, W, KT, P, D = 3, 2, 128, 128, 2, 16, 192
    grid = oracle.TokenGridShape(T // KT, H // P, W // P)
    video = workloads.rect_perturbation_clips(1201, 1, C, T, H, W, 0.5)
    weight = workloads.splitmix_normal(1202, (D, C, KT, P, P), 0.02)
    bias = workloads.splitmix_normal(1203, (D,), 0.02)
    mask = np.arange(0, len(grid), 2, dtype=np.int64)[:40]  # 40 rows: the single-CTA kernel
    coords = oracle.sparse_patchify_plan_coords(mask, grid, 1)
    vd = torch.from_numpy(video).to(dev, torch.float16)
    wd = torch.from_numpy(weight).to(dev, torch.float16)
    bd = torch.from_numpy(bias).to(dev)
    cd = torch.from_numpy(coords.astype(np.int32)).to(dev)
    cfg = bj.PatchifyConfig(C, D, T, H, W, KT, P, P)
    ref = oracle.sparse_patchify3d_forward(oracle.PatchifyConfig(C, D, T, H, W, KT, P, P),
                                           vd.float().cpu().numpy(), coords, wd.float().cpu().numpy(), bias)
    return cfg, vd, cd, wd, bd, ref


@pytest.mark.gpu
def test_wait_that_runs_out_sets_the_flag_and_the_next_launch_is_correct(cuda_device):
    import torch

    cfg, vd, cd, wd, bd, ref = _case(cuda_device)
    assert not bj.device_error_check()
    out = torch.full((cd.shape[0], wd.shape[0]), 7.0, dtype=torch.float32, device=cuda_device)
    try:
        bj.set_bounded_wait(1_000_000, stall=True)
        bj.sparse_patchify3d_forward(cfg, vd, cd, wd, bd, out=out)
        torch.cuda.synchronize()  # the launch returned: no hang, the context is alive
    finally:
        bj.set_bounded_wait(0, stall=False)
    assert bj.device_error_check(), "the expired wait was not reported"
    assert not bj.device_error_check(), "reading the flag must clear it"
    # the kernel gave up before any MMA: no row was written
    assert bool((out == 7.0).all())

    got = bj.sparse_patchify3d_forward(cfg, vd, cd, wd, bd, out=out)
    torch.cuda.synchronize()
    assert not bj.device_error_check()
    assert max_rel_err(got.cpu().numpy(), ref) <= 1e-2


def test_bounded_wait_rejects_a_bad_stall_value():
    assert bj.load().bjf_set_bounded_wait(0, 2) == bj._abi.BJF_ERR_INVALID_ARGUMENT
