"""EMA update mode and row resets of the token cache (src/feature_memory.rs:227-290, 348-386).

CPU: the oracle against the reference's own test values.  GPU (marked): the device kernels
against the reference's values and the oracle.  The EMA arithmetic is restated in the
reference's f32 operation order on both sides, so f32 caches compare bit-exactly."""
import numpy as np
import pytest

import oracle
from burn_jepa_b200 import workloads
from helpers import known_answers, max_rel_err

KA = known_answers()


def _oracle_memory(c):
    B, (d, h, w), D = c["batch"], c["grid"], c["embed_dim"]
    N = d * h * w
    return (np.zeros((B, N, D), np.float32), np.zeros((B, N), np.float32), np.zeros((B, N), np.float32))


def test_oracle_ema_golden():
    c = KA["feature_memory_ema"]
    feats, obs, age = _oracle_memory(c)
    for step, st in enumerate(c["steps"]):
        tok = np.array(st["tokens"], np.float32).reshape(st["tokens_shape"])
        idx = np.array(st["indices"], np.int32).reshape(c["batch"], -1)
        oracle.feature_memory_update_ema(feats, obs, age, tok, idx, c["alpha"], age_observed=step > 0)
        if "features" in st:
            assert feats.ravel().tolist() == st["features"]
    assert obs.ravel().tolist() == [1.0, 0.0]


def test_oracle_reset_rows_golden():
    c = KA["feature_memory_reset_rows"]
    feats, obs, age = _oracle_memory(c)
    u = c["update"]
    oracle.feature_memory_assign_latest(feats, obs, age, np.array(u["tokens"], np.float32).reshape(u["tokens_shape"]),
                                        np.array(u["indices"], np.int32).reshape(c["batch"], -1), age_observed=False)
    for r in c["reset"]:
        oracle.feature_memory_reset_rows(feats, obs, age, np.array(r["rows"], np.int32))
        assert feats.ravel().tolist() == r["features"]
        assert obs.ravel().tolist() == r["observed"]
    assert not age.any()


def test_oracle_ema_duplicates_add_deltas():
    """The reference's scatter-add semantics for a repeated index (ragged padding repeats the
    last index): both deltas land, so the row moves twice from the gathered previous value."""
    feats = np.full((1, 2, 1), 4.0, np.float32)
    obs = np.ones((1, 2), np.float32)
    age = np.zeros((1, 2), np.float32)
    oracle.feature_memory_update_ema(feats, obs, age, np.array([[[8.0], [8.0]]], np.float32),
                                     np.array([[1, 1]], np.int32), 0.5, age_observed=False)
    assert feats.ravel().tolist() == [4.0, 8.0]  # 4 + 2 * ((4*0.5 + 8*0.5) - 4)
    assert obs.ravel().tolist() == [1.0, 1.0]


# ---------------------------------------------------------------------------
# device
# ---------------------------------------------------------------------------
def _t(a, dev, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


@pytest.mark.gpu
def test_device_ema_golden(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    c = KA["feature_memory_ema"]
    f0, o0, a0 = _oracle_memory(c)
    feats, obs, age = _t(f0, cuda_device), _t(o0, cuda_device), _t(a0, cuda_device)
    for step, st in enumerate(c["steps"]):
        tok = _t(np.array(st["tokens"], np.float32).reshape(st["tokens_shape"]), cuda_device)
        idx = _t(np.array(st["indices"], np.int32).reshape(c["batch"], -1), cuda_device)
        bj.feature_memory_update_ema(feats, obs, age, tok, idx, c["alpha"], age_observed=step > 0)
        if "features" in st:
            assert feats.cpu().numpy().ravel().tolist() == st["features"]
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_device_reset_rows_golden(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    c = KA["feature_memory_reset_rows"]
    f0, o0, a0 = _oracle_memory(c)
    feats, obs, age = _t(f0, cuda_device), _t(o0, cuda_device), _t(a0, cuda_device)
    u = c["update"]
    bj.feature_memory_assign_latest(feats, obs, age,
                                    _t(np.array(u["tokens"], np.float32).reshape(u["tokens_shape"]), cuda_device),
                                    _t(np.array(u["indices"], np.int32).reshape(c["batch"], -1), cuda_device), False)
    for r in c["reset"]:
        bj.feature_memory_reset_rows(feats, obs, age, _t(np.array(r["rows"], np.int32), cuda_device))
        assert feats.cpu().numpy().ravel().tolist() == r["features"]
        assert obs.cpu().numpy().ravel().tolist() == r["observed"]
    assert not age.cpu().numpy().any()
    # out-of-range rows are skipped; an empty list is a no-op
    bj.feature_memory_reset_rows(feats, obs, age, _t(np.array([-1, 5], np.int32), cuda_device))
    bj.feature_memory_reset_rows(feats, obs, age, torch.zeros(0, dtype=torch.int32, device=cuda_device))
    torch.cuda.synchronize()


@pytest.mark.gpu
@pytest.mark.parametrize("cache_dtype,D,alpha", [("f32", 1024, 0.3), ("f32", 13, 0.75), ("f16", 1024, 0.1),
                                                 ("bf16", 768, 0.5), ("f32", 64, 1.7)])
def test_device_ema_matches_oracle(cuda_device, cache_dtype, D, alpha):
    import torch

    import burn_jepa_b200 as bj

    dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[cache_dtype]
    B, N, S = 3, 4096 if D > 64 else 300, 410 if D > 64 else 37
    rng = np.random.default_rng(D)
    cache0 = workloads.splitmix_normal(D, (B, N, D))
    obs0 = (rng.uniform(size=(B, N)) < 0.5).astype(np.float32)
    age0 = rng.integers(0, 5, size=(B, N)).astype(np.float32)
    feats = _t(cache0, cuda_device, dt)
    obs, age = _t(obs0, cuda_device), _t(age0, cuda_device)
    ref_f = feats.float().cpu().numpy()  # the oracle starts from the same (rounded) cache
    ref_o, ref_a = obs0.copy(), age0.copy()
    for step in range(3):  # unique indices per row (the device kernel's contract)
        idx = np.stack([np.sort(rng.choice(N, S, replace=False)) for _ in range(B)]).astype(np.int32)
        if step == 1:
            idx[0, 0] = -3
            idx[1, -1] = N + 7
        tok = workloads.splitmix_normal(D + 10 * step + 1, (B, S, D))
        bj.feature_memory_update_ema(feats, obs, age, _t(tok, cuda_device), _t(idx, cuda_device), alpha,
                                     age_observed=step > 0)
        oracle.feature_memory_update_ema(ref_f, ref_o, ref_a, tok, idx, alpha, age_observed=step > 0)
        if cache_dtype != "f32":  # the device cache rounds every step; follow it
            ref_f = torch.from_numpy(ref_f).to(dt).float().numpy()
    got = feats.float().cpu().numpy()
    if cache_dtype == "f32":
        assert np.array_equal(got, ref_f)
    else:
        assert max_rel_err(got, ref_f) <= 1e-2
    assert np.array_equal(obs.cpu().numpy(), ref_o) and np.array_equal(age.cpu().numpy(), ref_a)


@pytest.mark.gpu
def test_device_ema_shape_errors(cuda_device):
    import torch

    import burn_jepa_b200 as bj

    feats = torch.zeros((1, 4, 2), device=cuda_device)
    obs = torch.zeros((1, 4), device=cuda_device)
    with pytest.raises(bj.BjfError, match="index dims mismatch"):
        bj.feature_memory_update_ema(feats, obs, obs.clone(), torch.zeros((1, 1, 2), device=cuda_device),
                                     torch.zeros((1, 2), dtype=torch.int32, device=cuda_device), 0.5, False)
    with pytest.raises(bj.BjfError, match="requires at least one token"):
        bj.feature_memory_update_ema(feats, obs, obs.clone(), torch.zeros((1, 0, 2), device=cuda_device),
                                     torch.zeros((1, 0), dtype=torch.int32, device=cuda_device), 0.5, False)
