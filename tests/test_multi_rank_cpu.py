"""Multi-process host logic of the stream-sharded front end, on CPU with gloo ranks.

Each rank takes its block of global streams (burn_jepa_b200.sharding), builds their seeded
clips and runs the front end on them with the oracle (the CPU restatement of the reference
pipeline); the gathered per-stream results must equal a single-process run over all
streams, and the measurement reductions (max seconds, summed units) must match."""
from __future__ import annotations

import json
import os
import socket
import tempfile

import numpy as np
import pytest

C, T, H, W, KT, P, D = 3, 2, 64, 64, 2, 16, 32
N = (T // KT) * (H // P) * (W // P)
BASE_SEED = 2024


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stream_results(streams):
    """Oracle front end over the given global streams, each an independent batch-1 stream."""
    import oracle
    from burn_jepa_b200 import sharding, workloads

    cfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    mcfg = oracle.PatchDiffConfig.adaptive_threshold(1e-4, 1, N, 1)
    weight = workloads.splitmix_normal(7, (D, C, KT, P, P), std=0.02)
    bias = workloads.splitmix_normal(8, (D,), std=0.02)
    out = {}
    for gs in streams:
        video = workloads.rect_perturbation_clips(sharding.stream_seed(BASE_SEED, gs), 1, C, T, H, W, 0.25)
        cache = np.zeros((1, N, D), np.float32)
        obs = np.zeros((1, N), np.float32)
        age = np.zeros((1, N), np.float32)
        counts = oracle.front_end_streams(video, cfg, mcfg, weight, bias, cache, obs, age, age_observed=False)
        out[gs] = {"count": int(counts[0]), "observed": obs.ravel().tolist(),
                   "checksum": float(np.float64(cache).sum())}
    return out


def _rank_main(rank, world, port, total, result_path):
    import datetime

    import torch.distributed as dist

    from burn_jepa_b200 import sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        group = sharding.RankGroup()
        assert (group.rank, group.world) == (rank, world)
        mine = sharding.shard_streams(total, world, rank)
        results = _stream_results(mine)
        gathered = group.gather_objects(results)
        units = group.sum(sum(r["count"] for r in results.values()))
        secs = group.max(0.25 * (rank + 1))
        group.barrier()
        if rank == 0:
            merged = {}
            for part in gathered:
                merged.update(part)
            with open(result_path, "w") as f:
                json.dump({"results": {str(k): v for k, v in merged.items()}, "units": units, "secs": secs,
                           "owned": [list(sharding.shard_streams(total, world, r)) for r in range(world)]}, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 5), (3, 4)])
def test_stream_sharded_ranks_match_single_process(world, total):
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "rank0.json")
        mp.start_processes(_rank_main, args=(world, _free_port(), total, path), nprocs=world, join=True,
                           start_method="spawn")
        with open(path) as f:
            got = json.load(f)
    want = _stream_results(range(total))
    assert sorted(int(k) for k in got["results"]) == list(range(total))
    for gs in range(total):
        g, w = got["results"][str(gs)], want[gs]
        assert g["count"] == w["count"]
        assert g["observed"] == w["observed"]
        assert g["checksum"] == pytest.approx(w["checksum"], rel=1e-12, abs=1e-9)
    assert got["units"] == sum(w["count"] for w in want.values())
    assert got["secs"] == pytest.approx(0.25 * world)
    owned = [s for block in got["owned"] for s in block]
    assert owned == list(range(total))  # every stream exactly once, contiguous blocks


def test_shard_streams_blocks():
    from burn_jepa_b200.sharding import shard_streams, stream_seed

    assert [list(shard_streams(10, 4, r)) for r in range(4)] == [[0, 1, 2], [3, 4, 5], [6, 7], [8, 9]]
    assert [len(shard_streams(256, 8, r)) for r in range(8)] == [32] * 8
    assert list(shard_streams(2, 4, 3)) == []
    with pytest.raises(ValueError):
        shard_streams(4, 2, 2)
    seeds = {stream_seed(7, s) for s in range(1000)}
    assert len(seeds) == 1000
