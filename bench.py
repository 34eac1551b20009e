"""Benchmark of the B200 sparse front end on the live-stream workload.

Workload (per GPU, weak scaling): 32 independent 1024x1024 camera streams, each step a
two-frame clip [3, 2, 1024, 1024] f16 -> patch-diff mask (~10% active tubelets by default)
-> ViT-L/16 patch embed (D = 1024, K = 3*2*16*16 = 1536, f16 in, f32 accumulate) of the
active tubelets -> in-place write into the stream's persistent f16 token cache [4096, 1024]
(pre-filled N(0, 1)).  A "step" is one pass of that front end over every stream of the GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--density D]
                  [--sweep] [--no-rows]

For N > 1 it is launched by torch.distributed.run, one process per GPU; streams are
sharded with no data-path collective (streams share nothing), and timings are the max
over ranks.  Rank 0 prints one JSON line.

value: active tubelets/s with the clips already resident in HBM (two input sets of 403 MB
per GPU alternate, so every step reads its clips from HBM, not L2).
e2e:   the same metric through the public API with host buffers: every step copies its
clips from pinned host memory, runs the step and reads the per-stream active counts back.
rows:  (one GPU) every row of the path timed alone through its public entry point against its
roofline: the selection, the device plan, the standalone cache updates, the RGBA viewer scorer
and mask node, and the gather-GEMM on the ViT-g batch (32 x [3,16,512,512] bf16, 131 072 rows,
D = 1408) plain and with the encoder-input epilogue; beside them (cpu_ms) the oracle on a
bounded sample of the same work, scaled to the whole row.
--impl reference: the reference's CPU algorithm (the C restatement in oracle/, f32 as on
the reference's NdArray backend) on all host threads, over a bounded sample of streams.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "active tubelets/sec (1/2/4/8 B200) + % tensor-pipe/HBM roofline; ViT-L 1024² frames/s"
UNIT = "active tubelets/s"

STREAMS_PER_GPU = 32
KERNELS_PER_STEP = 3  # patch-diff scores, selection, gather-GEMM (+ row plan, + cache write)
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one scores launch per stream of
# this workload, from one ncu --set full capture of the scores kernel at 16 streams
# (207 767 552 bytes / 16), scaled by the stream count for the roofline's `traffic`.
SCORES_DRAM_BYTES_PER_STREAM = 12985472
# The same for the CTA-pair gather-GEMM per active row (34.7 MB read + 0.90 MB written at 6 581
# rows, profiles/gather_gemm_sm100_pair_live_streams_16.md; cold L2, so an upper bound for a warm step).
GEMM_DRAM_BYTES_PER_ROW = 5267
C, T, H, W, KT, P, D = 3, 2, 1024, 1024, 2, 16, 1024
K = C * KT * P * P
GRID = (T // KT, H // P, W // P)
N_TOKENS = GRID[0] * GRID[1] * GRID[2]


ROW_FLUSH_BYTES = 256 << 20  # written, then a second such buffer read, before every standalone row call: 2x L2
VITG = dict(B=32, C=3, T=16, H=512, W=512, KT=2, P=16, D=1408)  # the ViT-g batch


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--density", type=float, default=0.10)
    ap.add_argument("--streams", type=int, default=STREAMS_PER_GPU)
    ap.add_argument("--no-sweep", action="store_true", help="skip the density sweep (5/10/20/40%%)")
    ap.add_argument("--sweep-steps", type=int, default=10)
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling: 256 streams in total, split over the GPUs (default: 32 per GPU)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--load-seconds", type=float, default=2.0,
                    help="back-to-back steps before the timed ones, for the clock sampler (0 under a profiler)")
    ap.add_argument("--no-rows", action="store_true",
                    help="skip the standalone timings of each row of the path (one GPU only)")
    ap.add_argument("--rows", default="select,plan,cache,rgba,front_end,vitg,f32",
                    help="row groups to time: select, plan, cache, rgba, front_end (C2, C3), vitg, f32 (the "
                         "gather-GEMM on f32 operands, the reference's dtype)")
    ap.add_argument("--rows-only", action="store_true",
                    help="time only the row groups of --rows (front_end, vitg and/or f32) and print them, e.g. "
                         "to profile one row alone")
    ap.add_argument("--vitg-clips", type=int, default=32, help="clips of the ViT-g batch row (32 = the benchmark)")
    return ap.parse_args()


# nominal per-GPU figures the roofline fractions are also given against (HBM3e ~8 TB/s, dense
# bf16 2.25 PFLOP/s); the main fraction is against the measured peaks
NOMINAL_HBM_GBS = 8000.0
NOMINAL_BF16_TFLOPS = 2250.0


def read_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            time.sleep(0.5)  # let the sampler start before the load begins
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def errors(self) -> str:
        try:
            return self.proc.stderr.read()[:300] if self.proc else "nvidia-smi not started"
        except Exception:
            return ""

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "raw": self.lines[:3], "stderr": self.errors()}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# distributed plumbing (timing only; no data-path collective)
# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


# ---------------------------------------------------------------------------
# CPU (oracle) leg
# ---------------------------------------------------------------------------
def cpu_front_end_rate(video_f32_streams, weight_f32, bias_f32, thr, budget_s=15.0):
    """Times the oracle front end (f32, all OpenMP threads) stream by stream until `budget_s`
    of CPU work.  Returns (tubelets/s, tubelets, streams, seconds, threads)."""
    import numpy as np

    import oracle

    cfg = oracle.PatchifyConfig(C, D, T, H, W, KT, P, P)
    mcfg = oracle.PatchDiffConfig.adaptive_threshold(thr, 1, N_TOKENS, 1)
    cache = np.zeros((1, N_TOKENS, D), np.float32)
    obs = np.zeros((1, N_TOKENS), np.float32)
    age = np.zeros((1, N_TOKENS), np.float32)
    total, elapsed, streams = 0, 0.0, 0
    n = video_f32_streams.shape[0]
    while True:  # cycle through the sample until `budget_s` of CPU work
        s = streams % n
        v = np.ascontiguousarray(video_f32_streams[s:s + 1])
        t0 = time.perf_counter()
        counts = oracle.front_end_streams(v, cfg, mcfg, weight_f32, bias_f32, cache, obs, age, age_observed=True)
        elapsed += time.perf_counter() - t0
        total += int(counts.sum())
        streams += 1
        if elapsed >= budget_s:
            break
    return total / elapsed, total, streams, elapsed, oracle.num_threads()


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------
def cpu_rows(streams, budget_s=1.0):
    """The oracle (the reference's algorithms restated in C, f32, all host threads) on a bounded
    sample of each standalone row's workload, scaled to the whole workload of that row.  Returns
    {row name: {"cpu_ms": ms for the row's whole workload, "cpu_sample": what was run}}."""
    import numpy as np

    import oracle
    from burn_jepa_b200 import workloads

    def per_call_s(fn):  # mean seconds of fn over at least one call and about budget_s
        n, el = 0, 0.0
        while n == 0 or el < budget_s:
            t0 = time.perf_counter()
            fn()
            el += time.perf_counter() - t0
            n += 1
        return el / n

    rng = np.random.default_rng(31)
    grid = oracle.TokenGridShape(*GRID)
    out = {}

    scores = np.where(rng.uniform(size=N_TOKENS) < 0.1, rng.uniform(0.1, 1.0, N_TOKENS), 0.0).astype(np.float32)
    cfg = oracle.PatchDiffConfig.adaptive_threshold(0.05, 1, N_TOKENS, 1)
    s = per_call_s(lambda: oracle.patch_diff_context_mask_from_scores(scores, grid, cfg))
    out["patch_diff_select"] = (s * streams, f"one stream's {N_TOKENS} scores, x{streams} streams")

    width = 410
    feats = rng.standard_normal((1, N_TOKENS, D)).astype(np.float32)
    obs = np.zeros((1, N_TOKENS), np.float32)
    age = np.zeros((1, N_TOKENS), np.float32)
    toks = rng.standard_normal((1, width, D)).astype(np.float32)
    idx = np.sort(rng.choice(N_TOKENS, width, replace=False)).astype(np.int32)[None]
    s = per_call_s(lambda: oracle.feature_memory_assign_latest(feats, obs, age, toks, idx, True))
    out["feature_memory_assign_latest"] = (s * streams, f"one stream, {width} of {N_TOKENS} rows, x{streams}")
    s = per_call_s(lambda: oracle.feature_memory_update_ema(feats, obs, age, toks, idx, 0.5, True))
    out["feature_memory_update_ema"] = (s * streams, f"one stream, {width} of {N_TOKENS} rows, x{streams}")

    prev = rng.integers(0, 256, size=(H, W, 4), dtype=np.uint8)
    cur = prev.copy()
    cur[: H // 4, : W // 4, :3] = rng.integers(0, 256, size=(H // 4, W // 4, 3), dtype=np.uint8)
    vgrid = oracle.TokenGridShape(1, H // P, W // P)
    s = per_call_s(lambda: oracle.patch_diff_scores_from_rgba(prev, cur, W, P, vgrid))
    out["rgba_patch_diff_scores"] = (s * streams, f"one {W}x{H} RGBA frame pair, x{streams}")

    v = VITG
    clip = rng.standard_normal((1, v["C"], v["T"], v["H"], v["W"])).astype(np.float32)
    ggrid = oracle.TokenGridShape(v["T"] // v["KT"], v["H"] // v["P"], v["W"] // v["P"])
    gmask = workloads.multiblock_mask(601, ggrid.depth, ggrid.height, ggrid.width, len(ggrid) // 2)
    rows = 64
    coords = oracle.sparse_patchify_plan_coords(gmask[:rows], ggrid, 1)
    gw = rng.standard_normal((v["D"], v["C"], v["KT"], v["P"], v["P"])).astype(np.float32) * np.float32(0.02)
    gb = np.zeros(v["D"], np.float32)
    pcfg = oracle.PatchifyConfig(v["C"], v["D"], v["T"], v["H"], v["W"], v["KT"], v["P"], v["P"])
    s = per_call_s(lambda: oracle.sparse_patchify3d_forward(pcfg, clip, coords, gw, gb))
    total_rows = v["B"] * len(gmask)
    out["gather_gemm_vitg_batch"] = (s * total_rows / rows, f"{rows} of the {total_rows} rows, f32")
    return {k: {"cpu_ms": round(t * 1e3, 3), "cpu_sample": d} for k, (t, d) in out.items()}


def make_inputs(torch, dev, streams, density, seed_base):
    """Two input sets of this rank's global streams; each stream's clip depends only on its
    global id, so a stream's content is the same at every GPU count."""
    from burn_jepa_b200 import sharding, workloads

    sets = []
    for i in range(2):
        clips = [workloads.rect_perturbation_clips_torch(sharding.stream_seed(seed_base + 1000 * i, gs), 1, C, T, H, W,
                                                         density, dev, torch.float16) for gs in streams]
        sets.append(torch.cat(clips))
    return sets


def time_rows(torch, bj, dev, videos, weight, bias, mask_cfg, hbm_peak, tflops_peak, reps=20,
              groups=("select", "plan", "cache", "rgba", "front_end", "vitg", "f32"), vitg_clips=32):
    """Each row of the path timed alone through its public entry point, with CUDA events on the
    launching stream.  Before every call 256 MB are written (L2 flushed), another 256 MB are
    read (so L2 holds clean lines, not the flush's dirty ones) and the device sleeps while the
    host enqueues the call, so the events bracket device work only.  Returns
    {name: {row, workload, bound, avg_ms, achieved, unit, peak, frac, ...}}."""
    import numpy as np

    from burn_jepa_b200 import workloads

    stream = torch.cuda.current_stream()
    flush = torch.empty(ROW_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    # after the write flush, a read pass over a second buffer replaces its dirty lines with clean
    # ones, so a timed kernel does not pay for writing the flush buffer back
    flush_clean = torch.ones(ROW_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    flush_sum = torch.zeros((), dtype=torch.int64, device=dev)
    out = {}
    spread = {}  # median and 95th percentile of the last timed() call

    def timed(fn):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for i, (a, b) in enumerate(evs):
            flush.zero_()
            torch.sum(flush_clean, dim=0, dtype=torch.int64, out=flush_sum)
            torch.cuda._sleep(1_000_000)  # ~0.5 ms: longer than the host takes to enqueue the call
            a.record(stream)
            fn(i)
            b.record(stream)
        torch.cuda.synchronize()
        assert not bj.device_error_check(), "a kernel reported a bounded-wait timeout"
        times = sorted(a.elapsed_time(b) for a, b in evs)
        spread["p50_ms"] = round(statistics.median(times), 4)
        spread["p95_ms"] = round(times[min(len(times) - 1, int(0.95 * len(times)))], 4)
        return statistics.mean(times)

    def hbm(name, row, workload, ms, nbytes, **extra):
        gbs = nbytes / (ms / 1e3) / 1e9
        out[name] = {"row": row, "workload": workload, "bound": "hbm", "avg_ms": round(ms, 4), **spread,
                     "algorithmic_bytes": int(nbytes), "achieved": round(gbs, 1), "unit": "GB/s", "peak": hbm_peak,
                     "frac": round(gbs / hbm_peak, 4), "frac_of_nominal": round(gbs / NOMINAL_HBM_GBS, 4), **extra}

    def tensor(name, row, workload, ms, flops, **extra):
        tf = flops / (ms / 1e3) / 1e12
        out[name] = {"row": row, "workload": workload, "bound": "tensor", "avg_ms": round(ms, 4), **spread,
                     "algorithmic_flops": int(flops), "achieved": round(tf, 1), "unit": "TFLOP/s",
                     "peak": tflops_peak, "frac": round(tf / tflops_peak, 4),
                     "frac_of_nominal": round(tf / NOMINAL_BF16_TFLOPS, 4), **extra}

    def latency(name, row, workload, ms, **extra):
        out[name] = {"row": row, "workload": workload, "bound": "latency", "avg_ms": round(ms, 4), **spread, **extra}

    S = videos[0].shape[0] if videos is not None else 0
    live = f"{S} streams, grid {GRID[0]}x{GRID[1]}x{GRID[2]}"
    if {"select", "plan", "cache", "rgba"} & set(groups):
        time_live_rows(torch, bj, dev, videos, mask_cfg, groups, timed, hbm, latency, live)
    if "front_end" in groups:
        time_front_end_rows(torch, bj, dev, timed, hbm, tensor)
    if "vitg" in groups:
        time_vitg_rows(torch, bj, dev, timed, tensor, vitg_clips)
    if "f32" in groups:
        time_f32_rows(torch, bj, dev, timed, tensor)
    del flush, flush_clean
    torch.cuda.empty_cache()
    return out


def time_live_rows(torch, bj, dev, videos, mask_cfg, groups, timed, hbm, latency, live):
    """The selection, plan, cache and RGBA rows on the live-stream workload's frames."""
    import numpy as np

    S = videos[0].shape[0]
    # a2: selection (+ nothing else) on one step's scores
    sc = bj.patch_diff_token_scores(videos[0].unsqueeze(1), KT, P)
    idx = torch.empty((S, N_TOKENS), dtype=torch.int32, device=dev)
    cnt = torch.empty((S,), dtype=torch.int32, device=dev)
    bj.patch_diff_context_mask_from_scores(sc, GRID, mask_cfg, indices=idx, counts=cnt)
    if "select" in groups:
        ms = timed(lambda i: bj.patch_diff_context_mask_from_scores(sc, GRID, mask_cfg, indices=idx, counts=cnt))
        active = int(cnt.sum().item())
        latency("patch_diff_select", "a2", live, ms, active_tokens=active)
    if "plan" in groups:
        time_plan_row(torch, bj, dev, idx, cnt, S, timed, latency, live)
    if "cache" in groups:
        time_cache_rows(torch, bj, dev, S, timed, hbm)
    if "rgba" in groups:
        time_rgba_rows(torch, bj, dev, videos, S, timed, hbm, latency)


def time_plan_row(torch, bj, dev, idx, cnt, S, timed, latency, live):
    # a4 / f2: device plan from the selection
    coords = torch.empty((S * N_TOKENS, 4), dtype=torch.int32, device=dev)
    total = torch.empty((1,), dtype=torch.int32, device=dev)
    ms = timed(lambda i: bj.sparse_patchify_plan_coords(idx, GRID, batch=S, counts=cnt, capacity=S * N_TOKENS,
                                                        coords=coords, total_rows=total))
    latency("plan_coords", "a4", live, ms, rows=int(total.item()))


def time_cache_rows(torch, bj, dev, S, timed, hbm):
    import numpy as np

    # a6 / f3: standalone cache updates, 410 of 4096 tokens per stream (10 %), f16 tokens and cache
    width = 410
    rng = np.random.default_rng(21)
    ti = np.stack([np.sort(rng.choice(N_TOKENS, width, replace=False)) for _ in range(S)]).astype(np.int32)
    tok_idx = torch.from_numpy(ti).to(dev)
    tokens = torch.randn((S, width, D), device=dev).to(torch.float16)
    feats = torch.randn((S, N_TOKENS, D), device=dev).to(torch.float16)
    observed = torch.zeros((S, N_TOKENS), device=dev)
    age = torch.zeros((S, N_TOKENS), device=dev)
    m = S * width
    aging = S * N_TOKENS * 12  # read observed and age, write age
    wl = f"{S} streams x {width} of {N_TOKENS} tokens, D={D}, f16 tokens -> f16 cache"
    ms = timed(lambda i: bj.feature_memory_assign_latest(feats, observed, age, tokens, tok_idx, True))
    hbm("feature_memory_assign_latest", "a6", wl, ms, m * D * 4 + m * 4 + aging + m * 8)
    ms = timed(lambda i: bj.feature_memory_update_ema(feats, observed, age, tokens, tok_idx, 0.5, True))
    hbm("feature_memory_update_ema", "f3", wl, ms, m * D * 6 + m * 4 + aging + m * 8)
    reset_rows = [r for r in (1, 7, 19, 30) if r < S] or [0]
    reset = torch.tensor(reset_rows, dtype=torch.int32, device=dev)
    ms = timed(lambda i: bj.feature_memory_reset_rows(feats, observed, age, reset))
    hbm("feature_memory_reset_rows", "f3", f"{len(reset_rows)} of {S} stream caches [{N_TOKENS},{D}] f16 zeroed",
        ms, len(reset_rows) * N_TOKENS * (D * 2 + 8))
    # a6 again at 40 % (the density sweep's top point): four times the rows, where a call's fixed
    # cost (launch, first-load latency, tail) no longer dominates
    width4 = 4 * width
    ti4 = np.stack([np.sort(rng.choice(N_TOKENS, width4, replace=False)) for _ in range(S)]).astype(np.int32)
    tok_idx4 = torch.from_numpy(ti4).to(dev)
    del tokens
    tokens4 = torch.randn((S, width4, D), device=dev).to(torch.float16)
    m4 = S * width4
    ms = timed(lambda i: bj.feature_memory_assign_latest(feats, observed, age, tokens4, tok_idx4, True))
    hbm("feature_memory_assign_latest_40pct", "a6", f"{S} streams x {width4} of {N_TOKENS} tokens, D={D}, "
        "f16 tokens -> f16 cache", ms, m4 * D * 4 + m4 * 4 + aging + m4 * 8)
    del tokens4, feats, observed, age


def time_rgba_rows(torch, bj, dev, videos, S, timed, hbm, latency):
    # f1: the live viewer's RGBA scorer and mask node on the same streams' frames as RGBA u8
    def rgba(f):
        x = (videos[0][:, :, f].float().clamp(0, 1) * 255).round().to(torch.uint8).permute(0, 2, 3, 1)
        return torch.cat([x, torch.full_like(x[..., :1], 255)], dim=3).contiguous()

    prev, cur = rgba(0), rgba(1)
    vgrid = (1, H // P, W // P)
    wl = f"{S} streams x {W}x{H} RGBA u8 frame pairs, {P}x{P} patches"
    ms = timed(lambda i: bj.patch_diff_scores_from_rgba(prev, cur, P, vgrid))
    hbm("rgba_patch_diff_scores", "f1", wl, ms, 2 * prev.numel() + 4 * S * vgrid[1] * vgrid[2])
    vcfg = bj.PatchDiffConfig.adaptive_threshold(0.03, 0, vgrid[1] * vgrid[2], 1).with_dilation(1)
    policy = bj.ViewerMaskPolicy.new()
    res = {}
    ms = timed(lambda i: res.update(m=bj.viewer_patch_diff_masks_from_rgba(prev, cur, P, vgrid, vcfg, policy)))
    wi, wc, ei, ec = res["m"]
    latency("viewer_patch_diff_masks_from_rgba", "f1", wl + ", threshold 0.03, dilation 1, the viewer's default "
            "dense fallback and encode buckets", ms,
            write_density=round(float(wc.sum().item()) / (S * vgrid[1] * vgrid[2]), 4),
            encode_density=round(float(ec.sum().item()) / (S * vgrid[1] * vgrid[2]), 4))
    del prev, cur


def time_front_end_rows(torch, bj, dev, timed, hbm, tensor):
    from burn_jepa_b200 import workloads

    # C2 / C3: the other front-end configurations, each one fused step alone (inputs smaller
    # than L2 for C2, so the flush before every call matters)
    def front_end_row(name, row, S_, C_, T_, H_, W_, D_, density, seed):
        vids = workloads.rect_perturbation_clips_torch(seed, S_, C_, T_, H_, W_, density, dev, torch.float16)
        sc_ = bj.patch_diff_token_scores(vids.unsqueeze(1), KT, P).cpu().numpy().ravel()
        thr_ = workloads.choose_threshold(sc_, density, 1e-3)
        n_ = (T_ // KT) * (H_ // P) * (W_ // P)
        cfg_ = bj.PatchDiffConfig.adaptive_threshold(thr_, 1, n_, 1)
        fe_ = bj.FrontEnd(S_, C_, T_, H_, W_, KT, P, D_, cfg_, torch.float16, torch.float16, dev)
        w_ = torch.from_numpy(workloads.normal(seed + 1, (D_, C_, KT, P, P), std=0.02)).to(dev, torch.float16)
        b_ = torch.from_numpy(workloads.normal(seed + 2, (D_,), std=0.02)).to(dev)
        cache_ = torch.randn((S_, n_, D_), device=dev).to(torch.float16)
        obs_ = torch.zeros((S_, n_), device=dev)
        age_ = torch.zeros((S_, n_), device=dev)
        ms_ = timed(lambda i: fe_.step(vids, w_, b_, cache_, obs_, age_, age_observed=True))
        m_ = int(fe_.counts.sum().item())
        k_ = C_ * KT * P * P
        nbytes = vids.numel() * 2 + S_ * n_ * 4 + m_ * D_ * 2 + S_ * n_ * 12
        rate = m_ / (ms_ / 1e3)
        wl_ = (f"{S_} x [{C_},{T_},{H_},{W_}] f16, grid {T_ // KT}x{H_ // P}x{W_ // P}, ViT-L/16 D={D_}, "
               f"{m_} of {S_ * n_} tubelets active ({100.0 * m_ / (S_ * n_):.1f}%), f16 caches")
        hbm(name, row, wl_ + "; the fused step (scores, selection, gather-GEMM + cache write)", ms_, nbytes,
            active_tubelets=m_, active_tubelets_per_s=round(rate, 1), frames_per_s=round(S_ * (T_ // KT) /
                                                                                      (ms_ / 1e3), 1))
        # the gather-GEMM of the same rows alone (plain f16 output)
        _, idx_, cnt_ = bj.patch_diff_context_mask(vids.unsqueeze(1), KT, P, (T_ // KT, H_ // P, W_ // P), cfg_)
        co_, tot_ = bj.sparse_patchify_plan_coords(idx_, (T_ // KT, H_ // P, W_ // P), batch=S_, counts=cnt_,
                                                   capacity=S_ * n_)
        rows_ = int(tot_.item())
        co_ = co_[:rows_].contiguous()
        pc_ = bj.PatchifyConfig(C_, D_, T_, H_, W_, KT, P, P)
        fo_ = torch.empty((rows_, D_), device=dev, dtype=torch.float16)
        ms_ = timed(lambda i: bj.sparse_patchify3d_forward(pc_, vids, co_, w_, b_, out=fo_))
        tensor(name + "_gather_gemm", "a5", wl_ + "; the gather-GEMM of its active rows alone", ms_,
               2 * rows_ * k_ * D_, rows=rows_)
        del vids, cache_, fe_

    front_end_row("c2_vitl_clip_step", "a1-a6", 1, C, 16, 256, 256, D, 0.25, 711)
    front_end_row("c3_live_8_streams_step", "a1-a6", 8, C, T, H, W, D, 0.10, 721)


def time_f32_rows(torch, bj, dev, timed, tensor):
    from burn_jepa_b200 import workloads

    # a5 on f32 operands (the reference's CUDA dtype): the tensor cores through the bf16 split,
    # which executes three bf16 products per useful one (K' = 3K); the row reports the useful
    # FLOPs 2 M K D and the executed ones beside them
    def f32_row(name, S_, T_, H_, W_, density, seed):
        vids = workloads.rect_perturbation_clips_torch(seed, S_, C, T_, H_, W_, density, dev, torch.float32)
        grid_ = (T_ // KT, H_ // P, W_ // P)
        n_ = grid_[0] * grid_[1] * grid_[2]
        sc_ = bj.patch_diff_token_scores(vids.unsqueeze(1), KT, P).cpu().numpy().ravel()
        cfg_ = bj.PatchDiffConfig.adaptive_threshold(workloads.choose_threshold(sc_, density, 1e-3), 1, n_, 1)
        _, idx_, cnt_ = bj.patch_diff_context_mask(vids.unsqueeze(1), KT, P, grid_, cfg_)
        co_, tot_ = bj.sparse_patchify_plan_coords(idx_, grid_, batch=S_, counts=cnt_, capacity=S_ * n_)
        rows_ = int(tot_.item())
        co_ = co_[:rows_].contiguous()
        w_ = torch.from_numpy(workloads.normal(seed + 1, (D, C, KT, P, P), std=0.02)).to(dev)
        b_ = torch.from_numpy(workloads.normal(seed + 2, (D,), std=0.02)).to(dev)
        pc_ = bj.PatchifyConfig(C, D, T_, H_, W_, KT, P, P)
        fo_ = torch.empty((rows_, D), device=dev, dtype=torch.float32)
        ms_ = timed(lambda i: bj.sparse_patchify3d_forward(pc_, vids, co_, w_, b_, out=fo_))
        k_ = C * KT * P * P
        wl_ = (f"{S_} x [{C},{T_},{H_},{W_}] f32, grid {grid_[0]}x{grid_[1]}x{grid_[2]}, ViT-L/16 D={D}, {rows_} "
               f"active rows ({100.0 * rows_ / (S_ * n_):.1f}%), f32 weight and output; bf16 hi/lo split of both "
               f"operands (split kernels included), three bf16 products per term")
        tensor(name, "a5", wl_, ms_, 2 * rows_ * k_ * D, rows=rows_, executed_flops=6 * rows_ * k_ * D)
        del vids, fo_

    f32_row("gather_gemm_f32_c2_vitl_clip", 1, 16, 256, 256, 0.25, 731)
    f32_row("gather_gemm_f32_c3_live_8_streams", 8, T, H, W, 0.10, 741)


def time_vitg_rows(torch, bj, dev, timed, tensor, clips):
    import numpy as np

    from burn_jepa_b200 import workloads

    # a5 / f4: the ViT-g batch, a shared 4096-of-8192 multiblock mask, bf16
    v = dict(VITG, B=clips)
    g = torch.Generator(device=dev).manual_seed(602)
    clip = torch.empty((v["B"], v["C"], v["T"], v["H"], v["W"]), dtype=torch.bfloat16, device=dev)
    for b in range(v["B"]):
        clip[b] = ((torch.rand(clip.shape[1:], generator=g, device=dev) - 0.45) / 0.225).to(torch.bfloat16)
    ggrid = (v["T"] // v["KT"], v["H"] // v["P"], v["W"] // v["P"])
    gn = ggrid[0] * ggrid[1] * ggrid[2]
    gmask = workloads.multiblock_mask(601, *ggrid, gn // 2)
    gcoords, gtotal = bj.sparse_patchify_plan_coords(torch.from_numpy(gmask.astype(np.int32)).to(dev), ggrid,
                                                     batch=v["B"])
    rows = int(gtotal.item())
    gcoords = gcoords[:rows].contiguous()
    gk = v["C"] * v["KT"] * v["P"] * v["P"]
    gw = torch.from_numpy(workloads.normal(603, (v["D"], v["C"], v["KT"], v["P"], v["P"]), std=0.02)).to(
        dev, torch.bfloat16)
    gb = torch.from_numpy(workloads.normal(604, (v["D"],), std=0.02)).to(dev)
    gout = torch.empty((rows, v["D"]), dtype=torch.bfloat16, device=dev)
    pcfg = bj.PatchifyConfig(v["C"], v["D"], v["T"], v["H"], v["W"], v["KT"], v["P"], v["P"])
    wl = (f"{v['B']} clips [{v['C']},{v['T']},{v['H']},{v['W']}] bf16, {rows} rows (4096 of 8192 tokens each), "
          f"K={gk}, D={v['D']}, bf16 out")
    ms = timed(lambda i: bj.sparse_patchify3d_forward(pcfg, clip, gcoords, gw, gb, out=gout))
    tensor("gather_gemm_vitg_batch", "a5", wl, ms, 2 * rows * gk * v["D"], rows=rows)
    pos = torch.randn((gn, v["D"]), device=dev) * 0.02
    modality = torch.randn((v["D"],), device=dev) * 0.02
    ms = timed(lambda i: bj.sparse_patchify3d_forward_encoder_input(pcfg, clip, gcoords, gw, gb, position_table=pos,
                                                                     modality_embed=modality, out=gout))
    tensor("gather_gemm_vitg_encoder_input", "f4", wl + ", + position table row + modality vector", ms,
           2 * rows * gk * v["D"], rows=rows)
    del clip, gout


def run_ours(args, world, rank, local):
    import numpy as np
    import torch

    import burn_jepa_b200 as bj
    from burn_jepa_b200 import sharding, workloads

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    group = sharding.RankGroup(device=dev)
    if args.rows_only:  # one or more rows alone, e.g. for a profiler (groups front_end and vitg)
        groups = tuple(args.rows.split(","))
        if not set(groups) <= {"front_end", "vitg", "f32"}:
            raise SystemExit("--rows-only times the front_end, vitg and f32 row groups")
        hbm_peak, tflops_peak, _ = read_peaks()
        rows = time_rows(torch, bj, dev, None, None, None, None, hbm_peak, tflops_peak, groups=groups,
                         vitg_clips=args.vitg_clips)
        if rank == 0:
            print(json.dumps({"rows": rows}), flush=True)
        return
    if args.strong:  # strong scaling: 256 streams in total, split over the GPUs
        total = 256
        mine = sharding.shard_streams(total, world, rank)
        S = len(mine)
    else:  # weak scaling: S streams per GPU
        S = args.streams
        mine = sharding.shard_streams(S * world, world, rank)
    hbm_peak, tflops_peak, peak_kind = read_peaks()

    weight = torch.from_numpy(workloads.normal(11, (D, C, KT, P, P), std=0.02)).to(dev, torch.float16)
    bias = torch.from_numpy(workloads.normal(12, (D,), std=0.02)).to(dev)

    def setup(density):
        videos = make_inputs(torch, dev, mine, density, seed_base=7 + int(density * 1e4))
        # threshold: tubelets the rectangles do not touch score exactly 0, so any small positive
        # threshold keeps exactly the changed tubelets; take it inside a score gap of the first
        # global streams (rank 0's) and use it on every rank
        sc = bj.patch_diff_token_scores(videos[0][:4].unsqueeze(1), KT, P).cpu().numpy().ravel()
        thr = group.broadcast_object(workloads.choose_threshold(sc, density, 1e-3))
        mask = bj.PatchDiffConfig.adaptive_threshold(thr, 1, N_TOKENS, 1)
        fe = bj.FrontEnd(S, C, T, H, W, KT, P, D, mask, torch.float16, torch.float16, dev)
        caches = torch.randn((S, N_TOKENS, D), device=dev, dtype=torch.float32).to(torch.float16)
        observed = torch.zeros((S, N_TOKENS), device=dev)
        age = torch.zeros((S, N_TOKENS), device=dev)
        counts_per_set = []
        for v in videos:
            c = fe.step(v, weight, bias, caches, observed, age)
            counts_per_set.append(int(c.sum().item()))
        return videos, thr, fe, caches, observed, age, counts_per_set

    def time_steps(fe, videos, caches, observed, age, steps, warmup, load_s=0.0):
        stream = torch.cuda.current_stream()
        for i in range(warmup):
            fe.step(videos[i % 2], weight, bias, caches, observed, age)
        torch.cuda.synchronize()
        # sustained load right before the timed steps, long enough for the clock sampler
        t_end = time.perf_counter() + load_s
        while time.perf_counter() < t_end:
            for i in range(64):
                fe.step(videos[i % 2], weight, bias, caches, observed, age)
            torch.cuda.synchronize()
        group.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(steps):
            fe.step(videos[i % 2], weight, bias, caches, observed, age)
        end.record(stream)
        torch.cuda.synchronize()
        group.barrier()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / 1000.0

    videos, thr, fe, caches, observed, age, counts_per_set = setup(args.density)
    try:  # nvidia-smi ignores CUDA_VISIBLE_DEVICES: address the GPU by its UUID
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        gpu_id = str(local)
    with ClockSampler(gpu_id) as clocks:
        secs = time_steps(fe, videos, caches, observed, age, args.steps, args.warmup, load_s=args.load_seconds)
    tubelets = sum(counts_per_set[i % 2] for i in range(args.steps))
    max_secs = group.max(secs)
    all_tubelets = group.sum(float(tubelets))
    value = all_tubelets / max_secs
    frames_per_s = group.sum(float(S * args.steps)) / max_secs
    assert not bj.device_error_check(), "a kernel reported a bounded-wait timeout"

    # ---- per-kernel timings (CUDA events on the launching stream) ----
    stream = torch.cuda.current_stream()
    scores = torch.empty((S, N_TOKENS), device=dev)
    nk = max(args.steps, 5)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(nk)]
    for i in range(3):
        bj.patch_diff_token_scores(videos[i % 2].unsqueeze(1), KT, P, out=scores)
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(evs):
        a.record(stream)
        bj.patch_diff_token_scores(videos[i % 2].unsqueeze(1), KT, P, out=scores)
        b.record(stream)
    torch.cuda.synchronize()
    mask_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    mask_bytes = S * C * T * H * W * 2 + S * N_TOKENS * 4  # clip read once + scores written
    mask_gbs = mask_bytes / (mask_ms / 1e3) / 1e9

    # gather-GEMM alone on the step's active rows (plain f16 output), same inputs
    _, idx, cnt = bj.patch_diff_context_mask(videos[0].unsqueeze(1), KT, P, GRID, fe.desc.mask)
    coords, total = bj.sparse_patchify_plan_coords(idx, GRID, batch=S, counts=cnt, capacity=S * N_TOKENS)
    rows = int(total.item())
    coords = coords[:rows].contiguous()
    pcfg = bj.PatchifyConfig(C, D, T, H, W, KT, P, P)
    vflat = videos[0]
    feats = torch.empty((rows, D), device=dev, dtype=torch.float16)
    for _ in range(3):
        bj.sparse_patchify3d_forward(pcfg, vflat, coords, weight, bias, out=feats)
    torch.cuda.synchronize()
    for a, b in evs:
        a.record(stream)
        bj.sparse_patchify3d_forward(pcfg, vflat, coords, weight, bias, out=feats)
        b.record(stream)
    torch.cuda.synchronize()
    gemm_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    gemm_tflops = 2.0 * rows * K * D / (gemm_ms / 1e3) / 1e12

    step_ms = secs / args.steps * 1e3
    dominant = "patch_diff_scores" if mask_ms >= gemm_ms else "gather_gemm"
    if dominant == "patch_diff_scores":
        roofline = {"kernel": "patch_diff_scores_vec_kernel<__half>", "bound": "hbm", "achieved": round(mask_gbs, 1),
                    "peak": hbm_peak, "unit": "GB/s", "frac": round(mask_gbs / hbm_peak, 4),
                    "frac_of_nominal": round(mask_gbs / NOMINAL_HBM_GBS, 4),
                    "traffic": SCORES_DRAM_BYTES_PER_STREAM * S, "traffic_source": "ncu capture at 16 streams, "
                    "scaled by the stream count", "peak_source": peak_kind,
                    "algorithmic_bytes_per_launch": mask_bytes, "avg_launch_ms": round(mask_ms, 4)}
    else:
        roofline = {"kernel": "gather_gemm_sm100_pair_kernel<__half>", "bound": "tensor",
                    "achieved": round(gemm_tflops, 1),
                    "peak": tflops_peak, "unit": "TFLOP/s", "frac": round(gemm_tflops / tflops_peak, 4),
                    "frac_of_nominal": round(gemm_tflops / NOMINAL_BF16_TFLOPS, 4),
                    "traffic": GEMM_DRAM_BYTES_PER_ROW * rows, "traffic_source": "ncu capture at 16 streams, "
                    "scaled by the active rows", "peak_source": peak_kind,
                    "algorithmic_flops_per_launch": 2 * rows * K * D, "avg_launch_ms": round(gemm_ms, 4)}
    kernels = {
        "patch_diff_scores": {"avg_ms": round(mask_ms, 4), "GB/s": round(mask_gbs, 1),
                              "frac_hbm": round(mask_gbs / hbm_peak, 4)},
        "gather_gemm": {"avg_ms": round(gemm_ms, 4), "rows": rows, "TFLOP/s": round(gemm_tflops, 1),
                        "frac_tensor": round(gemm_tflops / tflops_peak, 4)},
    }

    # ---- e2e through the public API with host buffers ----
    # A live stream uploads one new frame per step: a 3-slot frame ring on the device, the next
    # frame copied from pinned host memory on a copy stream while the current step runs
    # (bjf_front_end_step_ring), each step's active counts read back to the host.  The frames
    # are one continuous synthetic sequence per stream (each frame perturbs the same base in
    # its own rectangles, so consecutive frames differ on the bench's ~10% of the area).
    seq = workloads.rect_perturbation_clips_torch(sharding.stream_seed(9000, mine[0]), S, C, 4, H, W, args.density,
                                                  dev, torch.float16)
    host_frames = seq.permute(2, 0, 1, 3, 4).contiguous().cpu().pin_memory()  # [4, S, C, H, W]
    del seq
    ring_slots = 3
    ring = torch.empty((S, C, ring_slots, H, W), dtype=torch.float16, device=dev)
    e2e_steps = max(1, args.e2e_steps)
    counts_host = torch.zeros((max(e2e_steps, 3) + 1, S), dtype=torch.int32).pin_memory()  # row i: step i
    # two copy streams, each uploading half of the streams' planes with bjf_frame_ring_upload
    # (one 2-D copy each), so two copy engines share the host link
    copy_streams = [torch.cuda.Stream(device=dev) for _ in range(2)]
    halves = [(0, S // 2), (S // 2, S)] if S > 1 else [(0, S)]
    frame_bytes = H * W * 2

    def upload(i, after=None):  # frame i into slot i % 3 on the copy streams
        evs = []
        for cs, half in zip(copy_streams, halves):
            if after is not None:
                cs.wait_event(after)
            fe.upload_frame(host_frames[i % 4], ring, i % ring_slots, streams=half, stream=cs)
            ev = torch.cuda.Event()
            ev.record(cs)
            evs.append(ev)
        return evs

    def e2e_run(n_steps, start_event=None):
        copied, done = {}, {}
        copied[0] = upload(0, start_event)
        tub = 0
        for i in range(1, n_steps + 1):
            # slot i % 3 last held frame i - 3, read by steps i - 3 and i - 2
            copied[i] = upload(i, done.get(i - 2, start_event))
            for ev in copied[i]:
                stream.wait_event(ev)
            fe.step_ring(ring, (i - 1) % ring_slots, i % ring_slots, weight, bias, caches, observed, age)
            counts_host[i].copy_(fe.counts, non_blocking=True)
            done[i] = torch.cuda.Event()
            done[i].record(stream)
        return tub

    e2e_run(3)  # warm-up
    torch.cuda.synchronize()
    group.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    e2e_run(e2e_steps, start_event=a)
    b.record(stream)
    torch.cuda.synchronize()
    e2e_tub = int(counts_host[1:e2e_steps + 1].sum())
    e2e_secs = group.max(a.elapsed_time(b) / 1e3)
    e2e_value = group.sum(float(e2e_tub)) / e2e_secs
    h2d = S * C * frame_bytes
    e2e_density = e2e_tub / (e2e_steps * S * N_TOKENS)
    del host_frames, ring

    sweep = None
    if not args.no_sweep and not args.strong:
        sweep = {}
        for dens in (0.05, 0.10, 0.20, 0.40):
            del fe, caches, observed, age
            torch.cuda.empty_cache()
            videos2, thr2, fe, caches, observed, age, cps = setup(dens)
            s2 = time_steps(fe, videos2, caches, observed, age, args.sweep_steps, args.warmup)
            tub2 = sum(cps[i % 2] for i in range(args.sweep_steps))
            s2m = group.max(s2)
            sweep[f"{int(dens * 100)}%"] = {
                "active_fraction": round(statistics.mean(cps) / (S * N_TOKENS), 4),
                "value": round(group.sum(float(tub2)) / s2m, 1),
                "ms_per_step": round(s2m / args.sweep_steps * 1e3, 4)}
            del videos2

    rows = None
    if world == 1 and not args.no_rows and not args.strong:
        rows = time_rows(torch, bj, dev, videos, weight, bias, fe.desc.mask, hbm_peak, tflops_peak,
                         groups=tuple(args.rows.split(",")), vitg_clips=args.vitg_clips)
        if rank == 0 and not args.no_cpu_baseline:
            try:  # the oracle beside each row; never at the cost of the bench line
                for name, c in cpu_rows(S).items():
                    rows[name].update(c)
                rows["cpu_cores"] = __import__("oracle").num_threads()
            except Exception as e:  # noqa: BLE001
                rows["cpu_error"] = f"{type(e).__name__}: {e}"[:300]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import numpy as np

        sample = videos[0][:8].float().cpu().numpy()
        rate, tub, ns, el, threads = cpu_front_end_rate(sample, weight.float().cpu().numpy(), bias.cpu().numpy(), thr)
        cpu = {"value": round(rate, 1), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{ns} stream-steps cycling over 8 of the {S} streams (first input set), {tub} active "
                          f"tubelets, {el:.1f} s of CPU work, f32"}

    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_secs / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": (f"live camera streams: 256 x [3,2,1024,1024] f16 split over {world} GPU(s)"
                                if args.strong else
                                "live camera streams: 32 x [3,2,1024,1024] f16 per GPU") +
                               ", ViT-L/16 patch embed (D=1024, K=1536), patch-diff mask, f16 token cache "
                               "[4096,1024] per stream",
                   "streams_per_gpu": S, "target_density": args.density,
                   "active_fraction": round(statistics.mean(counts_per_set) / (S * N_TOKENS), 4),
                   "active_tubelets_per_step_per_gpu": counts_per_set,
                   "threshold": thr,
                   "l2": f"inputs larger than L2: two {S * C * T * H * W * 2 / 1e6:.0f} MB clip sets per GPU "
                         "alternate between steps",
                   "clocks_note": "nvidia-smi sampled every 100 ms over 2 s of back-to-back steps "
                                  "immediately before and through the timed steps",
                   "parallelism": f"stream-sharded replicas x{world}, no collective"},
        "frames_per_s": round(frames_per_s, 1),
        "roofline": roofline, "kernels": kernels,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": S * 4,
                "steps": e2e_steps, "active_fraction": round(e2e_density, 4),
                "how": "bjf_front_end_step_ring on a 3-slot frame ring per stream: each step uploads its one new "
                       "[3,1024,1024] f16 frame per stream from pinned host memory with bjf_frame_ring_upload (two "
                       "2-D copies on two copy streams, overlapping the step before) and reads the per-stream "
                       "active counts back; timed with CUDA events"},
        "gpu_launches": KERNELS_PER_STEP * args.steps,
        "clocks": clocks.summary(),
    }
    if sweep:
        result["density_sweep"] = sweep
    if rows:
        result["rows"] = rows
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_reference(args, world, rank, local):
    """CPU reference arm: rank 0 times the oracle front end; other ranks exit."""
    if rank != 0:
        return
    import numpy as np

    import torch

    from burn_jepa_b200 import workloads

    # same recipe, generated on the host (no GPU in the reference arm)
    S = min(args.streams, 8)
    video = workloads.rect_perturbation_clips(7, S, C, T, H, W, args.density)
    weight = workloads.normal(11, (D, C, KT, P, P), std=0.02)
    bias = workloads.normal(12, (D,), std=0.02)
    import oracle

    sc = oracle.patch_diff_token_scores(video[0:1].astype(np.float16).astype(np.float32), KT, P)
    thr = workloads.choose_threshold(sc, args.density, 1e-3)
    vid = video.astype(np.float16).astype(np.float32)
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_front_end_rate(vid[:1], weight, bias, thr, budget_s=0.0)
    per_step = []
    tubelets = 0
    for _ in range(args.steps):
        rate, tub, ns, el, threads = cpu_front_end_rate(vid, weight, bias, thr, budget_s=2.0)
        per_step.append(el)
        tubelets += tub
    value = tubelets / sum(per_step)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(statistics.mean(per_step) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "live camera streams: [3,2,1024,1024] per stream, ViT-L/16 patch embed (D=1024, "
                               "K=1536), patch-diff mask, token cache [4096,1024] per stream",
                   "target_density": args.density, "parallelism": "host threads (OpenMP)"},
        "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"each step: stream-steps cycling over a {S}-stream sample until 2 s of CPU work"},
        "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse_args()
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
