"""Seeded synthetic inputs with the shapes and value distributions of the front-end workloads.

There is no dataset on this path: the reference's own benches feed synthetic or camera
frames.  These generators stand in for camera video:

* ``rect_perturbation_clips`` -- a smooth base image (Gaussian-blurred uniform noise) shared by
  every frame, plus per-frame uniform[-0.3, 0.3] perturbations inside random rectangles covering
  a chosen fraction of the frame.  Tubelets the rectangles touch change; the rest do not.
* ``normal`` -- patch-embed weights N(0, std^2).
* ``choose_threshold`` -- a patch-diff threshold inside a wide score gap near a target density,
  so that a mask computed with a different summation order selects the same tokens.
* ``multiblock_mask`` -- the ViT-g batch's shared mask: seeded 3-D blocks over the whole temporal
  extent unioned to a token budget (the reference has no multiblock generator of its own).
"""
from __future__ import annotations

import numpy as np


_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(seed: int, n: int) -> np.ndarray:
    """The first n outputs of the splitmix64 sequence started at `seed` (the reference's mixer,
    training/mask.rs:557-563): state_i = seed + (i+1)*golden, output = mix(state_i).  Pure integer
    arithmetic, so the values are identical on every machine."""
    with np.errstate(over="ignore"):
        i = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def splitmix_uniform(seed: int, shape) -> np.ndarray:
    """uniform[0, 1) float32 with 24-bit resolution, bit-identical everywhere."""
    n = int(np.prod(shape))
    return ((splitmix64(seed, n) >> np.uint64(40)).astype(np.float64) * 2.0 ** -24).astype(np.float32).reshape(shape)


def splitmix_normal(seed: int, shape, std: float = 1.0) -> np.ndarray:
    """Approximately N(0, std^2) (Irwin-Hall: sum of 12 uniforms - 6), bit-identical everywhere."""
    n = int(np.prod(shape))
    u = (splitmix64(seed, 12 * n) >> np.uint64(40)).astype(np.float64) * 2.0 ** -24
    return ((u.reshape(n, 12).sum(axis=1) - 6.0) * std).astype(np.float32).reshape(shape)


def _rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence(int(seed)))


def uniform(seed: int, shape, low: float = 0.0, high: float = 1.0) -> np.ndarray:
    return _rng(seed).uniform(low, high, size=shape).astype(np.float32)


def normal(seed: int, shape, std: float = 1.0) -> np.ndarray:
    return (_rng(seed).standard_normal(size=shape) * std).astype(np.float32)


def _blur(img: np.ndarray, sigma: float) -> np.ndarray:
    from scipy.ndimage import gaussian_filter

    return gaussian_filter(img, sigma=sigma, mode="reflect")


def smooth_base(seed: int, channels: int, height: int, width: int, sigma: float = 4.0) -> np.ndarray:
    """Gaussian-blurred uniform noise rescaled to [0, 1], shape [C, H, W]."""
    noise = uniform(seed, (channels, height, width))
    out = np.empty_like(noise)
    for c in range(channels):
        b = _blur(noise[c], sigma)
        lo, hi = float(b.min()), float(b.max())
        out[c] = (b - lo) / max(hi - lo, 1e-6)
    return out


def _rectangles(rng: np.random.Generator, height: int, width: int, area_fraction: float) -> np.ndarray:
    """Boolean [H, W] union of random rectangles covering about `area_fraction` of the frame."""
    mask = np.zeros((height, width), dtype=bool)
    if area_fraction <= 0:
        return mask
    target = area_fraction * height * width
    for _ in range(10000):
        if mask.sum() >= target:
            break
        side = max(1.0, np.sqrt(target) * rng.uniform(0.15, 0.45))
        aspect = rng.uniform(0.5, 2.0)
        h = int(min(height, max(1, round(side / np.sqrt(aspect)))))
        w = int(min(width, max(1, round(side * np.sqrt(aspect)))))
        y = int(rng.integers(0, height - h + 1))
        x = int(rng.integers(0, width - w + 1))
        mask[y:y + h, x:x + w] = True
    return mask


def rect_perturbation_clips(seed: int, streams: int, channels: int, frames: int, height: int, width: int,
                            area_fraction: float, amplitude: float = 0.3, sigma: float = 4.0) -> np.ndarray:
    """[streams, C, T, H, W] float32 clips: smooth base + per-frame rectangle perturbations.

    Each frame's rectangles cover about area_fraction / 2 of the frame, so a frame pair
    differs on about area_fraction of it."""
    rng = _rng(seed)
    out = np.empty((streams, channels, frames, height, width), dtype=np.float32)
    for s in range(streams):
        base = smooth_base(int(rng.integers(1 << 62)), channels, height, width, sigma)
        for f in range(frames):
            out[s, :, f] = base
            m = _rectangles(rng, height, width, area_fraction / 2.0)
            ys, xs = np.nonzero(m)
            if ys.size:
                noise = rng.uniform(-amplitude, amplitude, size=(channels, ys.size)).astype(np.float32)
                out[s, :, f, ys, xs] += noise.T
    return out


def choose_threshold(scores: np.ndarray, target_fraction: float, min_rel_gap: float = 1e-3) -> float:
    """A threshold near the `target_fraction` quantile (from the top) that sits in the middle
    of a gap between adjacent distinct scores at least `min_rel_gap` wide (relative), so that
    any f32 summation order selects the same tokens.  Returns a value > 0."""
    s = np.sort(np.asarray(scores, dtype=np.float64).ravel())[::-1]
    n = s.size
    k = int(round(target_fraction * n))
    k = min(max(k, 1), n - 1)
    best = None
    for radius in range(0, n):
        for kk in (k - radius, k + radius):
            if 1 <= kk <= n - 1:
                hi, lo = s[kk - 1], s[kk]
                if hi > 0 and (hi - lo) > min_rel_gap * hi:
                    best = 0.5 * (hi + lo) if lo > 0 else 0.5 * hi
                    break
        if best is not None:
            break
    if best is None:
        best = float(s[0]) * 0.5 if s[0] > 0 else 1.0
    return float(best)


def rect_perturbation_clips_torch(seed: int, streams: int, channels: int, frames: int, height: int, width: int,
                                  area_fraction: float, device, dtype=None, amplitude: float = 0.3,
                                  sigma: float = 4.0):
    """Device-side generator with the recipe of `rect_perturbation_clips` for bench-scale inputs
    (hundreds of MB): blur and noise on the GPU, rectangles drawn on the host.  Not bit-identical
    to the numpy generator; parity tests use the numpy one."""
    import torch
    import torch.nn.functional as F

    dtype = dtype or torch.float16
    g = torch.Generator(device=device).manual_seed(int(seed))
    rng = _rng(seed)
    radius = int(3 * sigma)
    x = torch.arange(-radius, radius + 1, device=device, dtype=torch.float32)
    k = torch.exp(-x * x / (2 * sigma * sigma))
    k = k / k.sum()
    out = torch.empty((streams, channels, frames, height, width), dtype=dtype, device=device)
    for s in range(streams):
        noise = torch.rand((channels, 1, height, width), generator=g, device=device)
        b = F.conv2d(F.pad(noise, (radius, radius, 0, 0), mode="reflect"), k.view(1, 1, 1, -1))
        b = F.conv2d(F.pad(b, (0, 0, radius, radius), mode="reflect"), k.view(1, 1, -1, 1))[:, 0]
        lo = b.amin(dim=(1, 2), keepdim=True)
        hi = b.amax(dim=(1, 2), keepdim=True)
        base = (b - lo) / (hi - lo).clamp_min(1e-6)
        for f in range(frames):
            frame = base.clone()
            m = torch.from_numpy(_rectangles(rng, height, width, area_fraction / 2.0)).to(device)
            pert = (torch.rand((channels, height, width), generator=g, device=device) * 2 - 1) * amplitude
            frame += pert * m
            out[s, :, f] = frame.to(dtype)
    return out


def multiblock_mask(seed: int, depth: int, height: int, width: int, keep: int) -> np.ndarray:
    """Seeded blocks of spatial scale 0.15-0.2 of the frame and aspect 0.75-1.5, each over the
    whole temporal extent, unioned until `keep` tokens are covered; returns the lowest `keep`
    covered token indices (t * height * width + r * width + c), ascending."""
    rng = np.random.default_rng(seed)
    covered = np.zeros((height, width), bool)
    while covered.sum() * depth < keep:
        area = rng.uniform(0.15, 0.2) * height * width
        aspect = rng.uniform(0.75, 1.5)
        h = max(1, min(height, int(round(np.sqrt(area * aspect)))))
        w = max(1, min(width, int(round(np.sqrt(area / aspect)))))
        r0 = rng.integers(0, height - h + 1)
        c0 = rng.integers(0, width - w + 1)
        covered[r0:r0 + h, c0:c0 + w] = True
    spatial = np.flatnonzero(covered.ravel())
    idx = (np.arange(depth)[:, None] * height * width + spatial[None, :]).ravel()
    return np.sort(idx)[:keep]
