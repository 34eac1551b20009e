"""B200 (sm_100a) sparse front end for burn_jepa.

The three steps of burn_jepa's sparse video front end -- patch-diff mask, sparse
patchify (gather-GEMM on tcgen05 tensor cores) and the in-place token-cache write --
as hand-written CUDA kernels behind the C ABI of ``include/bjf.h`` (``libbjf.so``).

This module is the Python face of that ABI for tests, the benchmark and scripting:
each function takes torch CUDA tensors (torch only provides device memory and the
current stream), checks shapes, and calls the C entry point that replaces the
named burn_jepa function.  Nothing here computes on the host or falls back to a
CPU implementation; the C library must be built (``build.build()``).
"""
from __future__ import annotations

import ctypes

from . import _abi
from ._abi import (  # noqa: F401  (re-exported)
    BjfError,
    FrontEndDesc,
    PatchDiffConfig,
    PatchifyConfig,
    check,
    last_error,
    load,
)

__all__ = [
    "BjfError",
    "FrontEnd",
    "PatchDiffConfig",
    "PatchDiffRefreshConfig",
    "PatchDiffRefreshState",
    "PatchifyConfig",
    "TokenGridShape",
    "device_error_check",
    "set_bounded_wait",
    "feature_memory_assign_latest",
    "load",
    "patch_diff_context_mask",
    "patch_diff_context_mask_from_scores",
    "patch_diff_token_scores",
    "sparse_patchify3d_forward",
    "sparse_patchify_plan_coords",
]


class TokenGridShape(tuple):
    """(depth, height, width) token grid (burn_jepa src/tokens.rs:5-32)."""

    def __new__(cls, depth: int, height: int, width: int):
        return super().__new__(cls, (int(depth), int(height), int(width)))

    depth = property(lambda self: self[0])
    height = property(lambda self: self[1])
    width = property(lambda self: self[2])

    def len(self) -> int:
        return self[0] * self[1] * self[2]

    def tokens_per_frame(self) -> int:
        return self[1] * self[2]


def _torch():
    import torch

    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    m = {torch.float32: _abi.DTYPE_F32, torch.float16: _abi.DTYPE_F16, torch.bfloat16: _abi.DTYPE_BF16,
         torch.int32: _abi.DTYPE_I32}
    if t.dtype not in m:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return m[t.dtype]


def _stream(stream=None) -> ctypes.c_void_p:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t) -> ctypes.c_void_p:
    if t is None:
        return ctypes.c_void_p(0)
    if not t.is_cuda:
        raise ValueError("tensor must be on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


def device_error_check(stream=None) -> bool:
    """True when a kernel gave up on a bounded wait since the last check (then cleared)."""
    flag = ctypes.c_int32(0)
    check(load().bjf_device_error_check(_stream(stream), ctypes.byref(flag)))
    return bool(flag.value)


def set_bounded_wait(limit_ns: int = 0, stall: bool = False) -> None:
    """bjf_set_bounded_wait: the time limit of the GEMM kernels' pipeline waits (0 = the 2 s
    default) and the give-up test hook (see include/bjf.h)."""
    check(load().bjf_set_bounded_wait(int(limit_ns), int(bool(stall))))


# ---------------------------------------------------------------------------
# Step 1: patch-diff mask
# ---------------------------------------------------------------------------
def _video_dims(video, streams):
    if video.dim() == 5:
        return (1, tuple(video.shape)) if streams is None else (streams, tuple(video.shape))
    if video.dim() == 6:
        return video.shape[0], tuple(video.shape[1:])
    raise ValueError("video must be [B,C,T,H,W] or [S,B,C,T,H,W]")


def patch_diff_token_scores(video, tubelet_size: int, patch_size: int, out=None, stream=None):
    """`patch_diff_token_scores` (src/nodes.rs:565-631) on the device.

    video: [B,C,T,H,W] or [S,B,C,T,H,W] (S independent videos).  Returns [N] or [S,N] f32."""
    torch = _torch()
    S, vd = _video_dims(video, None)
    B, C, T, H, W = vd
    n = (T // tubelet_size) * (H // patch_size) * (W // patch_size)
    if out is None:
        out = torch.empty((S, n), dtype=torch.float32, device=video.device)
    check(load().bjf_patch_diff_token_scores(_ptr(video), _dtype_code(video), _abi.dims(*vd), S, tubelet_size,
                                             patch_size, _ptr(out), _stream(stream)))
    return out[0] if video.dim() == 5 else out


def patch_diff_context_mask_from_scores(scores, grid, config: PatchDiffConfig, indices=None, counts=None,
                                        stream=None):
    """`patch_diff_context_mask_from_scores` (src/nodes.rs:458-537) on the device.

    scores: [N] or [S,N] f32.  Returns (indices [S,N] int32, counts [S] int32): row s holds
    counts[s] ascending token indices."""
    torch = _torch()
    sc = scores if scores.dim() == 2 else scores.unsqueeze(0)
    S, n = sc.shape
    if indices is None:
        indices = torch.empty((S, n), dtype=torch.int32, device=scores.device)
    if counts is None:
        counts = torch.empty((S,), dtype=torch.int32, device=scores.device)
    check(load().bjf_patch_diff_context_mask_from_scores(_ptr(sc.contiguous()), S, _abi.dims(*grid),
                                                         ctypes.byref(config), _ptr(indices), _ptr(counts),
                                                         _stream(stream)))
    return indices, counts


def patch_diff_context_mask(video, tubelet_size: int, patch_size: int, grid, config: PatchDiffConfig,
                            scores=None, indices=None, counts=None, stream=None):
    """`patch_diff_context_mask_from_video` (src/nodes.rs:539-546) on the device.

    Returns (scores [S,N] f32, indices [S,N] int32, counts [S] int32)."""
    torch = _torch()
    S, vd = _video_dims(video, None)
    n = int(grid[0]) * int(grid[1]) * int(grid[2])
    dev = video.device
    scores = torch.empty((S, n), dtype=torch.float32, device=dev) if scores is None else scores
    indices = torch.empty((S, n), dtype=torch.int32, device=dev) if indices is None else indices
    counts = torch.empty((S,), dtype=torch.int32, device=dev) if counts is None else counts
    check(load().bjf_patch_diff_context_mask(_ptr(video), _dtype_code(video), _abi.dims(*vd), S, tubelet_size,
                                             patch_size, _abi.dims(*grid), ctypes.byref(config), _ptr(scores),
                                             _ptr(indices), _ptr(counts), _stream(stream)))
    return scores, indices, counts


# ---------------------------------------------------------------------------
# Plans
# ---------------------------------------------------------------------------
def sparse_patchify_plan_coords(indices, grid, batch: int, counts=None, capacity: int | None = None,
                                coords=None, total_rows=None, stream=None):
    """Device `SparsePatchifyPlan::new` / `SparsePatchifyBatchPlan::new` (src/sparse_patchify.rs:236-330).

    indices: [mask_rows, stride] int32 (mask_rows 1 = uniform plan, or == batch).  Returns
    (coords [capacity, 4] int32, total_rows [1] int32 on the device)."""
    torch = _torch()
    idx = indices if indices.dim() == 2 else indices.unsqueeze(0)
    mask_rows, stride = idx.shape
    if capacity is None:
        capacity = batch * stride
    dev = indices.device
    coords = torch.empty((capacity, 4), dtype=torch.int32, device=dev) if coords is None else coords
    total_rows = torch.empty((1,), dtype=torch.int32, device=dev) if total_rows is None else total_rows
    check(load().bjf_sparse_patchify_plan_coords(_ptr(idx.contiguous()), stride, _ptr(counts), mask_rows, batch,
                                                 _abi.dims(*grid), _ptr(coords), capacity, _ptr(total_rows),
                                                 _stream(stream)))
    return coords, total_rows


# ---------------------------------------------------------------------------
# Step 2: sparse patchify
# ---------------------------------------------------------------------------
def sparse_patchify3d_forward(config: PatchifyConfig, input, coords, weight, bias=None, out=None,
                              out_dtype=None, stream=None):
    """`burn_flex_gmm::cuda::sparse_patchify3d_forward_cuda` on the sm_100a gather-GEMM.

    input [B,C,T,H,W]; coords [rows,4] int32; weight [D,C,kt,ph,pw]; bias [D] f32 or None.
    Returns [rows, D] (f32 unless out_dtype/out say otherwise)."""
    torch = _torch()
    rows = coords.shape[0]
    if out is None:
        out = torch.empty((rows, config.out_channels), dtype=out_dtype or torch.float32, device=input.device)
    check(load().bjf_sparse_patchify3d_forward(
        ctypes.byref(config), _ptr(input), _dtype_code(input), _abi.dims(*input.shape), _ptr(coords), rows,
        _ptr(weight), _dtype_code(weight), _abi.dims(*weight.shape), _ptr(bias), _ptr(out), _dtype_code(out),
        _stream(stream)))
    return out


def sparse_patchify3d_forward_encoder_input(config: PatchifyConfig, input, coords, weight, bias=None,
                                            position_table=None, modality_embed=None, out=None, out_dtype=None,
                                            stream=None):
    """Sparse patchify producing the encoder's input tokens (src/model.rs:690-703): after the bias
    each row adds position_table[its token index] ([grid tokens, D] f32 or None) and then
    modality_embed ([D] f32 or None)."""
    torch = _torch()
    rows = coords.shape[0]
    if out is None:
        out = torch.empty((rows, config.out_channels), dtype=out_dtype or torch.float32, device=input.device)
    check(load().bjf_sparse_patchify3d_forward_encoder_input(
        ctypes.byref(config), _ptr(input), _dtype_code(input), _abi.dims(*input.shape), _ptr(coords), rows,
        _ptr(weight), _dtype_code(weight), _abi.dims(*weight.shape), _ptr(bias), _ptr(position_table),
        _ptr(modality_embed), _ptr(out), _dtype_code(out), _stream(stream)))
    return out


# ---------------------------------------------------------------------------
# Step 3: token-cache write
# ---------------------------------------------------------------------------
def feature_memory_assign_latest(features, observed, age_frames, tokens, token_indices, age_observed: bool,
                                 stream=None):
    """`sparse_feature_memory_assign_latest_cuda_raw` (src/sparse_feature_memory.rs:296-313), in place.

    features [B,N,D]; observed/age_frames [B,N] f32; tokens [B,S,D]; token_indices [B,S] int32."""
    check(load().bjf_feature_memory_assign_latest(
        _ptr(features), _dtype_code(features), _abi.dims(*features.shape), _ptr(observed),
        _abi.dims(*observed.shape), _ptr(age_frames), _abi.dims(*age_frames.shape), _ptr(tokens),
        _dtype_code(tokens), _abi.dims(*tokens.shape), _ptr(token_indices), _abi.dims(*token_indices.shape),
        int(bool(age_observed)), _stream(stream)))


def feature_memory_update_ema(features, observed, age_frames, tokens, token_indices, alpha: float,
                              age_observed: bool, stream=None):
    """EMA mode of `InterframeJepaFeatureMemory::update_tokens` (src/feature_memory.rs:227-290), in place.

    Same shapes as feature_memory_assign_latest; alpha is clamped to [0, 1]."""
    check(load().bjf_feature_memory_update_ema(
        _ptr(features), _dtype_code(features), _abi.dims(*features.shape), _ptr(observed),
        _abi.dims(*observed.shape), _ptr(age_frames), _abi.dims(*age_frames.shape), _ptr(tokens),
        _dtype_code(tokens), _abi.dims(*tokens.shape), _ptr(token_indices), _abi.dims(*token_indices.shape),
        float(alpha), int(bool(age_observed)), _stream(stream)))


def feature_memory_reset_rows(features, observed, age_frames, rows, stream=None):
    """`InterframeJepaFeatureMemory::reset_rows` (src/feature_memory.rs:348-375): zero the listed batch rows.

    rows: device int32 [R]; rows outside [0, B) are skipped."""
    check(load().bjf_feature_memory_reset_rows(
        _ptr(features), _dtype_code(features), _abi.dims(*features.shape), _ptr(observed), _ptr(age_frames),
        _ptr(rows), int(rows.numel()), _stream(stream)))


# ---------------------------------------------------------------------------
# Live viewer scorer (RGBA u8 frames)
# ---------------------------------------------------------------------------
RgbaFrameStats = _abi.RgbaFrameStats


def patch_diff_scores_from_rgba(prev, current, patch_size: int, grid, stats: bool = False, stream=None):
    """`patch_diff_scores_from_rgba` (src/viewer.rs:1126-1157) for S frame pairs at once.

    prev / current: uint8 [S, H, W, 4] (or [H, W, 4]) RGBA on the device; grid = (1, gh, gw).
    Returns scores [S, gh * gw] f32 (and the per-stream RgbaFrameStats list when `stats`)."""
    torch = _torch()
    single = prev.dim() == 3
    if single:
        prev, current = prev.unsqueeze(0), current.unsqueeze(0)
    S, H, W, _ = prev.shape
    g = tuple(int(v) for v in (grid.depth, grid.height, grid.width)) if hasattr(grid, "depth") else tuple(grid)
    scores = torch.empty((S, g[1] * g[2]), dtype=torch.float32, device=prev.device)
    nbytes = load().bjf_rgba_patch_diff_workspace_bytes(S, _abi.dims(*g))
    ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=prev.device)
    st = torch.empty((S, ctypes.sizeof(RgbaFrameStats)), dtype=torch.uint8, device=prev.device) if stats else None
    check(load().bjf_rgba_patch_diff_scores(
        _ptr(prev), _ptr(current), S, W, H, int(patch_size), _abi.dims(*g), _ptr(scores),
        _ptr(st) if st is not None else None, _ptr(ws), ws.numel(), _stream(stream)))
    out = scores[0] if single else scores
    if not stats:
        return out
    raw = st.cpu().numpy().tobytes()
    sz = ctypes.sizeof(RgbaFrameStats)
    return out, [RgbaFrameStats.from_buffer_copy(raw[i * sz:(i + 1) * sz]) for i in range(S)]


ViewerMaskPolicy = _abi.ViewerMaskPolicy


def viewer_patch_diff_masks(direct_indices, direct_counts, grid, policy: "ViewerMaskPolicy", out=None,
                            stream=None):
    """The live viewer's policy after the selection (src/viewer.rs:780-816, 946-961) on the device.

    direct_indices [S, N] / direct_counts [S] int32 (a selection without dilation) ->
    (write_indices [S, N], write_counts [S], encode_indices [S, N], encode_counts [S]).
    `out` may name the direct buffers as the write buffers."""
    torch = _torch()
    S, N = direct_indices.shape
    if out is None:
        dev = direct_indices.device
        out = (torch.empty((S, N), dtype=torch.int32, device=dev), torch.empty((S,), dtype=torch.int32, device=dev),
               torch.empty((S, N), dtype=torch.int32, device=dev), torch.empty((S,), dtype=torch.int32, device=dev))
    wi, wc, ei, ec = out
    check(load().bjf_viewer_patch_diff_masks(_ptr(direct_indices), _ptr(direct_counts), S, _abi.dims(*grid),
                                             ctypes.byref(policy), _ptr(wi), _ptr(wc), _ptr(ei), _ptr(ec),
                                             _stream(stream)))
    return out


def viewer_patch_diff_masks_from_scores(scores, grid, config: PatchDiffConfig, policy: "ViewerMaskPolicy",
                                        stream=None):
    """patch_diff_masks_from_scores (src/viewer.rs:831-841) on the device for S streams: the
    selection of `config` without dilation, then the policy dilating by config.dilation.

    scores [S, N] f32 -> (write_indices [S, N], write_counts [S], encode_indices [S, N],
    encode_counts [S]), each row ascending up to its count."""
    torch = _torch()
    sc = scores if scores.dim() == 2 else scores.unsqueeze(0)
    S, N = sc.shape
    dev = scores.device
    wi = torch.empty((S, N), dtype=torch.int32, device=dev)
    wc = torch.empty((S,), dtype=torch.int32, device=dev)
    ei = torch.empty((S, N), dtype=torch.int32, device=dev)
    ec = torch.empty((S,), dtype=torch.int32, device=dev)
    check(load().bjf_viewer_patch_diff_masks_from_scores(_ptr(sc.contiguous()), S, _abi.dims(*grid),
                                                         ctypes.byref(config), ctypes.byref(policy), _ptr(wi),
                                                         _ptr(wc), _ptr(ei), _ptr(ec), _stream(stream)))
    return wi, wc, ei, ec


def viewer_patch_diff_masks_from_rgba(prev, current, patch_size: int, grid, config: PatchDiffConfig,
                                      policy: "ViewerMaskPolicy", stats: bool = False, stream=None):
    """The Bevy RGBA mask node without refresh state (crates/bevy_jepa/src/mask.rs:126-175) on
    the device: dense fast paths, else RGBA scores -> patch_diff_masks_from_scores.

    prev / current: [S, H, W, 4] (or [H, W, 4]) uint8 CUDA tensors.  Returns (write_indices,
    write_counts, encode_indices, encode_counts) and, with stats=True, the frame statistics."""
    torch = _torch()
    p = prev if prev.dim() == 4 else prev.unsqueeze(0)
    c = current if current.dim() == 4 else current.unsqueeze(0)
    S, H, W, _ = p.shape
    g = tuple(int(v) for v in grid)
    N = g[1] * g[2]
    dims = _abi.dims(*g)
    lib = load()
    nbytes = lib.bjf_viewer_rgba_masks_workspace_bytes(S, dims)
    ws = torch.empty((max(int(nbytes), 1) + 255,), dtype=torch.uint8, device=prev.device)
    off = (-ws.data_ptr()) % 256
    dev = prev.device
    wi = torch.empty((S, N), dtype=torch.int32, device=dev)
    wc = torch.empty((S,), dtype=torch.int32, device=dev)
    ei = torch.empty((S, N), dtype=torch.int32, device=dev)
    ec = torch.empty((S,), dtype=torch.int32, device=dev)
    st = torch.empty((S, ctypes.sizeof(_abi.RgbaFrameStats)), dtype=torch.uint8, device=dev) if stats else None
    check(lib.bjf_viewer_patch_diff_masks_from_rgba(
        _ptr(p.contiguous()), _ptr(c.contiguous()), S, W, H, patch_size, dims, ctypes.byref(config),
        ctypes.byref(policy), _ptr(wi), _ptr(wc), _ptr(ei), _ptr(ec), _ptr(st) if st is not None else None,
        ctypes.c_void_p(ws.data_ptr() + off), int(nbytes), _stream(stream)))
    if not stats:
        return wi, wc, ei, ec
    raw = st.cpu().numpy().tobytes()
    size = ctypes.sizeof(_abi.RgbaFrameStats)
    return (wi, wc, ei, ec), [_abi.RgbaFrameStats.from_buffer_copy(raw[i * size:(i + 1) * size]) for i in range(S)]


PatchDiffRefreshConfig = _abi.PatchDiffRefreshConfig


class PatchDiffRefreshState:
    """PatchDiffRefreshState (src/viewer.rs:275-528) of S streams, held on the device.

    Per stream and token: the decayed residual of below-threshold motion (f32) and the frames
    since the token was last written (u32, stored in an int32 tensor); per stream the frame
    index (u64, stored in an int64 tensor).  Each call advances every stream one frame in the
    viewer mask launch itself; nothing is read back.  Like the reference, the state starts over
    (zeros, frame 0) when the grid's token count changes, and on `reset()`."""

    def __init__(self, streams: int = 1, device=None):
        self.streams = int(streams)
        self.device = device
        self.dense_len = 0
        self.residual = self.age = self.frame = None

    def reset(self):
        self.dense_len = 0

    def _begin(self, n: int, device):
        torch = _torch()
        if self.dense_len != n or self.residual is None or self.residual.device != device:
            S = self.streams
            self.residual = torch.zeros((S, n), dtype=torch.float32, device=device)
            self.age = torch.zeros((S, n), dtype=torch.int32, device=device)
            self.frame = torch.zeros((S,), dtype=torch.int64, device=device)
            self.dense_len = n
        st = _abi.PatchDiffRefreshState(self.residual.data_ptr(), self.age.data_ptr(), self.frame.data_ptr())
        return st

    def frame_index(self):
        """Per-stream frame index (numpy uint64)."""
        return None if self.frame is None else self.frame.cpu().numpy().view("uint64")

    def subthreshold_residual(self):
        return None if self.residual is None else self.residual.cpu().numpy()

    def age_frames(self):
        """[S, N] numpy uint32."""
        return None if self.age is None else self.age.cpu().numpy().view("uint32")

    def _outputs(self, S, N, dev):
        torch = _torch()
        return (torch.empty((S, N), dtype=torch.int32, device=dev), torch.empty((S,), dtype=torch.int32, device=dev),
                torch.empty((S, N), dtype=torch.int32, device=dev), torch.empty((S,), dtype=torch.int32, device=dev))

    def masks_from_scores(self, scores, grid, config: PatchDiffConfig, policy: "ViewerMaskPolicy",
                          refresh: "PatchDiffRefreshConfig", stream=None):
        """PatchDiffRefreshState::masks_from_scores (src/viewer.rs:312-356): scores [S, N] f32 ->
        (write_indices, write_counts, encode_indices, encode_counts), as
        viewer_patch_diff_masks_from_scores with the refresh tokens in the write mask."""
        sc = scores if scores.dim() == 2 else scores.unsqueeze(0)
        S, N = sc.shape
        if S != self.streams:
            raise ValueError(f"refresh state holds {self.streams} streams, scores have {S}")
        st = self._begin(N, sc.device)
        wi, wc, ei, ec = self._outputs(S, N, sc.device)
        check(load().bjf_viewer_patch_diff_refresh_masks_from_scores(
            _ptr(sc.contiguous()), S, _abi.dims(*grid), ctypes.byref(config), ctypes.byref(policy),
            ctypes.byref(refresh), ctypes.byref(st), _ptr(wi), _ptr(wc), _ptr(ei), _ptr(ec), _stream(stream)))
        return wi, wc, ei, ec

    def masks_from_rgba(self, prev, current, patch_size: int, grid, config: PatchDiffConfig,
                        policy: "ViewerMaskPolicy", refresh: "PatchDiffRefreshConfig", stream=None):
        """The RGBA mask node with this refresh state (crates/bevy_jepa/src/mask.rs:126-185)."""
        torch = _torch()
        p = prev if prev.dim() == 4 else prev.unsqueeze(0)
        c = current if current.dim() == 4 else current.unsqueeze(0)
        S, H, W, _ = p.shape
        if S != self.streams:
            raise ValueError(f"refresh state holds {self.streams} streams, frames have {S}")
        g = tuple(int(v) for v in grid)
        N = g[1] * g[2]
        dims = _abi.dims(*g)
        lib = load()
        nbytes = lib.bjf_viewer_rgba_masks_workspace_bytes(S, dims)
        ws = torch.empty((max(int(nbytes), 1) + 255,), dtype=torch.uint8, device=prev.device)
        off = (-ws.data_ptr()) % 256
        st = self._begin(N, prev.device)
        wi, wc, ei, ec = self._outputs(S, N, prev.device)
        check(lib.bjf_viewer_patch_diff_refresh_masks_from_rgba(
            _ptr(p.contiguous()), _ptr(c.contiguous()), S, W, H, patch_size, dims, ctypes.byref(config),
            ctypes.byref(policy), ctypes.byref(refresh), ctypes.byref(st), _ptr(wi), _ptr(wc), _ptr(ei), _ptr(ec),
            None, ctypes.c_void_p(ws.data_ptr() + off), int(nbytes), _stream(stream)))
        return wi, wc, ei, ec

    def observe_write_mask(self, write_indices, write_counts, grid, stream=None):
        """observe_write_mask (src/viewer.rs:309-313): write_indices [S, N] / write_counts [S]."""
        S, N = write_indices.shape
        st = self._begin(N, write_indices.device)
        check(load().bjf_viewer_patch_diff_refresh_observe(_ptr(write_indices), _ptr(write_counts), S,
                                                            _abi.dims(*grid), ctypes.byref(st), _stream(stream)))


# ---------------------------------------------------------------------------
# Fused step over S independent streams
# ---------------------------------------------------------------------------
class FrontEnd:
    """One frame step of the whole front end for S independent streams (``bjf_front_end_step``).

    Each stream is a video [C, T, H, W] (batch 1) with its own persistent token cache
    [N, D], observed [N] and age [N].  ``step`` runs patch-diff scores -> selection ->
    tcgen05 gather-GEMM -> in-place cache write for every stream and returns the device
    tensor of per-stream active tubelet counts.  Owns its device workspace."""

    def __init__(self, streams: int, channels: int, frames: int, height: int, width: int, tubelet_size: int,
                 patch_size: int, embed_dim: int, mask: PatchDiffConfig, video_dtype, cache_dtype, device,
                 weight_dtype=None):
        torch = _torch()
        dt = {torch.float32: _abi.DTYPE_F32, torch.float16: _abi.DTYPE_F16, torch.bfloat16: _abi.DTYPE_BF16}
        self.desc = FrontEndDesc(streams, channels, frames, height, width, tubelet_size, patch_size, embed_dim,
                                 dt[video_dtype], dt[weight_dtype or video_dtype], dt[cache_dtype], mask)
        nbytes = load().bjf_front_end_workspace_bytes(ctypes.byref(self.desc))
        if nbytes == 0:
            raise BjfError(_abi.BJF_ERR_INVALID_ARGUMENT, last_error())
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.counts = torch.zeros(streams, dtype=torch.int32, device=device)
        self.grid = TokenGridShape(frames // tubelet_size, height // patch_size, width // patch_size)
        self.steps = 0

    def step(self, video, weight, bias, caches, observed, age_frames, age_observed=None, stream=None):
        """video [S,C,T,H,W]; weight [D,C,kt,P,P]; bias [D] f32 or None; caches [S,N,D];
        observed / age_frames [S,N] f32.  age_observed defaults to (this object has stepped)."""
        if age_observed is None:
            age_observed = self.steps > 0
        check(load().bjf_front_end_step(
            ctypes.byref(self.desc), _ptr(video), _ptr(weight), _ptr(bias), _ptr(caches), _ptr(observed),
            _ptr(age_frames), int(bool(age_observed)), _ptr(self.workspace), self.workspace.numel(),
            _ptr(self.counts), _stream(stream)))
        self.steps += 1
        return self.counts

    def step_ring(self, ring, prev_slot: int, cur_slot: int, weight, bias, caches, observed, age_frames,
                  age_observed=None, stream=None):
        """``bjf_front_end_step_ring``: the step on the clip (ring[:, :, prev_slot], ring[:, :, cur_slot])
        of a frame ring [S, C, R, H, W] (frames = tubelet = 2); results as ``step`` on that clip."""
        if age_observed is None:
            age_observed = self.steps > 0
        check(load().bjf_front_end_step_ring(
            ctypes.byref(self.desc), _ptr(ring), int(ring.shape[2]), int(prev_slot), int(cur_slot), _ptr(weight),
            _ptr(bias), _ptr(caches), _ptr(observed), _ptr(age_frames), int(bool(age_observed)),
            _ptr(self.workspace), self.workspace.numel(), _ptr(self.counts), _stream(stream)))
        self.steps += 1
        return self.counts

    def upload_frame(self, host_frame, ring, slot: int, streams=None, stream=None):
        """``bjf_frame_ring_upload``: host_frame [S, C, H, W] (pinned, contiguous) into slot `slot`
        of ring [S, C, R, H, W]; `streams` = (begin, end) uploads part of the streams."""
        if not host_frame.is_contiguous() or host_frame.device.type != "cpu":
            raise ValueError("host_frame must be a contiguous host tensor")
        b, e = (0, int(self.desc.streams)) if streams is None else streams
        check(load().bjf_frame_ring_upload(ctypes.byref(self.desc), ctypes.c_void_p(host_frame.data_ptr()), _ptr(ring),
                                           int(ring.shape[2]), int(slot), int(b), int(e), _stream(stream)))
