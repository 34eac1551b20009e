"""CPU oracle for the burn_jepa sparse front end -- TEST INFRASTRUCTURE ONLY.

A numpy/ctypes face over ``oracle/bjf_oracle.c``, the plain-C restatement of the
reference algorithm (mosure/burn_jepa 0.21.0).  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import it,
and only as the checker or the timed CPU baseline; the product never calls it.

Each wrapper names the reference file:line that the C function restates.  The
restatement is pinned by the known-answer vectors of the reference's own tests
(``tests/golden/reference_known_answers.json``) and, for the Conv3d arithmetic that
lives in the un-vendored crate burn_flex_gmm 0.21.2, by torch ``F.conv3d`` fixtures
(``tests/golden/conv3d_tiny.npz``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libbjf_oracle.so")

_ERRORS = {
    -1: "dense token count must be nonzero",
    -2: "sparse token index outside dense token range",
    -3: "patch-diff sparsity threshold must be finite and non-negative",
    -4: "patch-diff sparsity received unexpected score length",
    -5: "sparse JEPA mode requires at least two dense tokens",
    -6: "patch-diff sparsity requires frames/height/width divisible by tubelet and patch sizes",
    -7: "patch-diff sparsity grid must match the video shape",
    -8: "sparse patchify batch must be nonzero",
    -9: "feature memory sparse assignment requires at least one token",
    -10: "invalid argument",
}


class OracleError(RuntimeError):
    """Raised where the reference returns Err / fails an ensure!."""


def build() -> str:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class PatchDiffConfig(ctypes.Structure):
    """SparseJepaPatchDiffSparsityConfig (src/nodes.rs:97-157)."""

    _fields_ = [
        ("threshold", ctypes.c_float),
        ("context_tokens", ctypes.c_int64),
        ("target_tokens", ctypes.c_int64),
        ("dilation", ctypes.c_int64),
        ("min_context_tokens", ctypes.c_int64),
        ("fill_to_context_tokens", ctypes.c_int32),
        ("allow_full_context", ctypes.c_int32),
    ]

    @classmethod
    def new(cls, threshold, context_tokens, target_tokens):
        """SparseJepaPatchDiffSparsityConfig::new (nodes.rs:109-119)."""
        return cls(threshold, context_tokens, target_tokens, 0, 1, 1, 0)

    @classmethod
    def adaptive_threshold(cls, threshold, min_context_tokens, max_context_tokens, target_tokens):
        """SparseJepaPatchDiffSparsityConfig::adaptive_threshold (nodes.rs:121-136)."""
        return cls(threshold, max_context_tokens, target_tokens, 0, min_context_tokens, 0, 1)

    def with_dilation(self, dilation):
        """SparseJepaPatchDiffSparsityConfig::with_dilation (nodes.rs:138-141)."""
        c = PatchDiffConfig.from_buffer_copy(self)
        c.dilation = dilation
        return c


class PatchifyConfig(ctypes.Structure):
    """burn_flex_gmm::SparsePatchify3dConfig as built at src/model.rs:1297-1306."""

    _fields_ = [
        (n, ctypes.c_int64)
        for n in (
            "in_channels",
            "out_channels",
            "frames",
            "height",
            "width",
            "tubelet_size",
            "patch_h",
            "patch_w",
        )
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def _declare(L):
    L.bjo_token_index_to_coords.argtypes = [_I64] * 4 + [ctypes.POINTER(_I64)] * 3
    L.bjo_token_index_to_coords.restype = None
    L.bjo_coords_to_token_index.argtypes = [_I64] * 6
    L.bjo_coords_to_token_index.restype = _I64
    L.bjo_sparse_token_mask_new.argtypes = [_P, _I64, _I64]
    L.bjo_sparse_token_mask_new.restype = _I64
    L.bjo_from_keep_ratio.argtypes = [_I64, ctypes.c_float, _P]
    L.bjo_from_keep_ratio.restype = _I64
    L.bjo_evenly_spaced_indices.argtypes = [_I64, _I64, _P]
    L.bjo_evenly_spaced_indices.restype = _I64
    L.bjo_complement.argtypes = [_P, _I64, _I64, _P]
    L.bjo_complement.restype = _I64
    L.bjo_padded_to_len.argtypes = [_P, _I64, _I64, _I64, _P]
    L.bjo_padded_to_len.restype = _I64
    L.bjo_target_mask_from_context.argtypes = [_P, _I64, _I64, _I64, _P]
    L.bjo_target_mask_from_context.restype = _I64
    L.bjo_patch_diff_token_scores.argtypes = [_P] + [_I64] * 7 + [_P]
    L.bjo_patch_diff_token_scores.restype = ctypes.c_int
    L.bjo_patch_diff_context_mask_from_scores.argtypes = [_P, _I64, _I64, _I64, _I64, _P, _P, _P]
    L.bjo_patch_diff_context_mask_from_scores.restype = ctypes.c_int
    L.bjo_patch_diff_context_mask.argtypes = [_P] + [_I64] * 10 + [_P, _P, _P]
    L.bjo_patch_diff_context_mask.restype = ctypes.c_int
    L.bjo_sparse_patchify_plan.argtypes = [_P, _I64, _I64, _I64, _I64, _I64, _P]
    L.bjo_sparse_patchify_plan.restype = ctypes.c_int
    L.bjo_sparse_patchify3d_forward.argtypes = [_P, _I64, _P, _P, _I64, _P, _P, _P]
    L.bjo_sparse_patchify3d_forward.restype = ctypes.c_int
    L.bjo_patch_embed3d_dense.argtypes = [_P, _I64, _P, _P, _P, _P]
    L.bjo_patch_embed3d_dense.restype = ctypes.c_int
    L.bjo_feature_memory_assign_latest.argtypes = [_P] * 5 + [_I64] * 4 + [ctypes.c_int32]
    L.bjo_feature_memory_assign_latest.restype = ctypes.c_int
    L.bjo_feature_memory_update_ema.argtypes = [_P] * 5 + [_I64] * 4 + [ctypes.c_float, ctypes.c_int32]
    L.bjo_feature_memory_update_ema.restype = ctypes.c_int
    L.bjo_feature_memory_reset_rows.argtypes = [_P] * 3 + [_I64] * 3 + [_P, _I64]
    L.bjo_feature_memory_reset_rows.restype = ctypes.c_int
    L.bjo_sparse_3d_sincos_pos_embed.argtypes = [_I64] * 4 + [_P, _I64, _P]
    L.bjo_sparse_3d_sincos_pos_embed.restype = None
    L.bjo_patchify_encoder_input.argtypes = [_P, _I64, _P, _P, _I64, _P, _P, _P, _P, _P]
    L.bjo_patchify_encoder_input.restype = ctypes.c_int
    L.bjo_rgba_patch_diff_frame_stats.argtypes = [_P, _I64, _P, _I64, _P]
    L.bjo_rgba_patch_diff_frame_stats.restype = None
    L.bjo_patch_diff_scores_from_rgba.argtypes = [_P, _I64, _P, _I64] + [_I64] * 5 + [_P, _P]
    L.bjo_patch_diff_scores_from_rgba.restype = ctypes.c_int
    L.bjo_patch_diff_dense_fallback.argtypes = [_P, _I64, _I64, ctypes.c_float, _P]
    L.bjo_patch_diff_dense_fallback.restype = _I64
    L.bjo_dilate_sparse_patch_mask.argtypes = [_P] + [_I64] * 5 + [_P]
    L.bjo_dilate_sparse_patch_mask.restype = _I64
    L.bjo_bucket_sparse_mask.argtypes = [_P, _I64, _I64, _I64, _P]
    L.bjo_bucket_sparse_mask.restype = _I64
    L.bjo_front_end_streams.argtypes = [_P, _I64, _P, _P, _P, _P, _P, _P, _P, ctypes.c_int32, _P]
    L.bjo_front_end_streams.restype = ctypes.c_int
    L.bjo_splitmix64.argtypes = [ctypes.c_uint64]
    L.bjo_splitmix64.restype = ctypes.c_uint64
    L.bjo_num_threads.argtypes = []
    L.bjo_num_threads.restype = ctypes.c_int


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(rc: int):
    if rc < 0:
        raise OracleError(_ERRORS.get(int(rc), f"oracle error {rc}"))
    return rc


def num_threads() -> int:
    return int(lib().bjo_num_threads())


# --------------------------------------------------------------------------
# Grid addressing and masks (src/positional.rs, src/tokens.rs)
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class TokenGridShape:
    """src/tokens.rs:5-32."""

    depth: int
    height: int
    width: int

    def __len__(self):
        return self.depth * self.height * self.width

    def tokens_per_frame(self):
        return self.height * self.width


def token_index_to_coords(index: int, grid: TokenGridShape):
    """src/positional.rs:10-17."""
    f, r, c = _I64(), _I64(), _I64()
    lib().bjo_token_index_to_coords(index, grid.depth, grid.height, grid.width,
                                    ctypes.byref(f), ctypes.byref(r), ctypes.byref(c))
    return (f.value, r.value, c.value)


def coords_to_token_index(frame: int, row: int, col: int, grid: TokenGridShape) -> int:
    """src/positional.rs:19-21."""
    return int(lib().bjo_coords_to_token_index(frame, row, col, grid.depth, grid.height, grid.width))


def sparse_token_mask_new(indices, dense_len: int) -> np.ndarray:
    """SparseTokenMask::new (src/tokens.rs:41-50): sorted, deduplicated, range-checked."""
    a = np.ascontiguousarray(np.asarray(indices, dtype=np.int64).copy())
    n = _check(lib().bjo_sparse_token_mask_new(_ptr(a), a.size, dense_len))
    return a[:n].copy()


def from_keep_ratio(dense_len: int, keep_ratio: float) -> np.ndarray:
    """SparseTokenMask::from_keep_ratio (src/tokens.rs:52-59)."""
    out = np.zeros(max(dense_len, 1), dtype=np.int64)
    n = lib().bjo_from_keep_ratio(dense_len, keep_ratio, _ptr(out))
    return out[:n].copy()


def evenly_spaced_indices(dense_len: int, keep: int) -> np.ndarray:
    """SparseTokenMask::evenly_spaced_indices (src/tokens.rs:66-75)."""
    out = np.zeros(max(dense_len, keep, 1), dtype=np.int64)
    n = lib().bjo_evenly_spaced_indices(dense_len, keep, _ptr(out))
    return out[:n].copy()


def complement(indices, dense_len: int) -> np.ndarray:
    """SparseTokenMask::complement (src/tokens.rs:143-157)."""
    a = np.ascontiguousarray(np.asarray(indices, dtype=np.int64))
    out = np.zeros(max(dense_len, 1), dtype=np.int64)
    n = lib().bjo_complement(_ptr(a), a.size, dense_len, _ptr(out))
    return out[:n].copy()


def padded_to_len(indices, dense_len: int, target_len: int) -> np.ndarray:
    """SparseTokenMask::padded_to_len (src/tokens.rs:94-128)."""
    a = np.ascontiguousarray(np.asarray(indices, dtype=np.int64))
    out = np.zeros(max(dense_len, a.size, 1), dtype=np.int64)
    n = _check(lib().bjo_padded_to_len(_ptr(a), a.size, dense_len, target_len, _ptr(out)))
    return out[:n].copy()


def padded_to_multiple(indices, dense_len: int, multiple: int) -> np.ndarray:
    """SparseTokenMask::padded_to_multiple (src/tokens.rs:130-141)."""
    a = np.asarray(indices, dtype=np.int64)
    if multiple <= 1 or a.size >= dense_len:
        return a.copy()
    target = min(-(-a.size // multiple) * multiple, dense_len)
    return padded_to_len(a, dense_len, target)


def target_mask_from_context(context, dense_len: int, target_tokens: int) -> np.ndarray:
    """target_mask_from_context (src/tokens.rs:497-528)."""
    a = np.ascontiguousarray(np.asarray(context, dtype=np.int64))
    out = np.zeros(max(dense_len, 1), dtype=np.int64)
    n = _check(lib().bjo_target_mask_from_context(_ptr(a), a.size, dense_len, target_tokens, _ptr(out)))
    return out[:n].copy()


def make_context_target_masks(grid: TokenGridShape, context_keep_ratio: float):
    """make_context_target_masks (src/tokens.rs:488-495)."""
    context = from_keep_ratio(len(grid), context_keep_ratio)
    return context, complement(context, len(grid))


# --------------------------------------------------------------------------
# Patch-diff mask (src/nodes.rs)
# --------------------------------------------------------------------------
def patch_diff_token_scores(video: np.ndarray, tubelet_size: int, patch_size: int) -> np.ndarray:
    """patch_diff_token_scores (src/nodes.rs:565-631). video [B,C,T,H,W] -> [N] f32."""
    v = np.ascontiguousarray(video, dtype=np.float32)
    B, C, T, H, W = v.shape
    kt, P = max(tubelet_size, 1), max(patch_size, 1)
    out = np.zeros(max((T // kt) * (H // P) * (W // P), 1), dtype=np.float32)
    _check(lib().bjo_patch_diff_token_scores(_ptr(v), B, C, T, H, W, tubelet_size, patch_size, _ptr(out)))
    return out[: (T // kt) * (H // P) * (W // P)].copy()


def patch_diff_context_mask_from_scores(scores, grid: TokenGridShape, config: PatchDiffConfig) -> np.ndarray:
    """patch_diff_context_mask_from_scores (src/nodes.rs:458-537)."""
    s = np.ascontiguousarray(np.asarray(scores, dtype=np.float32))
    out = np.zeros(max(len(grid), 1), dtype=np.int64)
    cnt = _I64()
    _check(lib().bjo_patch_diff_context_mask_from_scores(
        _ptr(s), s.size, grid.depth, grid.height, grid.width, ctypes.byref(config), _ptr(out), ctypes.byref(cnt)))
    return out[: cnt.value].copy()


def patch_diff_context_mask_from_video(video: np.ndarray, tubelet_size: int, patch_size: int,
                                       grid: TokenGridShape, config: PatchDiffConfig) -> np.ndarray:
    """patch_diff_context_mask_from_video (src/nodes.rs:539-546 -> 411-456)."""
    v = np.ascontiguousarray(video, dtype=np.float32)
    B, C, T, H, W = v.shape
    out = np.zeros(max(len(grid), 1), dtype=np.int64)
    cnt = _I64()
    _check(lib().bjo_patch_diff_context_mask(
        _ptr(v), B, C, T, H, W, tubelet_size, patch_size, grid.depth, grid.height, grid.width,
        ctypes.byref(config), _ptr(out), ctypes.byref(cnt)))
    return out[: cnt.value].copy()


# --------------------------------------------------------------------------
# Sparse patchify (src/sparse_patchify.rs, flex-gmm semantics)
# --------------------------------------------------------------------------
def sparse_patchify_plan_coords(mask_indices, grid: TokenGridShape, batch: int) -> np.ndarray:
    """SparsePatchifyPlan::new coords (src/sparse_patchify.rs:236-269) -> [batch*n, 4] int32."""
    m = np.ascontiguousarray(np.asarray(mask_indices, dtype=np.int64))
    out = np.zeros((max(batch, 1) * m.size, 4), dtype=np.int32)
    _check(lib().bjo_sparse_patchify_plan(_ptr(m), m.size, grid.depth, grid.height, grid.width, batch, _ptr(out)))
    return out


def sparse_patchify3d_forward(config: PatchifyConfig, input: np.ndarray, coords: np.ndarray,
                              weight: np.ndarray, bias) -> np.ndarray:
    """flex-gmm sparse_patchify3d_forward semantics (Conv3d at selected tubelets) -> [rows, D]."""
    x = np.ascontiguousarray(input, dtype=np.float32)
    c = np.ascontiguousarray(coords, dtype=np.int32).reshape(-1, 4)
    w = np.ascontiguousarray(weight, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    out = np.zeros((c.shape[0], config.out_channels), dtype=np.float32)
    _check(lib().bjo_sparse_patchify3d_forward(
        ctypes.byref(config), x.shape[0], _ptr(x), _ptr(c), c.shape[0], _ptr(w),
        None if b is None else _ptr(b), _ptr(out)))
    return out


def patch_embed3d_dense(config: PatchifyConfig, input: np.ndarray, weight: np.ndarray, bias) -> np.ndarray:
    """PatchEmbed3d::forward (src/model.rs:88-93) -> [B, N, D]."""
    x = np.ascontiguousarray(input, dtype=np.float32)
    w = np.ascontiguousarray(weight, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    B = x.shape[0]
    n = (config.frames // config.tubelet_size) * (config.height // config.patch_h) * (config.width // config.patch_w)
    out = np.zeros((B, n, config.out_channels), dtype=np.float32)
    _check(lib().bjo_patch_embed3d_dense(ctypes.byref(config), B, _ptr(x), _ptr(w),
                                         None if b is None else _ptr(b), _ptr(out)))
    return out


# --------------------------------------------------------------------------
# Token cache (src/sparse_feature_memory.rs)
# --------------------------------------------------------------------------
def feature_memory_assign_latest(features, observed, age_frames, tokens, token_indices, age_observed: bool):
    """sparse_feature_memory_assign_latest (src/sparse_feature_memory.rs:22-108), in place on
    float32 numpy arrays features [B,N,D], observed/age [B,N]; tokens [B,S,D]; indices [B,S]."""
    for a in (features, observed, age_frames):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    t = np.ascontiguousarray(tokens, dtype=np.float32)
    i = np.ascontiguousarray(token_indices, dtype=np.int32)
    B, N, D = features.shape
    S = i.shape[1]
    _check(lib().bjo_feature_memory_assign_latest(
        _ptr(features), _ptr(observed), _ptr(age_frames), _ptr(t), _ptr(i), B, N, D, S, int(bool(age_observed))))


def feature_memory_update_ema(features, observed, age_frames, tokens, token_indices, alpha: float,
                              age_observed: bool):
    """EMA update mode (src/feature_memory.rs:227-290), in place on float32 numpy arrays."""
    for a in (features, observed, age_frames):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    t = np.ascontiguousarray(tokens, dtype=np.float32)
    i = np.ascontiguousarray(token_indices, dtype=np.int32)
    B, N, D = features.shape
    S = i.shape[1]
    _check(lib().bjo_feature_memory_update_ema(
        _ptr(features), _ptr(observed), _ptr(age_frames), _ptr(t), _ptr(i), B, N, D, S, float(alpha),
        int(bool(age_observed))))


def feature_memory_reset_rows(features, observed, age_frames, rows):
    """reset_rows (src/feature_memory.rs:348-375), in place."""
    for a in (features, observed, age_frames):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    r = np.ascontiguousarray(rows, dtype=np.int32)
    B, N, D = features.shape
    _check(lib().bjo_feature_memory_reset_rows(_ptr(features), _ptr(observed), _ptr(age_frames), B, N, D, _ptr(r),
                                              r.size))


# ---- encoder input (src/positional.rs, src/model.rs) ----
def sparse_3d_sincos_pos_embed(embed_dim: int, grid: "TokenGridShape", indices) -> np.ndarray:
    """sparse_3d_sincos_pos_embed (src/positional.rs:46-67): [len(indices), embed_dim] f32."""
    a = np.ascontiguousarray(np.asarray(indices, dtype=np.int64))
    out = np.zeros((a.size, embed_dim), dtype=np.float32)
    lib().bjo_sparse_3d_sincos_pos_embed(embed_dim, grid.depth, grid.height, grid.width, _ptr(a), a.size, _ptr(out))
    return out


def get_3d_sincos_pos_embed(embed_dim: int, grid: "TokenGridShape") -> np.ndarray:
    """get_3d_sincos_pos_embed (src/positional.rs:42-44): every token of the grid."""
    return sparse_3d_sincos_pos_embed(embed_dim, grid, np.arange(len(grid)))


def patchify_encoder_input(config: PatchifyConfig, input, coords, weight, bias, position_table, modality_embed):
    """Patch embed + position table + modality embedding per row (src/model.rs:690-703), f32."""
    x = np.ascontiguousarray(input, dtype=np.float32)
    c = np.ascontiguousarray(coords, dtype=np.int32)
    w = np.ascontiguousarray(weight, dtype=np.float32)
    rows = c.shape[0]
    out = np.zeros((rows, config.out_channels), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    pt = None if position_table is None else np.ascontiguousarray(position_table, dtype=np.float32)
    me = None if modality_embed is None else np.ascontiguousarray(modality_embed, dtype=np.float32)
    _check(lib().bjo_patchify_encoder_input(ctypes.byref(config), x.shape[0], _ptr(x), _ptr(c), rows, _ptr(w),
                                            None if b is None else _ptr(b), None if pt is None else _ptr(pt),
                                            None if me is None else _ptr(me), _ptr(out)))
    return out


# ---- live viewer policy (src/viewer.rs) ----
class RgbaFrameStats(ctypes.Structure):
    """RgbaPatchDiffFrameStats (src/viewer.rs:1067-1076) plus the means the decision compares."""

    _fields_ = [("channel_delta", ctypes.c_float * 3), ("luma_delta", ctypes.c_float),
                ("compensate_global_lighting", ctypes.c_int32), ("raw_abs", ctypes.c_float),
                ("residual_abs", ctypes.c_float)]


def rgba_patch_diff_frame_stats(prev, current) -> RgbaFrameStats:
    """rgba_patch_diff_frame_stats (src/viewer.rs:1079-1124) over two RGBA u8 buffers."""
    p = np.ascontiguousarray(prev, dtype=np.uint8).ravel()
    c = np.ascontiguousarray(current, dtype=np.uint8).ravel()
    st = RgbaFrameStats()
    lib().bjo_rgba_patch_diff_frame_stats(_ptr(p), p.size, _ptr(c), c.size, ctypes.byref(st))
    return st


def patch_diff_scores_from_rgba(prev, current, width: int, patch_size: int, grid: "TokenGridShape"):
    """patch_diff_scores_from_rgba (src/viewer.rs:1126-1157): scores [grid.len()] f32 and the stats."""
    p = np.ascontiguousarray(prev, dtype=np.uint8).ravel()
    c = np.ascontiguousarray(current, dtype=np.uint8).ravel()
    out = np.zeros(grid.height * grid.width, dtype=np.float32)
    st = RgbaFrameStats()
    _check(lib().bjo_patch_diff_scores_from_rgba(_ptr(p), p.size, _ptr(c), c.size, width, patch_size, grid.depth,
                                                 grid.height, grid.width, _ptr(out), ctypes.byref(st)))
    return out, st


def patch_diff_dense_fallback(indices, dense_len: int, fallback_density: float) -> np.ndarray:
    """patch_diff_dense_fallback (src/viewer.rs:780-793)."""
    a = np.ascontiguousarray(np.asarray(indices, dtype=np.int64))
    out = np.zeros(max(dense_len, a.size, 1), dtype=np.int64)
    n = lib().bjo_patch_diff_dense_fallback(_ptr(a), a.size, dense_len, float(fallback_density), _ptr(out))
    return out[:n].copy()


def dilate_sparse_patch_mask(indices, grid: "TokenGridShape", dilation: int) -> np.ndarray:
    """dilate_sparse_patch_mask (src/viewer.rs:796-816)."""
    a = np.ascontiguousarray(np.asarray(indices, dtype=np.int64))
    out = np.zeros(max(len(grid), a.size, 1), dtype=np.int64)
    n = _check(lib().bjo_dilate_sparse_patch_mask(_ptr(a), a.size, grid.depth, grid.height, grid.width, dilation,
                                                  _ptr(out)))
    return out[:n].copy()


def bucket_sparse_mask(indices, dense_len: int, bucket_tokens: int) -> np.ndarray:
    """bucket_sparse_mask (src/viewer.rs:873-885)."""
    a = np.ascontiguousarray(np.asarray(indices, dtype=np.int64))
    out = np.zeros(max(dense_len, a.size, 1), dtype=np.int64)
    n = lib().bjo_bucket_sparse_mask(_ptr(a), a.size, dense_len, bucket_tokens, _ptr(out))
    return out[:n].copy()


def sparse_mask_bucket_widths(dense_len: int, bucket_tokens: int, bucket_densities=()) -> list:
    """sparse_mask_bucket_widths (src/viewer.rs:887-925) with density_tokens(.., Ceil, 0.0)
    (:739-752): ascending unique encode widths, the grid length last; none below 256 tokens."""
    if dense_len < 256:
        return []
    widths = []
    if len(bucket_densities) == 0:
        if bucket_tokens > 1:
            bucket = min(bucket_tokens, max(dense_len // 4, 1))
            w = bucket
            while w < dense_len:
                widths.append(w)
                w += bucket
    else:
        for d in bucket_densities:
            d = np.float32(d)
            if np.isfinite(d) and d > 0:
                t = int(np.ceil(np.float32(dense_len) * np.float32(min(d, np.float32(1.0)))))
                widths.append(min(max(t, 1), max(dense_len, 1)))
    widths.append(dense_len)
    return sorted(set(widths))


def finalize_patch_diff_encode_masks(write, dense_len: int, bucketed: bool, bucket_tokens: int,
                                     bucket_densities=()) -> np.ndarray:
    """The encode mask of finalize_patch_diff_encode_masks (src/viewer.rs:946-961):
    Exact -> the write mask; BucketedContext -> bucket_sparse_mask_with_config (:927-944)."""
    write = np.asarray(write, dtype=np.int64)
    if not bucketed or dense_len < 256 or write.size == dense_len:
        return write.copy()
    for w in sparse_mask_bucket_widths(dense_len, bucket_tokens, bucket_densities):
        if w >= write.size:
            return padded_to_len(write, dense_len, w)
    return write.copy()


def viewer_patch_diff_masks(direct, grid: "TokenGridShape", dense_fallback_density: float, dilation: int,
                            bucketed: bool = True, bucket_tokens: int = 256,
                            bucket_densities=(0.10, 0.25, 0.50)):
    """patch_diff_base_mask_from_scores after its selection (src/viewer.rs:826-828) and
    finalize_patch_diff_encode_masks (:946-961): direct mask -> (write mask, encode mask)."""
    n = len(grid)
    m = patch_diff_dense_fallback(direct, n, dense_fallback_density)
    write = dilate_sparse_patch_mask(m, grid, dilation)
    return write, finalize_patch_diff_encode_masks(write, n, bucketed, bucket_tokens, bucket_densities)


def viewer_patch_diff_masks_from_scores(scores, grid: "TokenGridShape", config: "PatchDiffConfig",
                                        dense_fallback_density: float, bucketed: bool = True,
                                        bucket_tokens: int = 256, bucket_densities=(0.10, 0.25, 0.50)):
    """patch_diff_masks_from_scores (src/viewer.rs:831-841): the selection without dilation
    (:819-825), then the viewer policy dilating by the config's dilation."""
    direct = patch_diff_context_mask_from_scores(scores, grid, config.with_dilation(0))
    return viewer_patch_diff_masks(direct, grid, dense_fallback_density, config.dilation, bucketed, bucket_tokens,
                                   bucket_densities)


def patch_diff_can_use_dense_fast_path(config: "PatchDiffConfig", dense_len: int) -> bool:
    """patch_diff_can_use_dense_fast_path (src/viewer.rs:1031-1036)."""
    return config.threshold <= 0.0 and bool(config.allow_full_context) and config.context_tokens >= dense_len


def patch_diff_sampled_dense_fast_path_from_rgba(prev, current, width: int, patch_size: int, grid: "TokenGridShape",
                                                 config: "PatchDiffConfig", fallback_density: float) -> bool:
    """patch_diff_sampled_dense_fast_path_from_rgba (src/viewer.rs:1160-1195): the lighting
    statistics of the whole frames, then rgba_patch_diff_score on every stride-th patch row and
    column (each the same per-patch score as patch_diff_scores_from_rgba's)."""
    fb = np.float32(fallback_density)
    if not np.isnan(fb):
        fb = np.float32(min(max(fb, np.float32(0.0)), np.float32(1.0)))
    if fb >= 1.0 or config.threshold <= 0.0 or not config.allow_full_context or config.context_tokens < len(grid):
        return False
    scores, _ = patch_diff_scores_from_rgba(prev, current, width, patch_size, grid)
    stride = max(int(np.ceil(np.sqrt(np.float32(len(grid)) / np.float32(64.0)))), 1)
    sampled = active = 0
    for row in range(0, grid.height, stride):
        for col in range(0, grid.width, stride):
            sampled += 1
            active += bool(scores[row * grid.width + col] >= np.float32(config.threshold))
    required = 0 if np.isnan(fb) else int(np.ceil(np.float32(sampled) * fb))
    return sampled > 0 and active >= max(required, 1)


def viewer_patch_diff_masks_from_rgba(prev, current, width: int, patch_size: int, grid: "TokenGridShape",
                                      config: "PatchDiffConfig", dense_fallback_density: float,
                                      bucketed: bool = True, bucket_tokens: int = 256,
                                      bucket_densities=(0.10, 0.25, 0.50)):
    """patch_diff_mask_from_rgba without refresh state (crates/bevy_jepa/src/mask.rs:126-175):
    (write mask, encode mask)."""
    n = len(grid)
    if patch_diff_can_use_dense_fast_path(config, n) or patch_diff_sampled_dense_fast_path_from_rgba(
            prev, current, width, patch_size, grid, config, dense_fallback_density):
        all_ = np.arange(n, dtype=np.int64)
        return all_, all_.copy()
    scores, _ = patch_diff_scores_from_rgba(prev, current, width, patch_size, grid)
    return viewer_patch_diff_masks_from_scores(scores, grid, config, dense_fallback_density, bucketed, bucket_tokens,
                                               bucket_densities)


def density_tokens(dense_tokens: int, density: float, rounding: str, min_density: float) -> int:
    """density_tokens (src/viewer.rs:739-752) with f32 arithmetic; rounding in floor/round/ceil."""
    d = np.float32(density)
    d = np.float32(min(max(d, np.float32(min_density)), np.float32(1.0))) if not np.isnan(d) else d
    x = np.float32(dense_tokens) * d
    r = {"floor": np.floor, "ceil": np.ceil}.get(rounding)
    v = r(x) if r else np.float32(np.sign(x) * np.floor(np.abs(x) + np.float32(0.5)))  # half away from zero
    t = int(v) if np.isfinite(v) and v > 0 else 0
    return min(max(t, 1), max(dense_tokens, 1))


def patch_diff_sparsity_config(context_density: float, min_context_density: float, threshold: float,
                               dilation: int, grid: "TokenGridShape") -> "PatchDiffConfig":
    """patch_diff_sparsity_config (src/viewer.rs:1012-1028) for the viewer fields it reads."""
    n = len(grid)
    max_ctx = density_tokens(n, context_density, "round", 0.01)
    min_ctx = min(density_tokens(n, min_context_density, "ceil", 0.0), max_ctx)
    target = max(n - max_ctx, 1)
    return PatchDiffConfig.adaptive_threshold(threshold, min_ctx, max_ctx, target).with_dilation(dilation)


def _mix64(v: int) -> int:
    """mix64 (src/viewer.rs:530-536)."""
    m = (1 << 64) - 1
    v ^= v >> 30
    v = (v * 0xBF58476D1CE4E5B9) & m
    v ^= v >> 27
    v = (v * 0x94D049BB133111EB) & m
    return v ^ (v >> 31)


class PatchDiffRefreshState:
    """PatchDiffRefreshState (src/viewer.rs:272-528) over host scores; `refresh` is a dict of the
    PatchDiffRefreshConfig fields (src/viewer.rs:186-241)."""

    DEFAULTS = dict(enabled=False, subthreshold_enabled=False, subthreshold_decay=0.92, subthreshold_gain=1.0,
                    subthreshold_trigger=1.0, subthreshold_max_density=0.04, age_refresh_enabled=False,
                    age_refresh_interval_frames=90, age_refresh_max_density=0.01, blue_noise_enabled=False,
                    blue_noise_refresh_density=0.005, blue_noise_seed=0x9E3779B97F4A7C15, max_extra_density=0.05)

    def __init__(self):
        self.dense_len = 0
        self.frame_index = 0
        self.residual = np.zeros(0, np.float32)
        self.age = np.zeros(0, np.uint32)

    @staticmethod
    def can_add_tokens(c) -> bool:
        return (c["enabled"] and c["max_extra_density"] > 0.0
                and ((c["subthreshold_enabled"] and c["subthreshold_max_density"] > 0.0)
                     or (c["age_refresh_enabled"] and c["age_refresh_interval_frames"] > 0
                         and c["age_refresh_max_density"] > 0.0)
                     or (c["blue_noise_enabled"] and c["blue_noise_refresh_density"] > 0.0)))

    def _begin_frame(self, n):
        if self.dense_len != n:
            self.dense_len, self.frame_index = n, 0
            self.residual = np.zeros(n, np.float32)
            self.age = np.zeros(n, np.uint32)
        self.frame_index = min(self.frame_index + 1, (1 << 64) - 1)  # saturating_add
        self.age = np.minimum(self.age.astype(np.uint64) + 1, 0xFFFFFFFF).astype(np.uint32)

    def _reset_selected(self, idx):
        idx = np.asarray(idx, dtype=np.int64)
        self.residual[idx] = 0.0
        self.age[idx] = 0

    def _rank(self, index, grid, seed):
        m = (1 << 64) - 1
        w = max(grid.width, 1)
        row, col = index // w, index % w
        return _mix64(seed ^ ((row * 0x9E3779B97F4A7C15) & m) ^ ((col * 0xBF58476D1CE4E5B9) & m)
                      ^ ((self.frame_index * 0x94D049BB133111EB) & m))

    def _update_residual(self, scores, chosen, threshold, c):
        sel = np.zeros(len(scores), bool)
        sel[np.asarray(chosen, dtype=np.int64)] = True
        decay = np.float32(min(max(c["subthreshold_decay"], 0.0), 1.0))
        th = np.float32(max(np.float32(threshold), np.float32(1e-6)))
        gain = np.float32(max(c["subthreshold_gain"], 0.0))
        for i in range(len(scores)):
            if sel[i] or scores[i] >= np.float32(threshold):
                self.residual[i] = 0.0
            else:
                norm = np.float32(min(max(scores[i] / th, np.float32(0.0)), np.float32(1.0)))
                self.residual[i] = np.float32(np.float32(self.residual[i] * decay) + np.float32(norm * gain))

    def _add_ranked(self, selected, indices, budget, rank):
        if budget == 0:
            return 0
        cands = []
        for i in range(len(selected)):
            if not selected[i]:
                r = rank(i)
                if r is not None:
                    cands.append((i, r[0], r[1]))
        cands.sort(key=lambda t: (-t[1], t[2], t[0]))
        cands = cands[:budget]
        for i, _, _ in cands:
            selected[i] = True
            indices.append(i)
        return len(cands)

    def _augment(self, base, scores, grid, config, c):
        n = len(grid)
        if len(base) >= n:
            return base
        remaining = max(min(max(config.context_tokens, 1), n) - len(base), 0)
        remaining = min(remaining, density_tokens(n, c["max_extra_density"], "floor", 0.0))
        if remaining == 0:
            self._update_residual(scores, base, config.threshold, c)
            return base
        selected = np.zeros(n, bool)
        indices = [int(i) for i in base]
        selected[np.asarray(indices, dtype=np.int64)] = True
        self._update_residual(scores, indices, config.threshold, c)
        seed = c["blue_noise_seed"]
        if c["subthreshold_enabled"] and c["subthreshold_max_density"] > 0.0:
            budget = min(remaining, density_tokens(n, c["subthreshold_max_density"], "floor", 0.0))
            trig = max(np.float32(c["subthreshold_trigger"]), np.float32(1e-6))
            remaining -= self._add_ranked(selected, indices, budget, lambda i: (float(self.residual[i]),
                                          self._rank(i, grid, seed)) if self.residual[i] >= trig else None)
        if (remaining > 0 and c["age_refresh_enabled"] and c["age_refresh_interval_frames"] > 0
                and c["age_refresh_max_density"] > 0.0):
            interval = min(c["age_refresh_interval_frames"], 0xFFFFFFFF)
            budget = min(remaining, density_tokens(n, c["age_refresh_max_density"], "floor", 0.0))
            # the priority is `age as f32` (src/viewer.rs:436): ages round to the nearest f32
            remaining -= self._add_ranked(selected, indices, budget, lambda i: (float(np.float32(self.age[i])),
                                          self._rank(i, grid, seed)) if self.age[i] >= interval else None)
        if remaining > 0 and c["blue_noise_enabled"] and c["blue_noise_refresh_density"] > 0.0:
            budget = min(remaining, density_tokens(n, c["blue_noise_refresh_density"], "floor", 0.0))
            self._add_ranked(selected, indices, budget, lambda i: (0.0, self._rank(i, grid, seed)))
        return sparse_token_mask_new(indices, n)

    def observe_write_mask(self, mask, n: int):
        """observe_write_mask (src/viewer.rs:309-313)."""
        self._begin_frame(n)
        self._reset_selected(np.asarray(mask, dtype=np.int64))

    def masks_from_scores(self, scores, grid, config, dense_fallback_density, refresh, bucketed=True,
                          bucket_tokens=256, bucket_densities=(0.10, 0.25, 0.50)):
        """masks_from_scores (src/viewer.rs:312-347): (write mask, encode mask)."""
        c = dict(self.DEFAULTS, **refresh)
        scores = np.asarray(scores, dtype=np.float32)
        n = len(grid)
        if scores.size != n:
            raise OracleError("patch-diff refresh received unexpected score length")
        direct = patch_diff_context_mask_from_scores(scores, grid, config.with_dilation(0))
        base = dilate_sparse_patch_mask(patch_diff_dense_fallback(direct, n, dense_fallback_density), grid,
                                        config.dilation)
        self._begin_frame(n)
        if self.can_add_tokens(c) and not (len(base) == n):
            base = self._augment(base, scores, grid, config, c)
        enc = finalize_patch_diff_encode_masks(base, n, bucketed, bucket_tokens, bucket_densities)
        self._reset_selected(base)
        return np.asarray(base, dtype=np.int64), enc


def viewer_patch_diff_refresh_masks_from_rgba(state: "PatchDiffRefreshState", prev, current, width: int,
                                              patch_size: int, grid: "TokenGridShape", config: "PatchDiffConfig",
                                              dense_fallback_density: float, refresh, bucketed: bool = True,
                                              bucket_tokens: int = 256, bucket_densities=(0.10, 0.25, 0.50)):
    """patch_diff_mask_from_rgba with a refresh state (crates/bevy_jepa/src/mask.rs:126-185):
    a dense shortcut is observe_write_mask of every token, else masks_from_scores."""
    n = len(grid)
    if patch_diff_can_use_dense_fast_path(config, n) or patch_diff_sampled_dense_fast_path_from_rgba(
            prev, current, width, patch_size, grid, config, dense_fallback_density):
        all_ = np.arange(n, dtype=np.int64)
        state.observe_write_mask(all_, n)
        return all_, all_.copy()
    scores, _ = patch_diff_scores_from_rgba(prev, current, width, patch_size, grid)
    return state.masks_from_scores(scores, grid, config, dense_fallback_density, refresh, bucketed, bucket_tokens,
                                   bucket_densities)


def front_end_streams(video, config: PatchifyConfig, mask_config: PatchDiffConfig, weight, bias,
                      caches, observed, age_frames, age_observed: bool) -> np.ndarray:
    """One front-end step over S independent streams (f32), in place on the caches."""
    v = np.ascontiguousarray(video, dtype=np.float32)
    w = np.ascontiguousarray(weight, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    for a in (caches, observed, age_frames):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    S = v.shape[0]
    counts = np.zeros(S, dtype=np.int64)
    _check(lib().bjo_front_end_streams(
        _ptr(v), S, ctypes.byref(config), ctypes.byref(mask_config), _ptr(w),
        None if b is None else _ptr(b), _ptr(caches), _ptr(observed), _ptr(age_frames),
        int(bool(age_observed)), _ptr(counts)))
    return counts


def splitmix64(value: int) -> int:
    """training/mask.rs:557-563."""
    return int(lib().bjo_splitmix64(ctypes.c_uint64(value & 0xFFFFFFFFFFFFFFFF)))
