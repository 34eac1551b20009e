"""ctypes binding of ``libbjf.so`` (the C ABI declared in ``include/bjf.h``).

The library is built in-tree by ``burn_jepa_b200/build.py`` (nvcc, sm_100a).  Loading
fails loudly when it is missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
import re

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libbjf.so")
HEADER_PATH = os.path.join(os.path.dirname(_PKG), "include", "bjf.h")

BJF_OK = 0
BJF_ERR_INVALID_ARGUMENT = -1
BJF_ERR_UNSUPPORTED = -2
BJF_ERR_CUDA = 1

DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_I32 = 0, 1, 2, 3


class BjfError(RuntimeError):
    """A non-zero status from the C ABI, carrying the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class PatchifyConfig(ctypes.Structure):
    """bjf_patchify_config == burn_flex_gmm::SparsePatchify3dConfig (src/model.rs:1297-1306)."""

    _fields_ = [
        (n, ctypes.c_int64)
        for n in ("in_channels", "out_channels", "frames", "height", "width", "tubelet_size", "patch_h", "patch_w")
    ]


class PatchDiffConfig(ctypes.Structure):
    """bjf_patch_diff_config == SparseJepaPatchDiffSparsityConfig (src/nodes.rs:97-157)."""

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
    def new(cls, threshold: float, context_tokens: int, target_tokens: int) -> "PatchDiffConfig":
        """SparseJepaPatchDiffSparsityConfig::new (src/nodes.rs:109-119)."""
        return cls(threshold, context_tokens, target_tokens, 0, 1, 1, 0)

    @classmethod
    def adaptive_threshold(cls, threshold: float, min_context_tokens: int, max_context_tokens: int,
                           target_tokens: int) -> "PatchDiffConfig":
        """SparseJepaPatchDiffSparsityConfig::adaptive_threshold (src/nodes.rs:121-136)."""
        return cls(threshold, max_context_tokens, target_tokens, 0, min_context_tokens, 0, 1)

    def with_dilation(self, dilation: int) -> "PatchDiffConfig":
        c = PatchDiffConfig.from_buffer_copy(self)
        c.dilation = dilation
        return c

    def with_min_context_tokens(self, n: int) -> "PatchDiffConfig":
        c = PatchDiffConfig.from_buffer_copy(self)
        c.min_context_tokens = n
        return c

    def with_fill_to_context_tokens(self, v: bool) -> "PatchDiffConfig":
        c = PatchDiffConfig.from_buffer_copy(self)
        c.fill_to_context_tokens = int(bool(v))
        return c

    def with_allow_full_context(self, v: bool) -> "PatchDiffConfig":
        c = PatchDiffConfig.from_buffer_copy(self)
        c.allow_full_context = int(bool(v))
        return c


class FrontEndDesc(ctypes.Structure):
    """bjf_front_end_desc: S independent streams, each video [C, T, H, W] with batch 1."""

    _fields_ = [
        ("streams", ctypes.c_int64),
        ("channels", ctypes.c_int64),
        ("frames", ctypes.c_int64),
        ("height", ctypes.c_int64),
        ("width", ctypes.c_int64),
        ("tubelet_size", ctypes.c_int64),
        ("patch_size", ctypes.c_int64),
        ("embed_dim", ctypes.c_int64),
        ("video_dtype", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("cache_dtype", ctypes.c_int32),
        ("mask", PatchDiffConfig),
    ]


class RgbaFrameStats(ctypes.Structure):
    """bjf_rgba_frame_stats: RgbaPatchDiffFrameStats (src/viewer.rs:1067-1076) plus the two means."""

    _fields_ = [
        ("channel_delta", ctypes.c_float * 3),
        ("luma_delta", ctypes.c_float),
        ("compensate_global_lighting", ctypes.c_int32),
        ("raw_abs", ctypes.c_float),
        ("residual_abs", ctypes.c_float),
    ]


class ViewerMaskPolicy(ctypes.Structure):
    """bjf_viewer_mask_policy: the mask fields of FeatureFrameViewerConfig (src/viewer.rs:566-579)."""

    _fields_ = [
        ("dense_fallback_density", ctypes.c_float),
        ("dilation", ctypes.c_int64),
        ("bucketed_encode", ctypes.c_int32),
        ("bucket_tokens", ctypes.c_int64),
        ("bucket_density_count", ctypes.c_int32),
        ("bucket_densities", ctypes.c_float * 32),
    ]

    @classmethod
    def new(cls, dense_fallback_density: float = 0.75, dilation: int = 1, bucketed_encode: bool = True,
            bucket_tokens: int = 256, bucket_densities=(0.10, 0.25, 0.50)) -> "ViewerMaskPolicy":
        """Defaults are FeatureFrameViewerConfig::default()'s (src/viewer.rs:27-33, 604-616)."""
        d = list(bucket_densities)
        if len(d) > 32:
            raise ValueError("at most 32 bucket densities")
        p = cls(float(dense_fallback_density), int(dilation), int(bool(bucketed_encode)), int(bucket_tokens), len(d))
        for i, v in enumerate(d):
            p.bucket_densities[i] = float(v)
        return p


class PatchDiffRefreshConfig(ctypes.Structure):
    """bjf_patch_diff_refresh_config: PatchDiffRefreshConfig (src/viewer.rs:186-270)."""

    _fields_ = [
        ("enabled", ctypes.c_int32),
        ("subthreshold_enabled", ctypes.c_int32),
        ("subthreshold_decay", ctypes.c_float),
        ("subthreshold_gain", ctypes.c_float),
        ("subthreshold_trigger", ctypes.c_float),
        ("subthreshold_max_density", ctypes.c_float),
        ("age_refresh_enabled", ctypes.c_int32),
        ("age_refresh_interval_frames", ctypes.c_uint64),
        ("age_refresh_max_density", ctypes.c_float),
        ("blue_noise_enabled", ctypes.c_int32),
        ("blue_noise_refresh_density", ctypes.c_float),
        ("blue_noise_seed", ctypes.c_uint64),
        ("max_extra_density", ctypes.c_float),
    ]

    # the reference's defaults (src/viewer.rs:35-49, 243-256)
    DEFAULTS = dict(enabled=False, subthreshold_enabled=False, subthreshold_decay=0.92, subthreshold_gain=1.0,
                    subthreshold_trigger=1.0, subthreshold_max_density=0.04, age_refresh_enabled=False,
                    age_refresh_interval_frames=90, age_refresh_max_density=0.01, blue_noise_enabled=False,
                    blue_noise_refresh_density=0.005, blue_noise_seed=0x9E3779B97F4A7C15, max_extra_density=0.05)

    @classmethod
    def from_fields(cls, **fields) -> "PatchDiffRefreshConfig":
        unknown = set(fields) - set(cls.DEFAULTS)
        if unknown:
            raise TypeError(f"unknown refresh config fields: {sorted(unknown)}")
        c = dict(cls.DEFAULTS, **fields)
        return cls(**{k: (int(bool(v)) if k.endswith("enabled") else v) for k, v in c.items()})


class PatchDiffRefreshState(ctypes.Structure):
    """bjf_patch_diff_refresh_state: device pointers to a PatchDiffRefreshState of S streams."""

    _fields_ = [
        ("subthreshold_residual", ctypes.c_void_p),
        ("age_frames", ctypes.c_void_p),
        ("frame_index", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_DIMS = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes)
SIGNATURES = {
    "bjf_abi_version": (ctypes.c_int32, []),
    "bjf_get_last_error_string": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "bjf_device_error_check": (_I32, [_P, ctypes.POINTER(_I32)]),
    "bjf_set_bounded_wait": (_I32, [ctypes.c_uint64, _I32]),
    "bjf_patch_diff_token_scores": (_I32, [_P, _I32, _DIMS, _I64, _I64, _I64, _P, _P]),
    "bjf_patch_diff_context_mask_from_scores": (_I32, [_P, _I64, _DIMS, ctypes.POINTER(PatchDiffConfig), _P, _P, _P]),
    "bjf_patch_diff_context_mask": (_I32, [_P, _I32, _DIMS, _I64, _I64, _I64, _DIMS,
                                           ctypes.POINTER(PatchDiffConfig), _P, _P, _P, _P]),
    "bjf_sparse_patchify_plan_coords": (_I32, [_P, _I64, _P, _I64, _I64, _DIMS, _P, _I64, _P, _P]),
    "bjf_sparse_patchify3d_forward": (_I32, [ctypes.POINTER(PatchifyConfig), _P, _I32, _DIMS, _P, _I64, _P, _I32,
                                             _DIMS, _P, _P, _I32, _P]),
    "bjf_front_end_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(FrontEndDesc)]),
    "bjf_front_end_step": (_I32, [ctypes.POINTER(FrontEndDesc), _P, _P, _P, _P, _P, _P, _I32, _P, ctypes.c_size_t,
                                  _P, _P]),
    "bjf_front_end_step_no_alloc": (_I32, [ctypes.POINTER(FrontEndDesc), _P, _P, _P, _P, _P, _P, _I32, _P, _P]),
    "bjf_front_end_step_ring": (_I32, [ctypes.POINTER(FrontEndDesc), _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _I32,
                                       _P, ctypes.c_size_t, _P, _P]),
    "bjf_frame_ring_upload": (_I32, [ctypes.POINTER(FrontEndDesc), _P, _P, _I32, _I32, _I64, _I64, _P]),
    "bjf_rgba_patch_diff_workspace_bytes": (ctypes.c_size_t, [_I64, _DIMS]),
    "bjf_viewer_rgba_masks_workspace_bytes": (ctypes.c_size_t, [_I64, _DIMS]),
    "bjf_viewer_patch_diff_masks_from_rgba": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _DIMS,
                                                      ctypes.POINTER(PatchDiffConfig), ctypes.POINTER(ViewerMaskPolicy),
                                                      _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "bjf_viewer_patch_diff_masks": (_I32, [_P, _P, _I64, _DIMS, ctypes.POINTER(ViewerMaskPolicy), _P, _P, _P, _P, _P]),
    "bjf_viewer_patch_diff_masks_from_scores": (_I32, [_P, _I64, _DIMS, ctypes.POINTER(PatchDiffConfig),
                                                        ctypes.POINTER(ViewerMaskPolicy), _P, _P, _P, _P, _P]),
    "bjf_viewer_patch_diff_refresh_masks_from_scores": (_I32, [_P, _I64, _DIMS, ctypes.POINTER(PatchDiffConfig),
                                                                ctypes.POINTER(ViewerMaskPolicy),
                                                                ctypes.POINTER(PatchDiffRefreshConfig),
                                                                ctypes.POINTER(PatchDiffRefreshState),
                                                                _P, _P, _P, _P, _P]),
    "bjf_viewer_patch_diff_refresh_masks_from_rgba": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _DIMS,
                                                              ctypes.POINTER(PatchDiffConfig),
                                                              ctypes.POINTER(ViewerMaskPolicy),
                                                              ctypes.POINTER(PatchDiffRefreshConfig),
                                                              ctypes.POINTER(PatchDiffRefreshState),
                                                              _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "bjf_viewer_patch_diff_refresh_observe": (_I32, [_P, _P, _I64, _DIMS, ctypes.POINTER(PatchDiffRefreshState),
                                                      _P]),
    "bjf_sparse_patchify3d_forward_encoder_input": (_I32, [ctypes.POINTER(PatchifyConfig), _P, _I32, _DIMS, _P, _I64,
                                                           _P, _I32, _DIMS, _P, _P, _P, _P, _I32, _P]),
    "bjf_rgba_patch_diff_scores": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _DIMS, _P, _P, _P, ctypes.c_size_t, _P]),
    "bjf_feature_memory_assign_latest": (_I32, [_P, _I32, _DIMS, _P, _DIMS, _P, _DIMS, _P, _I32, _DIMS, _P, _DIMS,
                                                _I32, _P]),
    "bjf_feature_memory_update_ema": (_I32, [_P, _I32, _DIMS, _P, _DIMS, _P, _DIMS, _P, _I32, _DIMS, _P, _DIMS,
                                             ctypes.c_float, _I32, _P]),
    "bjf_feature_memory_reset_rows": (_I32, [_P, _I32, _DIMS, _P, _P, _P, _I64, _P]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every function ``include/bjf.h`` declares."""
    text = open(HEADER_PATH).read()
    return sorted(set(re.findall(r"BJF_API\s+[\w\s\*]+?\b(bjf_\w+)\s*\(", text)))


def header_abi_version() -> int:
    """BJF_ABI_VERSION as ``include/bjf.h`` defines it."""
    return int(re.search(r"#define\s+BJF_ABI_VERSION\s+(\d+)", open(HEADER_PATH).read()).group(1))


def load() -> ctypes.CDLL:
    """Loads libbjf.so (raises if it has not been built, or was built from another ABI version
    of include/bjf.h)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        built, want = lib.bjf_abi_version(), header_abi_version()
        if built != want:
            raise RuntimeError(f"{LIB_PATH} has ABI version {built} but include/bjf.h declares {want}: rebuild it")
        _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().bjf_get_last_error_string(buf, len(buf))
    return buf.value.decode()


def check(status: int) -> None:
    if status != BJF_OK:
        raise BjfError(status, last_error())


def dims(*values) -> ctypes.Array:
    arr = (ctypes.c_int64 * len(values))(*[int(v) for v in values])
    return arr
