"""C ABI checks that need no GPU: the library loads, exports every symbol include/bjf.h
declares, and rejects invalid arguments on the host with the reference's messages
before anything is launched."""
import ctypes

import pytest

import burn_jepa_b200 as bj
from burn_jepa_b200 import _abi

FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: every call below fails validation first


def test_library_exports_every_header_symbol():
    lib = bj.load()
    declared = _abi.header_symbols()
    assert declared, "no declarations parsed from include/bjf.h"
    for name in declared:
        assert hasattr(lib, name), f"libbjf.so does not export {name}"
    assert set(declared) == set(_abi.SIGNATURES), "ctypes signatures out of sync with include/bjf.h"


def test_abi_version():
    assert bj.load().bjf_abi_version() == _abi.header_abi_version() == 4


def _fm(features, observed, age, tokens, indices):
    return bj.load().bjf_feature_memory_assign_latest(
        FAKE, _abi.DTYPE_F32, _abi.dims(*features), FAKE, _abi.dims(*observed), FAKE, _abi.dims(*age), FAKE,
        _abi.DTYPE_F32, _abi.dims(*tokens), FAKE, _abi.dims(*indices), 0, None)


def test_feature_memory_shape_errors_mirror_reference_messages():
    from helpers import known_answers

    ka = known_answers()["feature_memory_shape_errors"]
    c = ka["index_shape_mismatch"]
    assert _fm(c["features"], c["features"][:2], c["features"][:2], c["tokens"], c["indices"]) == -1
    assert c["message_contains"] in bj.last_error()
    assert bj.last_error() == "feature memory index dims mismatch: indices=[1,2] expected=[1,1]"
    c = ka["sparse_len_zero"]
    assert _fm(c["features"], c["features"][:2], c["features"][:2], c["tokens"], c["indices"]) == -1
    assert bj.last_error() == c["message"]
    c = ka["metadata_mismatch"]
    assert _fm(c["features"], c["observed"], c["age"], [1, 1, 2], [1, 1]) == -1
    assert bj.last_error() == ("feature memory metadata dims mismatch: features=[1,4,2] observed=[1,3] "
                               "age=[1,4]")
    c = ka["token_dim_mismatch"]
    assert _fm(c["features"], c["features"][:2], c["features"][:2], c["tokens"], c["indices"]) == -1
    assert bj.last_error() == "feature memory token dims mismatch: tokens=[1,1,3] expected=[1,sparse,2]"


@pytest.mark.parametrize("threshold", [float("nan"), -1.0, float("inf")])
def test_patch_diff_threshold_rejected(threshold):
    cfg = bj.PatchDiffConfig.new(threshold, 1, 2)
    rc = bj.load().bjf_patch_diff_context_mask_from_scores(FAKE, 1, _abi.dims(2, 2, 2), ctypes.byref(cfg), FAKE,
                                                           FAKE, None)
    assert rc == -1 and bj.last_error() == "patch-diff sparsity threshold must be finite and non-negative"
    rc = bj.load().bjf_patch_diff_context_mask(FAKE, _abi.DTYPE_F32, _abi.dims(1, 3, 4, 32, 32), 1, 2, 16,
                                               _abi.dims(2, 2, 2), ctypes.byref(cfg), FAKE, FAKE, FAKE, None)
    assert rc == -1 and bj.last_error() == "patch-diff sparsity threshold must be finite and non-negative"


def test_patch_diff_video_shape_errors():
    cfg = bj.PatchDiffConfig.new(0.1, 1, 2)
    L = bj.load()
    rc = L.bjf_patch_diff_context_mask(FAKE, _abi.DTYPE_F32, _abi.dims(1, 3, 4, 30, 32), 1, 2, 16,
                                       _abi.dims(2, 2, 2), ctypes.byref(cfg), FAKE, FAKE, FAKE, None)
    assert rc == -1
    assert bj.last_error() == ("patch-diff sparsity requires frames/height/width divisible by tubelet and "
                               "patch sizes")
    rc = L.bjf_patch_diff_context_mask(FAKE, _abi.DTYPE_F32, _abi.dims(1, 3, 4, 32, 32), 1, 2, 16,
                                       _abi.dims(2, 1, 2), ctypes.byref(cfg), FAKE, FAKE, FAKE, None)
    assert rc == -1 and bj.last_error() == "patch-diff sparsity grid must match the video shape"
    # a one-token grid has no context budget (nodes.rs:379-385)
    rc = L.bjf_patch_diff_context_mask_from_scores(FAKE, 1, _abi.dims(1, 1, 1), ctypes.byref(cfg), FAKE, FAKE, None)
    assert rc == -1 and bj.last_error() == "sparse JEPA mode requires at least two dense tokens"


def test_patchify_config_errors():
    L = bj.load()
    cfg = bj.PatchifyConfig(3, 32, 4, 32, 32, 2, 16, 16)
    rc = L.bjf_sparse_patchify3d_forward(ctypes.byref(cfg), FAKE, _abi.DTYPE_F32, _abi.dims(1, 3, 4, 32, 16), FAKE,
                                         4, FAKE, _abi.DTYPE_F32, _abi.dims(32, 3, 2, 16, 16), None, FAKE,
                                         _abi.DTYPE_F32, None)
    assert rc == -1 and "input dims [1,3,4,32,16] do not match the config" in bj.last_error()
    rc = L.bjf_sparse_patchify3d_forward(ctypes.byref(cfg), FAKE, _abi.DTYPE_F32, _abi.dims(1, 3, 4, 32, 32), FAKE,
                                         4, FAKE, _abi.DTYPE_F32, _abi.dims(32, 3, 1, 16, 16), None, FAKE,
                                         _abi.DTYPE_F32, None)
    assert rc == -1 and "weight dims [32,3,1,16,16] do not match the config" in bj.last_error()
    bad = bj.PatchifyConfig(3, 32, 4, 32, 32, 0, 16, 16)
    rc = L.bjf_sparse_patchify3d_forward(ctypes.byref(bad), FAKE, _abi.DTYPE_F32, _abi.dims(1, 3, 4, 32, 32), FAKE,
                                         4, FAKE, _abi.DTYPE_F32, _abi.dims(32, 3, 0, 16, 16), None, FAKE,
                                         _abi.DTYPE_F32, None)
    assert rc == -1 and "must be positive" in bj.last_error()
    # zero rows is a valid no-op and launches nothing
    rc = L.bjf_sparse_patchify3d_forward(ctypes.byref(cfg), FAKE, _abi.DTYPE_F32, _abi.dims(1, 3, 4, 32, 32), FAKE,
                                         0, FAKE, _abi.DTYPE_F32, _abi.dims(32, 3, 2, 16, 16), None, FAKE,
                                         _abi.DTYPE_F32, None)
    assert rc == 0


def test_plan_errors():
    L = bj.load()
    rc = L.bjf_sparse_patchify_plan_coords(FAKE, 3, None, 1, 0, _abi.dims(2, 3, 4), FAKE, 6, None, None)
    assert rc == -1 and bj.last_error() == "sparse patchify batch must be nonzero"
    rc = L.bjf_sparse_patchify_plan_coords(FAKE, 3, None, 3, 2, _abi.dims(2, 3, 4), FAKE, 6, None, None)
    assert rc == -1 and "mask rows must be 1 or equal the batch" in bj.last_error()


def test_ring_step_rejects_bad_slots():
    desc = bj.FrontEndDesc(2, 3, 2, 64, 64, 2, 16, 256, _abi.DTYPE_F16, _abi.DTYPE_F16, _abi.DTYPE_F16,
                           bj.PatchDiffConfig.adaptive_threshold(0.1, 1, 16, 1))
    lib = bj.load()
    for slots, prev, cur in ((3, 1, 1), (3, 0, 3), (1, 0, 0), (3, -1, 0)):
        rc = lib.bjf_front_end_step_ring(ctypes.byref(desc), 16, slots, prev, cur, 16, None, 16, 16, 16, 0, 16, 1 << 20,
                                         None, None)
        assert rc == _abi.BJF_ERR_INVALID_ARGUMENT
        assert "frame ring" in bj.last_error()
    bad = bj.FrontEndDesc(2, 3, 4, 64, 64, 2, 16, 256, _abi.DTYPE_F16, _abi.DTYPE_F16, _abi.DTYPE_F16,
                          bj.PatchDiffConfig.adaptive_threshold(0.1, 1, 32, 1))
    assert lib.bjf_front_end_step_ring(ctypes.byref(bad), 16, 3, 0, 1, 16, None, 16, 16, 16, 0, 16, 1 << 20, None,
                                       None) == _abi.BJF_ERR_INVALID_ARGUMENT
    assert "frames = 2" in bj.last_error()


def test_ctypes_structs_have_the_c_layout(tmp_path):
    """Every ctypes mirror has the size and field offsets gcc gives the struct in bjf.h."""
    import os
    import subprocess

    structs = {"bjf_patchify_config": _abi.PatchifyConfig, "bjf_patch_diff_config": _abi.PatchDiffConfig,
               "bjf_front_end_desc": _abi.FrontEndDesc, "bjf_rgba_frame_stats": _abi.RgbaFrameStats,
               "bjf_viewer_mask_policy": _abi.ViewerMaskPolicy,
               "bjf_patch_diff_refresh_config": _abi.PatchDiffRefreshConfig,
               "bjf_patch_diff_refresh_state": _abi.PatchDiffRefreshState}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "bjf.h"', "int main(void) {"]
    want = []
    for cname, py in structs.items():
        lines.append(f'printf("%zu\\n", sizeof({cname}));')
        want.append(ctypes.sizeof(py))
        for field, *_ in py._fields_:
            lines.append(f'printf("%zu\\n", offsetof({cname}, {field}));')
            want.append(getattr(py, field).offset)
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    inc = os.path.dirname(_abi.HEADER_PATH)
    subprocess.run(["gcc", "-std=c11", "-I", inc, str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert got == want


def test_frame_ring_upload_rejects_bad_arguments():
    mask = bj.PatchDiffConfig.adaptive_threshold(0.1, 1, 16, 1)
    d = bj.FrontEndDesc(4, 3, 2, 64, 64, 2, 16, 64, _abi.DTYPE_F16, _abi.DTYPE_F16, _abi.DTYPE_F16, mask)
    up = bj.load().bjf_frame_ring_upload
    assert up(ctypes.byref(d), FAKE, FAKE, 3, 3, 0, 4, None) == _abi.BJF_ERR_INVALID_ARGUMENT
    assert "slot outside the ring" in bj.last_error()
    assert up(ctypes.byref(d), FAKE, FAKE, 1, 0, 0, 4, None) == _abi.BJF_ERR_INVALID_ARGUMENT
    assert up(ctypes.byref(d), FAKE, FAKE, 3, 0, 2, 5, None) == _abi.BJF_ERR_INVALID_ARGUMENT
    assert "streams outside" in bj.last_error()
    assert up(ctypes.byref(d), None, FAKE, 3, 0, 0, 4, None) == _abi.BJF_ERR_INVALID_ARGUMENT
    assert up(ctypes.byref(d), FAKE, FAKE, 3, 0, 2, 2, None) == 0  # nothing to copy


def test_refresh_entries_reject_bad_arguments_before_any_launch():
    lib = bj.load()
    cfg = bj.PatchDiffConfig.adaptive_threshold(0.1, 1, 16, 1)
    pol = bj._abi.ViewerMaskPolicy.new()
    refresh = bj.PatchDiffRefreshConfig.from_fields(enabled=True, blue_noise_enabled=True)
    dims = _abi.dims(1, 4, 4)
    state = _abi.PatchDiffRefreshState(FAKE.value, FAKE.value, FAKE.value)
    missing = _abi.PatchDiffRefreshState(None, None, None)
    out = [FAKE] * 4
    args = lambda r, st: (FAKE, 1, dims, ctypes.byref(cfg), ctypes.byref(pol), r, st, *out, None)  # noqa: E731
    assert lib.bjf_viewer_patch_diff_refresh_masks_from_scores(*args(ctypes.byref(refresh), None)) == -1
    assert "refresh state buffers" in bj.last_error()
    assert lib.bjf_viewer_patch_diff_refresh_masks_from_scores(*args(ctypes.byref(refresh),
                                                                     ctypes.byref(missing))) == -1
    assert "refresh state buffers" in bj.last_error()
    assert lib.bjf_viewer_patch_diff_refresh_masks_from_scores(*args(None, ctypes.byref(state))) == -1
    assert "refresh config" in bj.last_error()
    big = _abi.dims(2, 128, 256)  # 65 536 tokens: above the viewer kernels' 32 768
    assert lib.bjf_viewer_patch_diff_refresh_observe(FAKE, FAKE, 1, big, ctypes.byref(state), None) == -2
    assert "32768 tokens" in bj.last_error()
    assert lib.bjf_viewer_patch_diff_refresh_observe(None, FAKE, 1, dims, ctypes.byref(state), None) == -1
    assert lib.bjf_viewer_patch_diff_refresh_observe(FAKE, FAKE, 1, dims, ctypes.byref(missing), None) == -1
    assert lib.bjf_viewer_patch_diff_refresh_observe(FAKE, FAKE, 0, dims, ctypes.byref(state), None) == -1


def test_refresh_config_fields_and_defaults():
    c = bj.PatchDiffRefreshConfig.from_fields()
    assert (c.enabled, c.subthreshold_enabled, c.age_refresh_enabled, c.blue_noise_enabled) == (0, 0, 0, 0)
    assert c.age_refresh_interval_frames == 90 and c.blue_noise_seed == 0x9E3779B97F4A7C15
    assert abs(c.subthreshold_decay - 0.92) < 1e-7 and abs(c.max_extra_density - 0.05) < 1e-9
    with pytest.raises(TypeError, match="unknown refresh config fields"):
        bj.PatchDiffRefreshConfig.from_fields(nonsense=1)
