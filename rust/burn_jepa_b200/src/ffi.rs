//! Raw declarations of the C ABI of libbjf.so, one to one with include/bjf.h (the header is the
//! authority: its comments state each entry point's contract and the burn_jepa function it
//! replaces).  All pointers are device pointers unless the C header says "host"; work is
//! enqueued on `stream`; a status of 0 is success, negative an invalid argument (message from
//! `bjf_get_last_error_string`), positive a CUDA error.
#![allow(non_camel_case_types)]

use std::ffi::c_void;

pub type bjf_status = i32;
/// `cudaStream_t` (a `CUstream`); null is the legacy default stream.
pub type bjf_stream_t = *mut c_void;
/// `bjf_dtype` (a C enum, int-sized).
pub type bjf_dtype = i32;

pub const BJF_ABI_VERSION: i32 = 4;

pub const BJF_OK: bjf_status = 0;
pub const BJF_ERR_INVALID_ARGUMENT: bjf_status = -1;
pub const BJF_ERR_UNSUPPORTED: bjf_status = -2;
pub const BJF_ERR_CUDA: bjf_status = 1;

pub const BJF_DTYPE_F32: bjf_dtype = 0;
pub const BJF_DTYPE_F16: bjf_dtype = 1;
pub const BJF_DTYPE_BF16: bjf_dtype = 2;
pub const BJF_DTYPE_I32: bjf_dtype = 3;

/// `burn_flex_gmm::SparsePatchify3dConfig` as the encoder fills it (src/model.rs:1297-1306).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct bjf_patchify_config {
    pub in_channels: i64,
    pub out_channels: i64,
    pub frames: i64,
    pub height: i64,
    pub width: i64,
    pub tubelet_size: i64,
    pub patch_h: i64,
    pub patch_w: i64,
}

/// `SparseJepaPatchDiffSparsityConfig` (src/nodes.rs:97-157).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct bjf_patch_diff_config {
    pub threshold: f32,
    pub context_tokens: i64,
    pub target_tokens: i64,
    pub dilation: i64,
    pub min_context_tokens: i64,
    pub fill_to_context_tokens: i32,
    pub allow_full_context: i32,
}

/// `RgbaPatchDiffFrameStats` (src/viewer.rs:1067-1076) plus the two means it compares.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct bjf_rgba_frame_stats {
    pub channel_delta: [f32; 3],
    pub luma_delta: f32,
    pub compensate_global_lighting: i32,
    pub raw_abs: f32,
    pub residual_abs: f32,
}

/// The mask fields of `FeatureFrameViewerConfig` (src/viewer.rs:566-579).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct bjf_viewer_mask_policy {
    pub dense_fallback_density: f32,
    pub dilation: i64,
    pub bucketed_encode: i32,
    pub bucket_tokens: i64,
    pub bucket_density_count: i32,
    pub bucket_densities: [f32; 32],
}

/// `PatchDiffRefreshConfig` (src/viewer.rs:186-270); flags are 0 or 1.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct bjf_patch_diff_refresh_config {
    pub enabled: i32,
    pub subthreshold_enabled: i32,
    pub subthreshold_decay: f32,
    pub subthreshold_gain: f32,
    pub subthreshold_trigger: f32,
    pub subthreshold_max_density: f32,
    pub age_refresh_enabled: i32,
    pub age_refresh_interval_frames: u64,
    pub age_refresh_max_density: f32,
    pub blue_noise_enabled: i32,
    pub blue_noise_refresh_density: f32,
    pub blue_noise_seed: u64,
    pub max_extra_density: f32,
}

/// `PatchDiffRefreshState` (src/viewer.rs:275-283) of S streams in device memory: residuals
/// [S, N] f32, ages [S, N] u32, frame indices [S] u64; all zeros before the first frame.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct bjf_patch_diff_refresh_state {
    pub subthreshold_residual: *mut f32,
    pub age_frames: *mut u32,
    pub frame_index: *mut u64,
}

/// One video stream per index s: video [S, C, T, H, W], caches [S, N, D], observed / age [S, N].
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct bjf_front_end_desc {
    pub streams: i64,
    pub channels: i64,
    pub frames: i64,
    pub height: i64,
    pub width: i64,
    pub tubelet_size: i64,
    pub patch_size: i64,
    pub embed_dim: i64,
    pub video_dtype: bjf_dtype,
    pub weight_dtype: bjf_dtype,
    pub cache_dtype: bjf_dtype,
    pub mask: bjf_patch_diff_config,
}

unsafe extern "C" {
    pub fn bjf_abi_version() -> i32;
    pub fn bjf_get_last_error_string(buf: *mut u8, len: usize) -> usize;
    pub fn bjf_device_error_check(stream: bjf_stream_t, flag_out: *mut i32) -> bjf_status;
    pub fn bjf_set_bounded_wait(limit_ns: u64, stall: i32) -> bjf_status;

    pub fn bjf_patch_diff_token_scores(
        video: *const c_void,
        video_dtype: bjf_dtype,
        video_dims: *const i64,
        streams: i64,
        tubelet_size: i64,
        patch_size: i64,
        scores: *mut f32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_patch_diff_context_mask_from_scores(
        scores: *const f32,
        streams: i64,
        grid: *const i64,
        config: *const bjf_patch_diff_config,
        indices: *mut i32,
        counts: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_patch_diff_context_mask(
        video: *const c_void,
        video_dtype: bjf_dtype,
        video_dims: *const i64,
        streams: i64,
        tubelet_size: i64,
        patch_size: i64,
        grid: *const i64,
        config: *const bjf_patch_diff_config,
        scores: *mut f32,
        indices: *mut i32,
        counts: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;

    pub fn bjf_sparse_patchify_plan_coords(
        indices: *const i32,
        index_stride: i64,
        counts: *const i32,
        mask_rows: i64,
        batch: i64,
        grid: *const i64,
        coords: *mut i32,
        coords_capacity: i64,
        total_rows: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;

    pub fn bjf_sparse_patchify3d_forward(
        config: *const bjf_patchify_config,
        input: *const c_void,
        input_dtype: bjf_dtype,
        input_dims: *const i64,
        coords: *const i32,
        rows: i64,
        weight: *const c_void,
        weight_dtype: bjf_dtype,
        weight_dims: *const i64,
        bias: *const f32,
        out: *mut c_void,
        out_dtype: bjf_dtype,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_sparse_patchify3d_forward_encoder_input(
        config: *const bjf_patchify_config,
        input: *const c_void,
        input_dtype: bjf_dtype,
        input_dims: *const i64,
        coords: *const i32,
        rows: i64,
        weight: *const c_void,
        weight_dtype: bjf_dtype,
        weight_dims: *const i64,
        bias: *const f32,
        position_table: *const f32,
        modality_embed: *const f32,
        out: *mut c_void,
        out_dtype: bjf_dtype,
        stream: bjf_stream_t,
    ) -> bjf_status;

    pub fn bjf_feature_memory_assign_latest(
        features: *mut c_void,
        features_dtype: bjf_dtype,
        features_dims: *const i64,
        observed: *mut f32,
        observed_dims: *const i64,
        age_frames: *mut f32,
        age_dims: *const i64,
        tokens: *const c_void,
        tokens_dtype: bjf_dtype,
        tokens_dims: *const i64,
        token_indices: *const i32,
        indices_dims: *const i64,
        age_observed: i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_feature_memory_update_ema(
        features: *mut c_void,
        features_dtype: bjf_dtype,
        features_dims: *const i64,
        observed: *mut f32,
        observed_dims: *const i64,
        age_frames: *mut f32,
        age_dims: *const i64,
        tokens: *const c_void,
        tokens_dtype: bjf_dtype,
        tokens_dims: *const i64,
        token_indices: *const i32,
        indices_dims: *const i64,
        alpha: f32,
        age_observed: i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_feature_memory_reset_rows(
        features: *mut c_void,
        features_dtype: bjf_dtype,
        features_dims: *const i64,
        observed: *mut f32,
        age_frames: *mut f32,
        rows: *const i32,
        row_count: i64,
        stream: bjf_stream_t,
    ) -> bjf_status;

    pub fn bjf_rgba_patch_diff_workspace_bytes(streams: i64, grid: *const i64) -> usize;
    pub fn bjf_rgba_patch_diff_scores(
        prev: *const u8,
        current: *const u8,
        streams: i64,
        width: i64,
        height: i64,
        patch_size: i64,
        grid: *const i64,
        scores: *mut f32,
        stats_out: *mut bjf_rgba_frame_stats,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_viewer_patch_diff_masks(
        direct_indices: *const i32,
        direct_counts: *const i32,
        streams: i64,
        grid: *const i64,
        policy: *const bjf_viewer_mask_policy,
        write_indices: *mut i32,
        write_counts: *mut i32,
        encode_indices: *mut i32,
        encode_counts: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_viewer_patch_diff_masks_from_scores(
        scores: *const f32,
        streams: i64,
        grid: *const i64,
        config: *const bjf_patch_diff_config,
        policy: *const bjf_viewer_mask_policy,
        write_indices: *mut i32,
        write_counts: *mut i32,
        encode_indices: *mut i32,
        encode_counts: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_viewer_rgba_masks_workspace_bytes(streams: i64, grid: *const i64) -> usize;
    pub fn bjf_viewer_patch_diff_masks_from_rgba(
        prev: *const u8,
        current: *const u8,
        streams: i64,
        width: i64,
        height: i64,
        patch_size: i64,
        grid: *const i64,
        config: *const bjf_patch_diff_config,
        policy: *const bjf_viewer_mask_policy,
        write_indices: *mut i32,
        write_counts: *mut i32,
        encode_indices: *mut i32,
        encode_counts: *mut i32,
        stats_out: *mut bjf_rgba_frame_stats,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: bjf_stream_t,
    ) -> bjf_status;

    pub fn bjf_viewer_patch_diff_refresh_masks_from_scores(
        scores: *const f32,
        streams: i64,
        grid: *const i64,
        config: *const bjf_patch_diff_config,
        policy: *const bjf_viewer_mask_policy,
        refresh: *const bjf_patch_diff_refresh_config,
        state: *const bjf_patch_diff_refresh_state,
        write_indices: *mut i32,
        write_counts: *mut i32,
        encode_indices: *mut i32,
        encode_counts: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_viewer_patch_diff_refresh_masks_from_rgba(
        prev: *const u8,
        current: *const u8,
        streams: i64,
        width: i64,
        height: i64,
        patch_size: i64,
        grid: *const i64,
        config: *const bjf_patch_diff_config,
        policy: *const bjf_viewer_mask_policy,
        refresh: *const bjf_patch_diff_refresh_config,
        state: *const bjf_patch_diff_refresh_state,
        write_indices: *mut i32,
        write_counts: *mut i32,
        encode_indices: *mut i32,
        encode_counts: *mut i32,
        stats_out: *mut bjf_rgba_frame_stats,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_viewer_patch_diff_refresh_observe(
        write_indices: *const i32,
        write_counts: *const i32,
        streams: i64,
        grid: *const i64,
        state: *const bjf_patch_diff_refresh_state,
        stream: bjf_stream_t,
    ) -> bjf_status;

    pub fn bjf_frame_ring_upload(
        desc: *const bjf_front_end_desc,
        host_frame: *const c_void,
        frame_ring: *mut c_void,
        ring_slots: i32,
        slot: i32,
        stream_begin: i64,
        stream_end: i64,
        stream: bjf_stream_t,
    ) -> bjf_status;

    pub fn bjf_front_end_workspace_bytes(desc: *const bjf_front_end_desc) -> usize;
    pub fn bjf_front_end_step(
        desc: *const bjf_front_end_desc,
        video: *const c_void,
        weight: *const c_void,
        bias: *const f32,
        caches: *mut c_void,
        observed: *mut f32,
        age_frames: *mut f32,
        age_observed: i32,
        workspace: *mut c_void,
        workspace_bytes: usize,
        counts_out: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_front_end_step_ring(
        desc: *const bjf_front_end_desc,
        frame_ring: *const c_void,
        ring_slots: i32,
        prev_slot: i32,
        cur_slot: i32,
        weight: *const c_void,
        bias: *const f32,
        caches: *mut c_void,
        observed: *mut f32,
        age_frames: *mut f32,
        age_observed: i32,
        workspace: *mut c_void,
        workspace_bytes: usize,
        counts_out: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
    pub fn bjf_front_end_step_no_alloc(
        desc: *const bjf_front_end_desc,
        video: *const c_void,
        weight: *const c_void,
        bias: *const f32,
        caches: *mut c_void,
        observed: *mut f32,
        age_frames: *mut f32,
        age_observed: i32,
        counts_out: *mut i32,
        stream: bjf_stream_t,
    ) -> bjf_status;
}

/// The message of the last failing call on this thread.
pub fn last_error() -> String {
    let mut buf = vec![0u8; 1024];
    let n = unsafe { bjf_get_last_error_string(buf.as_mut_ptr(), buf.len()) };
    buf.truncate(n.min(buf.len() - 1));
    String::from_utf8_lossy(&buf).into_owned()
}

/// Ok for BJF_OK, else Err with the library's message (the reference's texts for shape errors).
pub fn check(status: bjf_status) -> Result<(), String> {
    if status == BJF_OK { Ok(()) } else { Err(last_error()) }
}

/// Fails when the loaded library was built from another ABI version of include/bjf.h.
pub fn check_abi() -> Result<(), String> {
    let built = unsafe { bjf_abi_version() };
    if built == BJF_ABI_VERSION {
        Ok(())
    } else {
        Err(format!("libbjf.so has ABI version {built}, this crate expects {BJF_ABI_VERSION}"))
    }
}
