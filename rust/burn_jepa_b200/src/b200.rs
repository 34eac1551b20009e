//! The reference's CUDA sparse-patchify and tiled-assign calls on libbjf.so, over Burn CUDA tensors.
//!
//! Tensor -> device pointer glue: a Burn float tensor's primitive is a `CubeTensor<CudaRuntime>`
//! (`tensor.into_primitive().tensor()`, as src/sparse_feature_memory.rs:169-173 does); its buffer
//! is resolved through the compute client (`device_ptr` below: the one cubecl-cuda 0.10 accessor
//! this crate depends on, written from the cubecl 0.10 server API and unverified here).
//!
//! Streams: CubeCL enqueues on its own CUDA stream for the device.  Without an accessor for that
//! stream, each call synchronises the device before enqueueing on the legacy default stream and
//! synchronises it again before returning, so Burn's later work sees the results.  Passing
//! CubeCL's stream instead (where the runtime exposes it) removes both synchronisations.
use burn::tensor::{DType, Int, Tensor, TensorPrimitive};
use burn_cubecl::tensor::CubeTensor;
use cubecl_cuda::CudaRuntime;

use crate::ffi;

/// burn_jepa's CUDA backend for these calls (`RawCudaBackend`, src/sparse_feature_memory.rs:273-275;
/// burn_flex_gmm's `cuda::DefaultCudaBackend` is the same f32 / i32 / u8 CubeBackend).
pub type RawCudaBackend = burn_cubecl::CubeBackend<CudaRuntime, f32, i32, u8>;
pub type DefaultCudaBackend = RawCudaBackend;

/// burn_flex_gmm 0.21.2's `SparsePatchify3dConfig`, field for field (src/model.rs:1297-1306).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub struct SparsePatchify3dConfig {
    pub in_channels: usize,
    pub out_channels: usize,
    pub frames: usize,
    pub height: usize,
    pub width: usize,
    pub tubelet_size: usize,
    pub patch_h: usize,
    pub patch_w: usize,
}

/// `SparseFeatureMemoryAssignOutput` (src/sparse_feature_memory.rs:4-9).
#[derive(Debug)]
pub struct SparseFeatureMemoryAssignOutput<B: burn::tensor::backend::Backend> {
    pub features: Tensor<B, 3>,
    pub observed: Tensor<B, 2>,
    pub age_frames: Tensor<B, 2>,
}

fn dims_i64<const D: usize>(dims: [usize; D]) -> [i64; D] {
    dims.map(|d| d as i64)
}

fn dtype_code(dtype: DType) -> Result<ffi::bjf_dtype, String> {
    match dtype {
        DType::F32 => Ok(ffi::BJF_DTYPE_F32),
        DType::F16 => Ok(ffi::BJF_DTYPE_F16),
        DType::BF16 => Ok(ffi::BJF_DTYPE_BF16),
        DType::I32 => Ok(ffi::BJF_DTYPE_I32),
        other => Err(format!("libbjf: unsupported dtype {other:?}")),
    }
}

/// CUDA device address of a contiguous tensor's first element.
fn device_ptr(t: &CubeTensor<CudaRuntime>) -> Result<u64, String> {
    if !t.is_contiguous() {
        return Err("libbjf: tensors must be contiguous".to_string());
    }
    let resource = t.client.get_resource(t.handle.clone().binding());
    Ok(resource.resource().ptr)
}

fn sync(t: &CubeTensor<CudaRuntime>) -> Result<(), String> {
    burn::tensor::backend::Backend::sync(&t.device).map_err(|e| format!("libbjf: device sync failed: {e:?}"))
}

fn null_stream() -> ffi::bjf_stream_t {
    std::ptr::null_mut()
}

/// The legacy default stream's work is complete (the library enqueued there).
fn finish(t: &CubeTensor<CudaRuntime>) -> Result<(), String> {
    let mut flag = 0i32;
    ffi::check(unsafe { ffi::bjf_device_error_check(null_stream(), &mut flag) })?;
    if flag != 0 {
        return Err("libbjf: a kernel gave up on a bounded wait (device timeout)".to_string());
    }
    sync(t)
}

/// Replaces `burn_flex_gmm::cuda::sparse_patchify3d_forward_cuda`: out[m, d] = bias[d] +
/// sum_k W[d, k] x[coords[m], k], Conv3d with stride = kernel at the selected tubelets.  The
/// output is allocated through the Burn client as [rows, out_channels] f32, as the reference's is.
pub fn sparse_patchify3d_forward_cuda(
    config: &SparsePatchify3dConfig,
    input: Tensor<DefaultCudaBackend, 5>,
    coords: Tensor<DefaultCudaBackend, 2, Int>,
    weight: Tensor<DefaultCudaBackend, 5>,
    bias: Tensor<DefaultCudaBackend, 1>,
) -> Result<Tensor<DefaultCudaBackend, 2>, String> {
    ffi::check_abi()?;
    let input_dims = input.dims();
    let weight_dims = weight.dims();
    let [rows, coord_width] = coords.dims();
    if coord_width != 4 {
        return Err(format!("sparse patchify coords must be [rows, 4], got [{rows},{coord_width}]"));
    }
    let device = input.device();
    let out = Tensor::<DefaultCudaBackend, 2>::empty([rows, config.out_channels], &device);
    if rows == 0 {
        return Ok(out);
    }
    let input_p = input.into_primitive().tensor();
    let coords_p = coords.into_primitive();
    let weight_p = weight.into_primitive().tensor();
    let bias_p = bias.into_primitive().tensor();
    let out_p = out.into_primitive().tensor();
    let cfg = ffi::bjf_patchify_config {
        in_channels: config.in_channels as i64,
        out_channels: config.out_channels as i64,
        frames: config.frames as i64,
        height: config.height as i64,
        width: config.width as i64,
        tubelet_size: config.tubelet_size as i64,
        patch_h: config.patch_h as i64,
        patch_w: config.patch_w as i64,
    };
    let id = dims_i64(input_dims);
    let wd = dims_i64(weight_dims);
    sync(&input_p)?;
    let status = unsafe {
        ffi::bjf_sparse_patchify3d_forward(
            &cfg,
            device_ptr(&input_p)? as *const _,
            dtype_code(input_p.dtype)?,
            id.as_ptr(),
            device_ptr(&coords_p)? as *const i32,
            rows as i64,
            device_ptr(&weight_p)? as *const _,
            dtype_code(weight_p.dtype)?,
            wd.as_ptr(),
            device_ptr(&bias_p)? as *const f32,
            device_ptr(&out_p)? as *mut _,
            ffi::BJF_DTYPE_F32,
            null_stream(),
        )
    };
    ffi::check(status)?;
    finish(&out_p)?;
    Ok(Tensor::from_primitive(TensorPrimitive::Float(out_p)))
}

/// Replaces `sparse_feature_memory_assign_latest_cuda_raw`, with its shape checks and messages
/// (src/sparse_feature_memory.rs:125-150).  The update runs in place: a buffer that another
/// tensor still shares is copied first, so snapshots the caller holds stay unchanged, as with
/// the reference's fresh outputs.
pub fn sparse_feature_memory_assign_latest_cuda_raw(
    features: Tensor<RawCudaBackend, 3>,
    observed: Tensor<RawCudaBackend, 2>,
    age_frames: Tensor<RawCudaBackend, 2>,
    tokens: Tensor<RawCudaBackend, 3>,
    token_indices: Tensor<RawCudaBackend, 2, Int>,
    age_observed: bool,
) -> Result<SparseFeatureMemoryAssignOutput<RawCudaBackend>, String> {
    ffi::check_abi()?;
    let [batch, dense_tokens, embed_dim] = features.dims();
    let [observed_batch, observed_tokens] = observed.dims();
    let [age_batch, age_tokens] = age_frames.dims();
    if observed_batch != batch || observed_tokens != dense_tokens || age_batch != batch || age_tokens != dense_tokens {
        return Err(format!(
            "feature memory metadata dims mismatch: features=[{batch},{dense_tokens},{embed_dim}] observed=[{observed_batch},{observed_tokens}] age=[{age_batch},{age_tokens}]"
        ));
    }
    let [token_batch, sparse_len, token_dim] = tokens.dims();
    let [index_batch, index_len] = token_indices.dims();
    if token_batch != batch || token_dim != embed_dim {
        return Err(format!(
            "feature memory token dims mismatch: tokens=[{token_batch},{sparse_len},{token_dim}] expected=[{batch},sparse,{embed_dim}]"
        ));
    }
    if index_batch != batch || index_len != sparse_len {
        return Err(format!(
            "feature memory index dims mismatch: indices=[{index_batch},{index_len}] expected=[{batch},{sparse_len}]"
        ));
    }
    if sparse_len == 0 {
        return Err("feature memory sparse assignment requires at least one token".to_string());
    }
    // in place on buffers nothing else shares; a shared buffer is copied first
    let own = |p: CubeTensor<CudaRuntime>| -> CubeTensor<CudaRuntime> {
        if p.handle.can_mut() {
            p
        } else {
            let t = Tensor::<RawCudaBackend, 1>::from_primitive(TensorPrimitive::Float(p));
            t.add_scalar(0.0).into_primitive().tensor()
        }
    };
    let features_p = own(features.into_primitive().tensor());
    let observed_p = own(observed.into_primitive().tensor());
    let age_p = own(age_frames.into_primitive().tensor());
    let tokens_p = tokens.into_primitive().tensor();
    let idx_p = token_indices.into_primitive();
    let fd = dims_i64([batch, dense_tokens, embed_dim]);
    let md = dims_i64([batch, dense_tokens]);
    let td = dims_i64([token_batch, sparse_len, token_dim]);
    let xd = dims_i64([index_batch, index_len]);
    sync(&features_p)?;
    let status = unsafe {
        ffi::bjf_feature_memory_assign_latest(
            device_ptr(&features_p)? as *mut _,
            dtype_code(features_p.dtype)?,
            fd.as_ptr(),
            device_ptr(&observed_p)? as *mut f32,
            md.as_ptr(),
            device_ptr(&age_p)? as *mut f32,
            md.as_ptr(),
            device_ptr(&tokens_p)? as *const _,
            dtype_code(tokens_p.dtype)?,
            td.as_ptr(),
            device_ptr(&idx_p)? as *const i32,
            xd.as_ptr(),
            age_observed as i32,
            null_stream(),
        )
    };
    ffi::check(status)?;
    finish(&features_p)?;
    Ok(SparseFeatureMemoryAssignOutput {
        features: Tensor::from_primitive(TensorPrimitive::Float(features_p)),
        observed: Tensor::from_primitive(TensorPrimitive::Float(observed_p)),
        age_frames: Tensor::from_primitive(TensorPrimitive::Float(age_p)),
    })
}
