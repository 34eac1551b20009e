//! Rust face of the B200 (sm_100a) sparse front end, libbjf.so.
//!
//! `ffi` declares every entry point of include/bjf.h.  With the `sparse-patchify-b200` feature,
//! `b200` wraps the two calls burn_jepa's `sparse-patchify-cuda` lane makes on Burn CUDA tensors,
//! with the reference's signatures, so the call sites change only their path:
//!
//! | burn_jepa 0.21.0 call | replacement |
//! |---|---|
//! | `burn_flex_gmm::cuda::sparse_patchify3d_forward_cuda` (src/model.rs:1140, 1197, 1319; src/sparse_patchify.rs:184) | [`b200::sparse_patchify3d_forward_cuda`] |
//! | `sparse_feature_memory_assign_latest_cuda_raw` (src/sparse_feature_memory.rs:296-313, called at src/feature_memory.rs:629) | [`b200::sparse_feature_memory_assign_latest_cuda_raw`] |
//!
//! Compile-unchecked: this repository's build image has no cargo/rustc or crates.io registry.
pub mod ffi;

#[cfg(feature = "sparse-patchify-b200")]
pub mod b200;
