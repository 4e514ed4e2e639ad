//! burn-extended's `moe` / `quant` API over the B200 MXFP4 MoE library.
//!
//! The reference crate's `MoeGatedSwiGLU::forward` (src/moe/mod.rs:99-115)
//! is bound to `B: Backend<FloatTensorPrimitive = CubeTensor<WgpuRuntime>>`;
//! this crate keeps the same names, fields and call sequence
//! (`MoeConfig::init`, `MoeQuantLayerResident::new`, `set_resident`,
//! `forward`) with the activations in CUDA device memory
//! ([`tensor::DeviceTensor`]).  Failures panic with the library's message,
//! as the reference panics (src/moe/mod.rs:112); loaders return `Result`.
//!
//! Module map (reference file -> here):
//!   src/moe/mod.rs               -> moe
//!   src/quant/{mod,gpu}.rs       -> quant
//!   src/loader/mxfp4.rs          -> loader::mxfp4
//!   src/loader/modelbin.rs (MoE) -> loader::modelbin
//!   src/models/gpt_oss.rs (MoE)  -> models::gpt_oss
//!   src/attention/streaming_mqa.rs -> attention

pub mod attention;
pub mod error;
pub mod loader;
pub mod models;
pub mod moe;
pub mod quant;
pub mod tensor;

pub use burn_extended_cuda_sys as sys;
