//! Loaders: the MXFP4 dequant helper and the model.bin MoE reader.
pub mod modelbin;
pub mod mxfp4;
