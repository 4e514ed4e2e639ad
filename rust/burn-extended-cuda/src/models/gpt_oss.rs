//! The MoE side of `GptOssModel` (src/models/gpt_oss.rs).
//!
//! In the reference, `GptOssLayer::forward` (:101-113) ends with
//!
//! ```text
//! let hidden = hidden + context;
//! self.mlp.forward(hidden)     // MoeGatedSwiGLU on WGPU
//! ```
//!
//! and the weights arrive through `set_moe_quant_from_host` (:467-488) ->
//! `set_moe_quant_resident` (:458-466) -> `MoeGatedSwiGLU::set_resident`.
//! The drop-in keeps that sequence with the hidden state in CUDA memory:
//! [`GptOssMoeLayers`] holds one `MoeGatedSwiGLU` per decoder block, and the
//! decoder block calls [`GptOssMoeLayers::mlp_forward`] where it called
//! `self.mlp.forward(hidden)`.  The only bound that changes is the
//! reference's `B: Backend<FloatTensorPrimitive = CubeTensor<WgpuRuntime>>`
//! (src/moe/mod.rs:100-105): the activations are `DeviceTensor`s.
use std::sync::Arc;

use crate::moe::{MoeConfig, MoeGatedSwiGLU};
use crate::quant::{CudaDevice, MoeQuantLayerHost, MoeQuantLayerResident};
use crate::tensor::DeviceTensor;

/// The MoE blocks of a GPT-OSS model, one per decoder layer.
#[derive(Debug, Clone)]
pub struct GptOssMoeLayers {
    pub layers: Vec<MoeGatedSwiGLU>,
    pub device: CudaDevice,
    resident: Vec<MoeQuantLayerResident>,
}

impl GptOssMoeLayers {
    /// `num_blocks` layers with the GPT-OSS MoE config.
    pub fn new(cfg: &MoeConfig, num_blocks: usize, device: CudaDevice) -> Self {
        Self { layers: (0..num_blocks).map(|_| cfg.init(&device)).collect(), device, resident: Vec::new() }
    }

    /// `set_moe_quant_resident` (src/models/gpt_oss.rs:458-466).
    pub fn set_moe_quant_resident(&mut self, layers: Vec<MoeQuantLayerResident>) {
        assert_eq!(layers.len(), self.layers.len(), "resident layers len mismatch");
        for (mlp, res) in self.layers.iter_mut().zip(layers.iter()) {
            mlp.set_resident(Arc::new(res.clone()));
        }
        self.resident = layers;
    }

    /// `set_moe_quant_from_host` (src/models/gpt_oss.rs:467-488).
    pub fn set_moe_quant_from_host(&mut self, layers: Vec<MoeQuantLayerHost>) {
        let device = self.device;
        let residents = layers.into_iter().map(|h| MoeQuantLayerResident::from_host(&device, h)).collect();
        self.set_moe_quant_resident(residents);
    }

    /// The MoE step of `GptOssLayer::forward` (src/models/gpt_oss.rs:112):
    /// the block handles its own RmsNorm and residual.
    pub fn mlp_forward(&self, layer: usize, hidden: DeviceTensor<3>) -> DeviceTensor<3> {
        self.layers[layer].forward(hidden)
    }
}
