//! `quant` (src/quant/mod.rs:3-21, src/quant/gpu.rs:14-83) over libmxmoe.
//!
//! The reference uploads the raw MXFP4 buffers in `MoeQuantLayerResident::new`
//! (`client.create`, src/quant/gpu.rs:31-53).  Here the library repacks them
//! into its tensor-core operand layout, which needs the layer's biases and
//! router too, so the device copy is made when the resident weights are
//! attached (`MoeGatedSwiGLU::set_resident`); `new` takes ownership of the
//! host buffers exactly as the reference does (:50-51).
use std::sync::Arc;

use crate::sys;

/// `quant::QuantLinearMxFp4Desc` (src/quant/mod.rs:3-11).
#[derive(Debug, Clone, Copy, PartialEq, Eq)]
pub struct QuantLinearMxFp4Desc {
    pub experts: usize,
    pub rows: usize,
    pub cols: usize,
    /// bytes per row of blocks
    pub bpr: usize,
    /// groups per row for scales (per 32 columns)
    pub gpr: usize,
    pub ue8_offset: i32,
}

impl QuantLinearMxFp4Desc {
    /// The descriptor of a `[experts][rows][cols]` MXFP4 matrix.
    pub fn for_shape(experts: usize, rows: usize, cols: usize, ue8_offset: i32) -> Self {
        Self { experts, rows, cols, bpr: (cols + 1) / 2, gpr: (cols + 31) / 32, ue8_offset }
    }

    pub(crate) fn to_c(self) -> sys::mxmoe_quant_desc {
        sys::mxmoe_quant_desc {
            experts: self.experts as u64,
            rows: self.rows as u64,
            cols: self.cols as u64,
            bpr: self.bpr as u64,
            gpr: self.gpr as u64,
            ue8_offset: self.ue8_offset,
        }
    }
}

/// `quant::MoeQuantLayerHost` (src/quant/mod.rs:13-21).
#[derive(Debug, Clone)]
pub struct MoeQuantLayerHost {
    pub w1_desc: QuantLinearMxFp4Desc,
    pub w2_desc: QuantLinearMxFp4Desc,
    pub w1_blocks: Vec<u8>,
    pub w1_scales: Vec<u8>,
    pub w2_blocks: Vec<u8>,
    pub w2_scales: Vec<u8>,
}

/// The CUDA device a layer lives on (replaces `WgpuDevice`).
#[derive(Debug, Clone, Copy, PartialEq, Eq, Default)]
pub struct CudaDevice {
    pub index: i32,
}

impl CudaDevice {
    pub fn new(index: i32) -> Self {
        Self { index }
    }
}

/// `quant::QuantLinearMxFp4Resident` (src/quant/gpu.rs:14-23): the
/// descriptor and the host copies the reference also keeps (:20-21).
#[derive(Debug, Clone)]
pub struct QuantLinearMxFp4Resident {
    pub desc: QuantLinearMxFp4Desc,
    pub blocks_host: Vec<u8>,
    pub scales_host: Vec<u8>,
}

/// `quant::MoeQuantLayerResident` (src/quant/gpu.rs:25-54).
#[derive(Debug, Clone)]
pub struct MoeQuantLayerResident {
    pub w1: QuantLinearMxFp4Resident,
    pub w2: QuantLinearMxFp4Resident,
    pub device: CudaDevice,
}

impl MoeQuantLayerResident {
    /// Same signature and ownership as the reference (src/quant/gpu.rs:31-53).
    pub fn new(
        device: &CudaDevice,
        w1_desc: QuantLinearMxFp4Desc,
        w1_blocks: Vec<u8>,
        w1_scales: Vec<u8>,
        w2_desc: QuantLinearMxFp4Desc,
        w2_blocks: Vec<u8>,
        w2_scales: Vec<u8>,
    ) -> Self {
        assert_eq!(w1_blocks.len(), w1_desc.experts * w1_desc.rows * w1_desc.bpr, "w1 blocks size");
        assert_eq!(w1_scales.len(), w1_desc.experts * w1_desc.rows * w1_desc.gpr, "w1 scales size");
        assert_eq!(w2_blocks.len(), w2_desc.experts * w2_desc.rows * w2_desc.bpr, "w2 blocks size");
        assert_eq!(w2_scales.len(), w2_desc.experts * w2_desc.rows * w2_desc.gpr, "w2 scales size");
        Self {
            w1: QuantLinearMxFp4Resident { desc: w1_desc, blocks_host: w1_blocks, scales_host: w1_scales },
            w2: QuantLinearMxFp4Resident { desc: w2_desc, blocks_host: w2_blocks, scales_host: w2_scales },
            device: *device,
        }
    }

    pub fn from_host(device: &CudaDevice, host: MoeQuantLayerHost) -> Self {
        Self::new(device, host.w1_desc, host.w1_blocks, host.w1_scales, host.w2_desc, host.w2_blocks, host.w2_scales)
    }
}

/// `attach_quant_to_model_layers` (src/quant/gpu.rs:57-70).
pub fn attach_quant_to_model_layers(
    model: &mut crate::models::gpt_oss::GptOssMoeLayers,
    layers: Vec<MoeQuantLayerResident>,
) {
    model.set_moe_quant_resident(layers);
}

/// `attach_quant_from_host_to_model` (src/quant/gpu.rs:72-83).
pub fn attach_quant_from_host_to_model(
    model: &mut crate::models::gpt_oss::GptOssMoeLayers,
    layers: Vec<MoeQuantLayerHost>,
) {
    model.set_moe_quant_from_host(layers);
}

pub(crate) type SharedResident = Arc<MoeQuantLayerResident>;
