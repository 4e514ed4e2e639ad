//! `moe` (src/moe/mod.rs:22-115) over libmxmoe.
//!
//! `MoeGatedSwiGLU::forward` keeps the reference's contract: x [batch, seq,
//! d_model] in, x + MoE(RmsNorm(x)) out, the input consumed; a layer without
//! resident weights panics (src/moe/mod.rs:111-113); `disabled` returns x
//! unchanged (:106-108).  The whole layer -- RmsNorm, gate, top-k + softmax,
//! permutation, both expert projections with SwiGLU-clamp, the combine and
//! the residual -- runs in one call into the library on the layer's device.
use std::ffi::c_void;
use std::ptr;
use std::sync::Arc;

use crate::error::{check, check_or_panic, MxMoeError};
use crate::quant::{CudaDevice, MoeQuantLayerResident, SharedResident};
use crate::sys;
use crate::tensor::{DType, DeviceTensor};

/// Placeholder of Burn's `Initializer`: weights are always loaded.
#[derive(Debug, Clone, Copy, PartialEq, Eq, Default)]
pub enum Initializer {
    #[default]
    Loaded,
}

/// `moe::MoeConfig` (src/moe/mod.rs:22-33).
#[derive(Debug, Clone)]
pub struct MoeConfig {
    pub d_model: usize,
    pub ffn_hidden: usize,
    pub num_experts: usize,
    pub experts_per_token: usize,
    pub swiglu_alpha: f32,
    pub swiglu_limit: f32,
    pub initializer: Initializer,
    pub disabled: bool,
    pub verbose: bool,
}

impl MoeConfig {
    pub fn new(d_model: usize, ffn_hidden: usize, num_experts: usize, experts_per_token: usize) -> Self {
        Self {
            d_model,
            ffn_hidden,
            num_experts,
            experts_per_token,
            swiglu_alpha: 1.702,
            swiglu_limit: 7.0,
            initializer: Initializer::default(),
            disabled: false,
            verbose: false,
        }
    }

    /// `MoeConfig::init` (src/moe/mod.rs:60-91): an empty layer on `device`
    /// with zero router and bias parameters; loaders fill them in.
    pub fn init(&self, device: &CudaDevice) -> MoeGatedSwiGLU {
        let cfg = sys::mxmoe_config {
            d_model: self.d_model as u32,
            ffn_hidden: self.ffn_hidden as u32,
            num_experts: self.num_experts as u32,
            experts_per_token: self.experts_per_token as u32,
            swiglu_alpha: self.swiglu_alpha,
            swiglu_limit: self.swiglu_limit,
            rms_eps: 1e-5,
            flags: if self.disabled { sys::MXMOE_FLAG_DISABLED } else { 0 },
            device: device.index,
        };
        let mut h: *mut sys::mxmoe_layer = ptr::null_mut();
        check_or_panic(unsafe { sys::mxmoe_create(&cfg, &mut h) });
        MoeGatedSwiGLU {
            norm: RmsNorm { gamma: vec![1.0; self.d_model], epsilon: 1e-5 },
            gate: Linear::zeros(self.d_model, self.num_experts),
            mlp1_bias: vec![0.0; self.num_experts * self.ffn_hidden * 2],
            mlp2_bias: vec![0.0; self.num_experts * self.d_model],
            num_experts: self.num_experts,
            experts_per_token: self.experts_per_token,
            swiglu_alpha: self.swiglu_alpha,
            swiglu_limit: self.swiglu_limit,
            d_model: self.d_model,
            ffn_hidden: self.ffn_hidden,
            disabled: self.disabled,
            verbose: self.verbose,
            resident: None,
            device: *device,
            layer: Arc::new(LayerHandle(h)),
            ready: false,
        }
    }
}

/// Burn's `RmsNorm` parameters (the MoE block's `norm`, src/moe/mod.rs:37).
#[derive(Debug, Clone)]
pub struct RmsNorm {
    pub gamma: Vec<f32>,
    pub epsilon: f32,
}

/// Burn's `Linear` parameters as Burn stores them: weight [d_input][d_output].
#[derive(Debug, Clone)]
pub struct Linear {
    pub weight: Vec<f32>,
    pub bias: Option<Vec<f32>>,
    pub d_input: usize,
    pub d_output: usize,
}

impl Linear {
    pub fn zeros(d_input: usize, d_output: usize) -> Self {
        Self { weight: vec![0.0; d_input * d_output], bias: Some(vec![0.0; d_output]), d_input, d_output }
    }

    /// Output-major [d_output][d_input], the layout of the library's router.
    fn weight_output_major(&self) -> Vec<f32> {
        let mut w = vec![0.0f32; self.weight.len()];
        for i in 0..self.d_input {
            for o in 0..self.d_output {
                w[o * self.d_input + i] = self.weight[i * self.d_output + o];
            }
        }
        w
    }
}

/// Owns one libmxmoe layer (destroyed with the last clone of the module).
#[derive(Debug)]
pub(crate) struct LayerHandle(pub(crate) *mut sys::mxmoe_layer);
unsafe impl Send for LayerHandle {}
unsafe impl Sync for LayerHandle {}
impl Drop for LayerHandle {
    fn drop(&mut self) {
        if !self.0.is_null() {
            unsafe {
                sys::mxmoe_destroy(self.0);
            }
        }
    }
}

/// `moe::MoeGatedSwiGLU` (src/moe/mod.rs:35-57).  The MXFP4 block and scale
/// tensors live in `resident`, as the reference's fast path expects; the
/// biases are host parameters uploaded with them.
#[derive(Debug, Clone)]
pub struct MoeGatedSwiGLU {
    pub norm: RmsNorm,
    pub gate: Linear,
    /// [E][2 * ffn_hidden] (split-half rows: GLU then linear, as src/quant/gpu.rs:108-113 reads)
    pub mlp1_bias: Vec<f32>,
    /// [E][d_model]
    pub mlp2_bias: Vec<f32>,
    pub num_experts: usize,
    pub experts_per_token: usize,
    pub swiglu_alpha: f32,
    pub swiglu_limit: f32,
    pub d_model: usize,
    pub ffn_hidden: usize,
    pub disabled: bool,
    pub verbose: bool,
    pub resident: Option<SharedResident>,
    pub device: CudaDevice,
    pub(crate) layer: Arc<LayerHandle>,
    pub(crate) ready: bool,
}

impl MoeGatedSwiGLU {
    /// `set_resident` (src/moe/mod.rs:95-97): attaches the quantized experts
    /// and uploads them, with the router and biases, into the library.
    pub fn set_resident(&mut self, res: Arc<MoeQuantLayerResident>) {
        self.try_set_resident(res).unwrap_or_else(|e| panic!("{e}"));
    }

    pub fn try_set_resident(&mut self, res: Arc<MoeQuantLayerResident>) -> Result<(), MxMoeError> {
        self.upload_router()?;
        let w1 = res.w1.desc.to_c();
        let w2 = res.w2.desc.to_c();
        unsafe {
            check(sys::mxmoe_upload_experts(
                self.layer.0,
                &w1,
                res.w1.blocks_host.as_ptr(),
                res.w1.scales_host.as_ptr(),
                &w2,
                res.w2.blocks_host.as_ptr(),
                res.w2.scales_host.as_ptr(),
                self.mlp1_bias.as_ptr() as *const c_void,
                self.mlp2_bias.as_ptr() as *const c_void,
                sys::MXMOE_F32,
                ptr::null_mut(),
            ))?;
        }
        self.resident = Some(res);
        self.ready = true;
        Ok(())
    }

    /// Re-uploads `norm` and `gate` after they change (the loaders set them
    /// before `set_resident`, which uploads them too).
    pub fn upload_router(&mut self) -> Result<(), MxMoeError> {
        let w = self.gate.weight_output_major();
        let b = self.gate.bias.clone().unwrap_or_else(|| vec![0.0; self.num_experts]);
        unsafe {
            check(sys::mxmoe_set_router(
                self.layer.0,
                self.norm.gamma.as_ptr() as *const c_void,
                w.as_ptr() as *const c_void,
                b.as_ptr() as *const c_void,
                sys::MXMOE_F32,
                ptr::null_mut(),
            ))
        }
    }

    /// `MoeGatedSwiGLU::forward` (src/moe/mod.rs:99-115): y = x + MoE(RmsNorm(x)),
    /// same shape and element type as x.
    pub fn forward(&self, x: DeviceTensor<3>) -> DeviceTensor<3> {
        if self.disabled {
            return x;
        }
        if !self.ready {
            panic!("MoE resident buffers missing; fastest path requires device-resident weights");
        }
        assert_eq!(x.device(), self.device.index, "input on another device");
        let [b, t, d] = x.dims();
        assert_eq!(d, self.d_model, "d_model mismatch");
        let mut y = DeviceTensor::<3>::empty([b, t, d], x.dtype(), x.device()).unwrap_or_else(|e| panic!("{e}"));
        unsafe {
            check_or_panic(sys::mxmoe_forward(
                self.layer.0,
                x.as_ptr(),
                x.dtype().code(),
                y.as_mut_ptr(),
                y.dtype().code(),
                (b * t) as u32,
                ptr::null_mut(),
            ));
        }
        y
    }

    /// The library handle (for the expert-parallel and profiling entry points).
    pub fn raw(&self) -> *mut sys::mxmoe_layer {
        self.layer.0
    }

    /// A layer created and loaded by the library itself (model.bin reader).
    pub(crate) fn from_loaded(handle: *mut sys::mxmoe_layer, cfg: sys::mxmoe_config) -> Self {
        let (d, f, e) = (cfg.d_model as usize, cfg.ffn_hidden as usize, cfg.num_experts as usize);
        Self {
            norm: RmsNorm { gamma: Vec::new(), epsilon: cfg.rms_eps },
            gate: Linear { weight: Vec::new(), bias: None, d_input: d, d_output: e },
            mlp1_bias: Vec::new(),
            mlp2_bias: Vec::new(),
            num_experts: e,
            experts_per_token: cfg.experts_per_token as usize,
            swiglu_alpha: cfg.swiglu_alpha,
            swiglu_limit: cfg.swiglu_limit,
            d_model: d,
            ffn_hidden: f,
            disabled: cfg.flags & sys::MXMOE_FLAG_DISABLED != 0,
            verbose: false,
            resident: None,
            device: CudaDevice::new(cfg.device),
            layer: Arc::new(LayerHandle(handle)),
            ready: true,
        }
    }
}

/// Convenience for tests and examples: a bf16 device tensor from f32 host
/// values (round to nearest even).
pub fn bf16_tensor(values: &[f32], shape: [usize; 3], device: i32) -> DeviceTensor<3> {
    let bits: Vec<u16> = values.iter().map(|v| half::bf16::from_f32(*v).to_bits()).collect();
    DeviceTensor::from_host(&bits, shape, DType::BF16, device).unwrap_or_else(|e| panic!("{e}"))
}
