//! `attention::streaming_mqa` (src/attention/streaming_mqa.rs:12-435) over
//! libmxmoe's `mxmqa_*` entry points.
//!
//! Same names and call sequence as the reference:
//! `StreamingMultiQueryAttentionConfig::new(d_model, n_heads, kv_heads)
//! .with_quiet_softmax(..).init(device)`, `StreamingMqaCache::new(..)`,
//! `forward_streaming(x, &mut cache, StreamingMqaParams { .. })`.  Weights
//! come from the loaders as Burn keeps Linear layers ([d_in][d_out] +
//! bias); RoPE is a property of the module (`set_rope`) instead of a
//! per-call reference.  Failures panic with the library's message, as the
//! reference panics.
use std::ffi::c_void;
use std::ptr;

use crate::error::{check, check_or_panic, MxMoeError};
use crate::quant::CudaDevice;
use crate::sys;
use crate::tensor::{DType, DeviceTensor};

/// `AttnWindow` (src/attention/streaming.rs:14-19).
#[derive(Debug, Clone, Copy, PartialEq, Eq)]
pub enum AttnWindow {
    Full,
    Window(usize),
}

impl AttnWindow {
    fn code(self) -> u32 {
        match self {
            AttnWindow::Full => 0,
            AttnWindow::Window(w) => w as u32,
        }
    }
}

/// RoPE with the NTK/YaRN scaling of `init_ntk_yarn` (src/rope/mod.rs:11-50).
#[derive(Debug, Clone, Copy)]
pub struct RopeConfig {
    pub max_seq_len: usize,
    pub theta: f32,
    pub scaling_factor: f32,
    pub initial_context: f32,
    pub ntk_alpha: f32,
    pub ntk_beta: f32,
}

/// `StreamingMultiQueryAttentionConfig` (:12-42).
#[derive(Debug, Clone)]
pub struct StreamingMultiQueryAttentionConfig {
    pub d_model: usize,
    pub n_heads: usize,
    pub num_key_value_heads: usize,
    pub head_dim: usize,
    pub dropout: f64,
    pub quiet_softmax: bool,
    pub learned_sinks: bool,
    pub pre_scaled_qk: bool,
    /// Reproduce the reference's RoPE call, whose rotation index runs over heads.
    pub rope_by_head: bool,
}

impl StreamingMultiQueryAttentionConfig {
    pub fn new(d_model: usize, n_heads: usize, num_key_value_heads: usize) -> Self {
        Self {
            d_model,
            n_heads,
            num_key_value_heads,
            head_dim: d_model / n_heads,
            dropout: 0.0,
            quiet_softmax: false,
            learned_sinks: false,
            pre_scaled_qk: false,
            rope_by_head: false,
        }
    }
    pub fn with_dropout(mut self, p: f64) -> Self {
        self.dropout = p;
        self
    }
    pub fn with_quiet_softmax(mut self, q: bool) -> Self {
        self.quiet_softmax = q;
        self
    }
    pub fn with_head_dim(mut self, d: usize) -> Self {
        self.head_dim = d;
        self
    }
    pub fn with_learned_sinks(mut self, s: bool) -> Self {
        self.learned_sinks = s;
        self
    }
    pub fn with_pre_scaled_qk(mut self, s: bool) -> Self {
        self.pre_scaled_qk = s;
        self
    }

    /// `init` (:94-131): an attention module without weights; set them with
    /// `set_weights` (inference only, dropout must be 0).
    pub fn init(&self, device: &CudaDevice) -> StreamingMultiQueryAttention {
        assert!(self.dropout == 0.0, "inference only: dropout must be 0");
        let mut flags = 0u32;
        if self.quiet_softmax {
            flags |= sys::MXMQA_FLAG_QUIET_SOFTMAX;
        }
        if self.pre_scaled_qk {
            flags |= sys::MXMQA_FLAG_PRE_SCALED_QK;
        }
        if self.rope_by_head {
            flags |= sys::MXMQA_FLAG_ROPE_BY_HEAD;
        }
        let cfg = sys::mxmqa_config {
            d_model: self.d_model as u32,
            n_heads: self.n_heads as u32,
            kv_heads: self.num_key_value_heads as u32,
            head_dim: self.head_dim as u32,
            flags,
            device: device.index,
        };
        let mut h: *mut sys::mxmqa_layer = ptr::null_mut();
        check_or_panic(unsafe { sys::mxmqa_create(&cfg, &mut h) });
        StreamingMultiQueryAttention { handle: h, d_model: self.d_model, n_heads: self.n_heads, device: device.index }
    }
}

/// `StreamingMultiQueryAttention` (:44-74).
pub struct StreamingMultiQueryAttention {
    handle: *mut sys::mxmqa_layer,
    d_model: usize,
    n_heads: usize,
    device: i32,
}

unsafe impl Send for StreamingMultiQueryAttention {}

/// `StreamingMqaParams` (:205-218) without the RoPE reference (a module property here).
pub struct StreamingMqaParams<'a> {
    pub start_pos: usize,
    pub window: AttnWindow,
    /// Per-call sinks logits [n_heads] (device f32), instead of the module's.
    pub sinks: Option<&'a DeviceTensor<1>>,
    /// Additive bias [batch, n_heads, seq_len, active window] (device f32).
    pub attn_bias: Option<&'a DeviceTensor<4>>,
}

impl StreamingMultiQueryAttention {
    /// The query / key / value / output Linear layers as Burn stores them:
    /// weight [d_in][d_out] row-major, bias [d_out] (None = zero), f32 values.
    #[allow(clippy::too_many_arguments)]
    pub fn set_weights(
        &mut self,
        wq: &[f32],
        bq: Option<&[f32]>,
        wk: &[f32],
        bk: Option<&[f32]>,
        wv: &[f32],
        bv: Option<&[f32]>,
        wo: &[f32],
        bo: Option<&[f32]>,
    ) -> Result<(), MxMoeError> {
        let p = |b: Option<&[f32]>| b.map_or(ptr::null(), |s| s.as_ptr() as *const c_void);
        check(unsafe {
            sys::mxmqa_set_weights(
                self.handle,
                wq.as_ptr() as *const c_void,
                p(bq),
                wk.as_ptr() as *const c_void,
                p(bk),
                wv.as_ptr() as *const c_void,
                p(bv),
                wo.as_ptr() as *const c_void,
                p(bo),
                DType::F32.code(),
                ptr::null_mut(),
            )
        })
    }

    /// Learned sinks [kv_heads][groups] (`learned_sinks`, :117-124); None removes them.
    pub fn set_sinks(&mut self, sinks: Option<&[f32]>) -> Result<(), MxMoeError> {
        check(unsafe { sys::mxmqa_set_sinks(self.handle, sinks.map_or(ptr::null(), |s| s.as_ptr())) })
    }

    /// RoPE for every forward of this module; None = no rotation.
    pub fn set_rope(&mut self, rope: Option<RopeConfig>) -> Result<(), MxMoeError> {
        let r = rope.map(|r| sys::mxmqa_rope {
            max_seq_len: r.max_seq_len as u32,
            theta: r.theta,
            scaling_factor: r.scaling_factor,
            initial_context: r.initial_context,
            ntk_alpha: r.ntk_alpha,
            ntk_beta: r.ntk_beta,
        });
        check(unsafe { sys::mxmqa_set_rope(self.handle, r.as_ref().map_or(ptr::null(), |r| r as *const _)) })
    }

    /// `forward_streaming` (:239-435): x [batch, seq, d_model] -> same shape;
    /// writes the new keys and values into `cache`.
    pub fn forward_streaming(
        &self,
        x: DeviceTensor<3>,
        cache: &mut StreamingMqaCache,
        params: StreamingMqaParams<'_>,
    ) -> DeviceTensor<3> {
        let [b, t, d] = x.dims();
        assert_eq!(d, self.d_model, "x last dimension {} != d_model {}", d, self.d_model);
        if let Some(s) = params.sinks {
            assert_eq!(s.dims(), [self.n_heads], "sinks must be [n_heads]");
        }
        let mut y = DeviceTensor::<3>::empty([b, t, d], x.dtype(), self.device)
            .unwrap_or_else(|e| panic!("{}", e));
        check_or_panic(unsafe {
            sys::mxmqa_forward_streaming(
                self.handle,
                cache.handle,
                x.as_ptr(),
                x.dtype().code(),
                b as u32,
                t as u32,
                params.start_pos as u64,
                params.window.code(),
                params.sinks.map_or(ptr::null(), |s| s.as_ptr() as *const f32),
                params.attn_bias.map_or(ptr::null(), |s| s.as_ptr() as *const f32),
                y.as_mut_ptr(),
                y.dtype().code(),
                ptr::null_mut(),
            )
        });
        y
    }
}

impl Drop for StreamingMultiQueryAttention {
    fn drop(&mut self) {
        unsafe { sys::mxmqa_destroy(self.handle) };
    }
}

/// `StreamingMqaCache` (:132-203): keys and values of `cache_len` positions
/// per sequence, the first `sink_tokens` never evicted.
pub struct StreamingMqaCache {
    handle: *mut sys::mxmqa_cache,
}

unsafe impl Send for StreamingMqaCache {}

impl StreamingMqaCache {
    pub fn new(
        attn: &StreamingMultiQueryAttention,
        batch: usize,
        cache_len: usize,
        sink_tokens: usize,
    ) -> Result<Self, MxMoeError> {
        let mut h: *mut sys::mxmqa_cache = ptr::null_mut();
        check(unsafe {
            sys::mxmqa_cache_create(attn.handle, batch as u32, cache_len as u32, sink_tokens as u32, &mut h)
        })?;
        Ok(Self { handle: h })
    }
    /// `reset` (:169-173).
    pub fn reset(&mut self) {
        check_or_panic(unsafe { sys::mxmqa_cache_reset(self.handle) });
    }
    /// (global_end_index, local_end_index).
    pub fn state(&self) -> (u64, u64) {
        let (mut g, mut l) = (0u64, 0u64);
        check_or_panic(unsafe { sys::mxmqa_cache_state(self.handle, &mut g, &mut l) });
        (g, l)
    }
    pub fn len(&self) -> usize {
        self.state().1 as usize
    }
    pub fn is_empty(&self) -> bool {
        self.len() == 0
    }
}

impl Drop for StreamingMqaCache {
    fn drop(&mut self) {
        unsafe { sys::mxmqa_cache_destroy(self.handle) };
    }
}
