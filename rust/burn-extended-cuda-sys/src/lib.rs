//! Raw bindings to `include/mxmoe.h` (ABI version 1), one `extern "C"`
//! declaration per entry point, plus the few CUDA runtime calls the safe
//! crate needs for device buffers.  Every `mxmoe_*` function returns an
//! `mxmoe_status` (0 = OK); the message of the last failure on the calling
//! thread comes from `mxmoe_last_error`.  Streams are `cudaStream_t` passed as
//! `*mut c_void` (null = the legacy default stream).
#![allow(non_camel_case_types)]

use core::ffi::{c_char, c_int, c_void};

pub const MXMOE_ABI_VERSION: c_int = 1;

pub type mxmoe_status = c_int;
pub const MXMOE_OK: mxmoe_status = 0;
pub const MXMOE_ERR_INVALID_ARG: mxmoe_status = 1;
pub const MXMOE_ERR_NOT_READY: mxmoe_status = 2;
pub const MXMOE_ERR_CUDA: mxmoe_status = 3;
pub const MXMOE_ERR_OOM: mxmoe_status = 4;
pub const MXMOE_ERR_UNSUPPORTED: mxmoe_status = 5;
pub const MXMOE_ERR_TIMEOUT: mxmoe_status = 6;
pub const MXMOE_ERR_TOO_LARGE: mxmoe_status = 7;

pub type mxmoe_dtype = c_int;
pub const MXMOE_F32: mxmoe_dtype = 0;
pub const MXMOE_BF16: mxmoe_dtype = 1;

pub const MXMOE_FLAG_INTERLEAVED_GLU: u32 = 0x1;
pub const MXMOE_FLAG_BIAS_PER_FTILE: u32 = 0x2;
pub const MXMOE_FLAG_NO_RESIDUAL: u32 = 0x4;
pub const MXMOE_FLAG_DISABLED: u32 = 0x8;
pub const MXMOE_FLAG_SIMT: u32 = 0x10;
pub const MXMOE_FLAG_NO_GRAPHS: u32 = 0x20;
pub const MXMOE_FLAG_NO_FP4: u32 = 0x40;
pub const MXMOE_FLAG_NO_GEMV: u32 = 0x80;

pub const MXMOE_FAULT_NONE: u32 = 0;
pub const MXMOE_FAULT_SKIP_SIGNAL: u32 = 1;

pub const MXMOE_IPC_HANDLE_BYTES: usize = 64;
pub const MXMOE_RETURN_FROM_EPILOGUE: u32 = 0x1;

/// Mirrors `moe::MoeConfig` (src/moe/mod.rs:22-33) plus the RmsNorm epsilon,
/// behaviour flags and the CUDA device.
#[repr(C)]
#[derive(Debug, Clone, Copy, Default)]
pub struct mxmoe_config {
    pub d_model: u32,
    pub ffn_hidden: u32,
    pub num_experts: u32,
    pub experts_per_token: u32,
    pub swiglu_alpha: f32,
    pub swiglu_limit: f32,
    pub rms_eps: f32,
    pub flags: u32,
    pub device: i32,
}

/// Field-for-field `quant::QuantLinearMxFp4Desc` (src/quant/mod.rs:3-11).
#[repr(C)]
#[derive(Debug, Clone, Copy, Default)]
pub struct mxmoe_quant_desc {
    pub experts: u64,
    pub rows: u64,
    pub cols: u64,
    pub bpr: u64,
    pub gpr: u64,
    pub ue8_offset: i32,
}

/// Header fields of a GPT-OSS v1.0 model.bin (src/loader/modelbin.rs:75-151)
/// and the byte offsets derived from them.
#[repr(C)]
#[derive(Debug, Clone, Copy, Default)]
pub struct mxmoe_modelbin_header {
    pub context_length: u32,
    pub num_blocks: u32,
    pub num_experts: u32,
    pub num_active_experts: u32,
    pub embedding_dim: u32,
    pub mlp_dim: u32,
    pub swiglu_limit: f32,
    pub head_dim: u32,
    pub num_heads: u32,
    pub num_kv_heads: u32,
    pub attention_window: u32,
    pub rms_eps: f32,
    pub num_text_tokens: u32,
    pub num_special_tokens: u32,
    pub dense_offset: u64,
    pub moe_offset: u64,
    pub moe_layer_stride: u64,
    pub file_bytes: u64,
}

/// The caller's barrier for mxmoe_ep_forward (0 = success).
pub type mxmoe_ep_barrier_fn = Option<unsafe extern "C" fn(ctx: *mut c_void, stream: *mut c_void) -> c_int>;

/// Opaque layer handle.
#[repr(C)]
pub struct mxmoe_layer {
    _private: [u8; 0],
}

/// Streaming multi-query attention configuration (`mxmqa_config`).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct mxmqa_config {
    pub d_model: u32,
    pub n_heads: u32,
    pub kv_heads: u32,
    pub head_dim: u32,
    pub flags: u32,
    pub device: i32,
}

/// RoPE with NTK/YaRN scaling (`mxmqa_rope`).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct mxmqa_rope {
    pub max_seq_len: u32,
    pub theta: f32,
    pub scaling_factor: f32,
    pub initial_context: f32,
    pub ntk_alpha: f32,
    pub ntk_beta: f32,
}

pub const MXMQA_FLAG_QUIET_SOFTMAX: u32 = 0x1;
pub const MXMQA_FLAG_PRE_SCALED_QK: u32 = 0x2;
pub const MXMQA_FLAG_ROPE_BY_HEAD: u32 = 0x4;

/// Opaque attention layer handle.
#[repr(C)]
pub struct mxmqa_layer {
    _private: [u8; 0],
}

/// Opaque streaming KV cache handle.
#[repr(C)]
pub struct mxmqa_cache {
    _private: [u8; 0],
}

extern "C" {
    pub fn mxmoe_abi_version() -> c_int;
    pub fn mxmoe_build_info() -> *const c_char;
    pub fn mxmoe_last_error(buf: *mut c_char, cap: usize) -> c_int;

    pub fn mxmoe_create(cfg: *const mxmoe_config, out: *mut *mut mxmoe_layer) -> c_int;
    pub fn mxmoe_fp4_operands(layer: *mut mxmoe_layer, ptrs: *mut *mut c_void, rows4: *mut u32) -> c_int;
    pub fn mxmoe_get_config(layer: *const mxmoe_layer, out: *mut mxmoe_config) -> c_int;
    pub fn mxmoe_destroy(layer: *mut mxmoe_layer) -> c_int;
    pub fn mxmoe_set_router(
        layer: *mut mxmoe_layer,
        norm_gamma: *const c_void,
        gate_w: *const c_void,
        gate_b: *const c_void,
        dtype: mxmoe_dtype,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_upload_experts(
        layer: *mut mxmoe_layer,
        w1_desc: *const mxmoe_quant_desc,
        w1_blocks: *const u8,
        w1_scales: *const u8,
        w2_desc: *const mxmoe_quant_desc,
        w2_blocks: *const u8,
        w2_scales: *const u8,
        b1: *const c_void,
        b2: *const c_void,
        bias_dtype: mxmoe_dtype,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_reserve(layer: *mut mxmoe_layer, max_tokens: u32) -> c_int;
    pub fn mxmoe_forward(
        layer: *mut mxmoe_layer,
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        y: *mut c_void,
        y_dtype: mxmoe_dtype,
        n_tokens: u32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_forward_host(
        layer: *mut mxmoe_layer,
        x_host: *const c_void,
        x_dtype: mxmoe_dtype,
        y_host: *mut c_void,
        y_dtype: mxmoe_dtype,
        n_tokens: u32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_routing_results(
        layer: *mut mxmoe_layer,
        topk_idx: *mut *const i32,
        topk_w: *mut *const f32,
        offsets: *mut *const i32,
        perm: *mut *const i32,
        inv: *mut *const i32,
        logits: *mut *const f32,
    ) -> c_int;
    pub fn mxmoe_dequant_mxfp4_bytes(
        blocks: *const u8,
        rows_total: u64,
        b: u64,
        scales: *const u8,
        out: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_dequant_rows(
        desc: *const mxmoe_quant_desc,
        blocks: *const u8,
        scales: *const u8,
        out: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_topk_softmax(
        logits: *const f32,
        n_tokens: u32,
        num_experts: u32,
        k: u32,
        topk_idx: *mut i32,
        topk_w: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_permute(
        topk_idx: *const i32,
        n_tokens: u32,
        k: u32,
        num_experts: u32,
        offsets: *mut i32,
        perm: *mut i32,
        inv: *mut i32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_permute_noalloc(
        topk_idx: *const i32,
        n_tokens: u32,
        k: u32,
        num_experts: u32,
        offsets: *mut i32,
        perm: *mut i32,
        inv: *mut i32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_sync_status(layer: *mut mxmoe_layer, stream: *mut c_void) -> c_int;
    pub fn mxmoe_set_profiling(layer: *mut mxmoe_layer, enable: c_int) -> c_int;
    pub fn mxmoe_set_fault_injection(layer: *mut mxmoe_layer, mode: u32) -> c_int;
    pub fn mxmoe_last_profile(layer: *mut mxmoe_layer, ms: *mut f32, cap: c_int, count: *mut c_int) -> c_int;
    pub fn mxmoe_set_expert_shard(layer: *mut mxmoe_layer, expert_begin: u32, expert_count: u32) -> c_int;

    pub fn mxmoe_route(
        layer: *mut mxmoe_layer,
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        n_tokens: u32,
        rscale: *mut f32,
        topk_idx: *mut i32,
        topk_w: *mut f32,
        offsets: *mut i32,
        perm: *mut i32,
        inv: *mut i32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_gather_pairs(
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        n_tokens: u32,
        d_model: u32,
        k: u32,
        perm: *const i32,
        rscale: *const f32,
        topk_idx: *const i32,
        topk_w: *const f32,
        out_x: *mut c_void,
        out_meta: *mut u32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_forward_local(
        layer: *mut mxmoe_layer,
        xr: *const c_void,
        xr_dtype: mxmoe_dtype,
        rscale: *const f32,
        expert: *const i32,
        weight: *const f32,
        n_pairs: u32,
        out: *mut c_void,
        out_dtype: mxmoe_dtype,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_ipc_alloc(bytes: usize, device: c_int, ptr: *mut *mut c_void, handle: *mut c_void) -> c_int;
    pub fn mxmoe_ipc_free(ptr: *mut c_void, device: c_int) -> c_int;
    pub fn mxmoe_ipc_open(handle: *const c_void, device: c_int, peer_ptr: *mut *mut c_void) -> c_int;
    pub fn mxmoe_ipc_close(peer_ptr: *mut c_void, device: c_int) -> c_int;
    pub fn mxmoe_dispatch_pairs(
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        n_tokens: u32,
        d_model: u32,
        k: u32,
        perm: *const i32,
        rscale: *const f32,
        topk_idx: *const i32,
        topk_w: *const f32,
        offsets: *const i32,
        experts_per_rank: u32,
        world: u32,
        rank: u32,
        counts: *const i32,
        peer_x: *const *mut c_void,
        peer_meta: *const *mut u32,
        recv_cap: u32,
        err: *mut c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_forward_local_meta(
        layer: *mut mxmoe_layer,
        xr: *const c_void,
        xr_dtype: mxmoe_dtype,
        meta: *const u32,
        n_pairs: u32,
        ret_ptrs: *const *mut c_void,
        world: u32,
        ret_rows: u32,
        flags: u32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_ep_reserve(layer: *mut mxmoe_layer, max_tokens: u32, world: u32, handles: *mut c_void) -> c_int;
    pub fn mxmoe_ep_buffers(layer: *mut mxmoe_layer, ptrs: *mut *mut c_void) -> c_int;
    pub fn mxmoe_ep_dispatch(
        layer: *mut mxmoe_layer,
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        n_tokens: u32,
        rscale: *const f32,
        topk_idx: *const i32,
        topk_w: *const f32,
        inv: *const i32,
        offsets: *const i32,
        counts: *const i32,
        rank: u32,
        peer_bufs: *const *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_ep_attach(
        layer: *mut mxmoe_layer,
        rank: u32,
        world: u32,
        peer_bufs: *const *mut c_void,
        peer_ret: *const *mut c_void,
        peer_counts: *const *mut i32,
        barrier: mxmoe_ep_barrier_fn,
        barrier_ctx: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_ep_forward(
        layer: *mut mxmoe_layer,
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        n_tokens: u32,
        y: *mut c_void,
        y_dtype: mxmoe_dtype,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_ep_plan_replicas(loads: *const f64, num_experts: u32, extra: u32, src: *mut i32) -> c_int;
    pub fn mxmoe_ep_balanced_placement(loads: *const f64, num_experts: u32, world: u32, order: *mut i32) -> c_int;
    pub fn mxmoe_ep_experts(
        layer: *mut mxmoe_layer,
        x_dtype: mxmoe_dtype,
        peer_ret: *const *mut c_void,
        ret_rows: u32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmoe_combine(
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        n_tokens: u32,
        d_model: u32,
        k: u32,
        topk_idx: *const i32,
        inv: *const i32,
        pair_out: *const c_void,
        pair_dtype: mxmoe_dtype,
        residual: c_int,
        y: *mut c_void,
        y_dtype: mxmoe_dtype,
        stream: *mut c_void,
    ) -> c_int;

    pub fn mxmoe_modelbin_info(path: *const c_char, out: *mut mxmoe_modelbin_header) -> c_int;
    pub fn mxmoe_modelbin_load_layer(
        path: *const c_char,
        layer: u32,
        device: i32,
        flags: u32,
        expert_begin: u32,
        expert_count: u32,
        stream: *mut c_void,
        out: *mut *mut mxmoe_layer,
    ) -> c_int;
    pub fn mxmoe_safetensors_load_layer(
        paths: *const *const c_char,
        n_paths: u32,
        layer: u32,
        cfg: *const mxmoe_config,
        expert_begin: u32,
        expert_count: u32,
        stream: *mut c_void,
        out: *mut *mut mxmoe_layer,
    ) -> c_int;

    pub fn mxmqa_create(cfg: *const mxmqa_config, out: *mut *mut mxmqa_layer) -> c_int;
    pub fn mxmqa_destroy(layer: *mut mxmqa_layer) -> c_int;
    pub fn mxmqa_set_weights(
        layer: *mut mxmqa_layer,
        wq: *const c_void,
        bq: *const c_void,
        wk: *const c_void,
        bk: *const c_void,
        wv: *const c_void,
        bv: *const c_void,
        wo: *const c_void,
        bo: *const c_void,
        dtype: mxmoe_dtype,
        stream: *mut c_void,
    ) -> c_int;
    pub fn mxmqa_set_sinks(layer: *mut mxmqa_layer, sinks: *const f32) -> c_int;
    pub fn mxmqa_set_rope(layer: *mut mxmqa_layer, rope: *const mxmqa_rope) -> c_int;
    pub fn mxmqa_cache_create(
        layer: *const mxmqa_layer,
        batch: u32,
        cache_len: u32,
        sink_tokens: u32,
        out: *mut *mut mxmqa_cache,
    ) -> c_int;
    pub fn mxmqa_cache_reset(cache: *mut mxmqa_cache) -> c_int;
    pub fn mxmqa_cache_state(cache: *const mxmqa_cache, global_end: *mut u64, local_end: *mut u64) -> c_int;
    pub fn mxmqa_cache_destroy(cache: *mut mxmqa_cache) -> c_int;
    pub fn mxmqa_forward_streaming(
        layer: *mut mxmqa_layer,
        cache: *mut mxmqa_cache,
        x: *const c_void,
        x_dtype: mxmoe_dtype,
        batch: u32,
        seq_len: u32,
        start_pos: u64,
        window: u32,
        sinks: *const f32,
        attn_bias: *const f32,
        y: *mut c_void,
        y_dtype: mxmoe_dtype,
        stream: *mut c_void,
    ) -> c_int;
}

/// The CUDA runtime calls the safe crate uses for its device buffers (the
/// library links the same shared runtime).
pub mod cudart {
    use core::ffi::{c_int, c_void};

    pub type cudaError_t = c_int;
    pub const CUDA_SUCCESS: cudaError_t = 0;
    pub const CUDA_MEMCPY_HOST_TO_DEVICE: c_int = 1;
    pub const CUDA_MEMCPY_DEVICE_TO_HOST: c_int = 2;
    pub const CUDA_MEMCPY_DEVICE_TO_DEVICE: c_int = 3;

    extern "C" {
        pub fn cudaSetDevice(device: c_int) -> cudaError_t;
        pub fn cudaGetDevice(device: *mut c_int) -> cudaError_t;
        pub fn cudaMalloc(ptr: *mut *mut c_void, bytes: usize) -> cudaError_t;
        pub fn cudaFree(ptr: *mut c_void) -> cudaError_t;
        pub fn cudaMemcpy(dst: *mut c_void, src: *const c_void, bytes: usize, kind: c_int) -> cudaError_t;
        pub fn cudaDeviceSynchronize() -> cudaError_t;
    }
}
