//! The MoE part of `load_modelbin_into` (src/loader/modelbin.rs:158-462):
//! one layer's router and experts from a GPT-OSS v1.0 model.bin, read and
//! uploaded by the library (scale offset 14 removed, rows repacked).
use std::ffi::CString;
use std::ptr;

use crate::error::{check, MxMoeError};
use crate::moe::MoeGatedSwiGLU;
use crate::sys;

/// `parse_modelbin` (src/loader/modelbin.rs:75-156): the header fields.
pub fn modelbin_info(path: &str) -> Result<sys::mxmoe_modelbin_header, MxMoeError> {
    let c = CString::new(path).expect("path with an interior NUL");
    let mut h = sys::mxmoe_modelbin_header::default();
    check(unsafe { sys::mxmoe_modelbin_info(c.as_ptr(), &mut h) })?;
    Ok(h)
}

/// Layer `layer` on `device`; `experts = Some((begin, count))` loads one
/// expert shard (expert parallelism), `None` all experts.
pub fn load_moe_layer(
    path: &str,
    layer: u32,
    device: i32,
    flags: u32,
    experts: Option<(u32, u32)>,
) -> Result<MoeGatedSwiGLU, MxMoeError> {
    let c = CString::new(path).expect("path with an interior NUL");
    let (b, n) = experts.unwrap_or((0, 0));
    let mut h: *mut sys::mxmoe_layer = ptr::null_mut();
    check(unsafe { sys::mxmoe_modelbin_load_layer(c.as_ptr(), layer, device, flags, b, n, ptr::null_mut(), &mut h) })?;
    let mut cfg = sys::mxmoe_config::default();
    check(unsafe { sys::mxmoe_get_config(h, &mut cfg) })?;
    Ok(MoeGatedSwiGLU::from_loaded(h, cfg))
}
