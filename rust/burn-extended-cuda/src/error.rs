//! Status codes of libmxmoe as a Rust error, and the panic the reference's
//! `forward` raises where the library reports a failure.
use std::ffi::CStr;
use std::fmt;
use std::os::raw::c_char;

use crate::sys;

#[derive(Debug, Clone, PartialEq, Eq)]
pub struct MxMoeError {
    pub code: i32,
    pub message: String,
}

impl fmt::Display for MxMoeError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "mxmoe error {}: {}", self.code, self.message)
    }
}

impl std::error::Error for MxMoeError {}

/// The calling thread's last library message.
pub fn last_error() -> String {
    let mut buf = [0 as c_char; 512];
    unsafe {
        sys::mxmoe_last_error(buf.as_mut_ptr(), buf.len());
        CStr::from_ptr(buf.as_ptr()).to_string_lossy().into_owned()
    }
}

/// Turns a status into a `Result`.
pub fn check(code: i32) -> Result<(), MxMoeError> {
    if code == sys::MXMOE_OK {
        Ok(())
    } else {
        Err(MxMoeError { code, message: last_error() })
    }
}

/// The reference's behaviour for failures on the forward path: panic.
pub fn check_or_panic(code: i32) {
    if let Err(e) = check(code) {
        panic!("{e}");
    }
}

/// CUDA runtime status -> error (code MXMOE_ERR_CUDA).
pub fn cuda_check(code: i32, what: &str) -> Result<(), MxMoeError> {
    if code == sys::cudart::CUDA_SUCCESS {
        Ok(())
    } else {
        Err(MxMoeError { code: sys::MXMOE_ERR_CUDA, message: format!("{what} failed with CUDA error {code}") })
    }
}
