//! `loader::mxfp4::dequant_mxfp4_bytes` (src/loader/mxfp4.rs:57-79) on the GPU:
//! out[r, 2i + {0, 1}] = FP4(lo / hi nibble of blocks[r, i]) * 2^(scales[r] - 127),
//! one scale per row of `b` bytes.  Bit-identical to the reference (exact
//! powers of two; the E2M1 values are exact in f32).
use crate::error::check_or_panic;
use crate::sys;
use crate::tensor::{DType, DeviceTensor};

/// Same signature as the reference; runs on CUDA device 0 (the layer
/// loaders use the layer's own device).
pub fn dequant_mxfp4_bytes(blocks: &[u8], blocks_shape: &[usize], scales: &[u8], scales_shape: &[usize]) -> Vec<f32> {
    dequant_mxfp4_bytes_on(0, blocks, blocks_shape, scales, scales_shape)
}

pub fn dequant_mxfp4_bytes_on(
    device: i32,
    blocks: &[u8],
    blocks_shape: &[usize],
    scales: &[u8],
    scales_shape: &[usize],
) -> Vec<f32> {
    let rows_total: usize = scales_shape.iter().product();
    let b = *blocks_shape.last().expect("blocks_shape is empty");
    assert!(blocks.len() >= rows_total * b && scales.len() >= rows_total, "buffers shorter than their shapes");
    if rows_total * b == 0 {
        return Vec::new();
    }
    // the byte buffers go up as 2-byte elements (little-endian: byte i lands at offset i)
    let blk = bytes_to_device(&blocks[..rows_total * b], device);
    let scl = bytes_to_device(&scales[..rows_total], device);
    let mut out = DeviceTensor::<1>::empty([rows_total * b * 2], DType::F32, device).expect("device buffer");
    unsafe {
        check_or_panic(sys::mxmoe_dequant_mxfp4_bytes(
            blk.as_ptr() as *const u8,
            rows_total as u64,
            b as u64,
            scl.as_ptr() as *const u8,
            out.as_mut_ptr() as *mut f32,
            std::ptr::null_mut(),
        ));
    }
    out.to_host::<f32>().expect("device to host copy")
}

/// A byte buffer on the device (as 2-byte elements, zero-padded to an even length).
fn bytes_to_device(bytes: &[u8], device: i32) -> DeviceTensor<1> {
    let mut padded: Vec<u16> = vec![0; (bytes.len() + 1) / 2];
    for (i, &v) in bytes.iter().enumerate() {
        padded[i / 2] |= (v as u16) << (8 * (i % 2));
    }
    DeviceTensor::<1>::from_host(&padded, [padded.len()], DType::BF16, device).expect("device buffer")
}
