//! The reference's MXFP4 known-answer test (tests/mxfp4_dequant_tests.rs:4-25)
//! through the drop-in's device dequant.  Needs a CUDA device: run with
//! `cargo test -- --ignored`.
use burn_extended_cuda::loader::mxfp4::dequant_mxfp4_bytes;

#[test]
#[ignore = "needs a CUDA device and libmxmoe.so"]
fn dequant_known_answers() {
    let blocks = [0x10u8, 0x21];
    assert_eq!(dequant_mxfp4_bytes(&blocks, &[1, 2], &[127], &[1]), vec![0.0, 0.5, 0.5, 1.0]);
    assert_eq!(dequant_mxfp4_bytes(&blocks, &[1, 2], &[128], &[1]), vec![0.0, 1.0, 1.0, 2.0]);
}
