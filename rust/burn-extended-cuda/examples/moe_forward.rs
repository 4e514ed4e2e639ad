//! The reference's MoE call sequence through the drop-in: MoeConfig::init,
//! MoeQuantLayerResident::new, set_resident, forward.  Random GPT-OSS-style
//! weights (E2M1 codes uniform in 0..15, E8M0 scales 118..130), one decode
//! token; prints the first outputs.  Needs a CUDA device and libmxmoe.so.
use std::sync::Arc;

use burn_extended_cuda::moe::{bf16_tensor, MoeConfig};
use burn_extended_cuda::quant::{CudaDevice, MoeQuantLayerResident, QuantLinearMxFp4Desc};

fn lcg(state: &mut u64) -> u64 {
    *state = state.wrapping_mul(6364136223846793005).wrapping_add(1442695040888963407);
    *state >> 33
}

fn main() {
    let (d, f, e, k) = (512usize, 512usize, 8usize, 4usize);
    let device = CudaDevice::new(0);
    let cfg = MoeConfig::new(d, f, e, k);
    let mut mlp = cfg.init(&device);
    let mut s = 7u64;
    for w in mlp.gate.weight.iter_mut() {
        *w = ((lcg(&mut s) % 2001) as f32 - 1000.0) * 2e-5;
    }
    let w1 = QuantLinearMxFp4Desc::for_shape(e, 2 * f, d, 0);
    let w2 = QuantLinearMxFp4Desc::for_shape(e, d, f, 0);
    let bytes = |n: usize, s: &mut u64| (0..n).map(|_| (lcg(s) & 0xFF) as u8).collect::<Vec<u8>>();
    let scales = |n: usize, s: &mut u64| (0..n).map(|_| 118 + (lcg(s) % 13) as u8).collect::<Vec<u8>>();
    let res = MoeQuantLayerResident::new(
        &device,
        w1,
        bytes(e * 2 * f * w1.bpr, &mut s),
        scales(e * 2 * f * w1.gpr, &mut s),
        w2,
        bytes(e * d * w2.bpr, &mut s),
        scales(e * d * w2.gpr, &mut s),
    );
    mlp.set_resident(Arc::new(res));
    let x: Vec<f32> = (0..d).map(|i| ((i * 37 % 101) as f32 - 50.0) / 25.0).collect();
    let y = mlp.forward(bf16_tensor(&x, [1, 1, d], device.index));
    let out: Vec<u16> = y.to_host().expect("copy back");
    let head: Vec<f32> = out.iter().take(8).map(|b| half::bf16::from_bits(*b).to_f32()).collect();
    println!("y[0..8] = {head:?}");
}
