"""Regenerates tests/golden/tiny_seed0.npz: the BASELINE tiny configuration
(d = f = 256, 2 experts, top-2, 16 tokens, f32 activations, seed 0) with the
CPU oracle's routing and layer output.

    python tests/golden/make_golden.py

The reference crate cannot run here (Rust + wgpu), so these vectors freeze
the oracle's restatement; the oracle itself is pinned only by the reference's
dequant known-answer test (tests/mxfp4_dequant_tests.rs).  Inputs are drawn by
mxmoe.synth (numpy PCG64, seed 0).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "burn-extended_b200"), os.path.join(ROOT, "oracle")]

import oracle  # noqa: E402
from mxmoe import synth  # noqa: E402


def main():
    inp = synth.make_config("tiny", seed=0)
    out = {}
    for flags, tag in ((0, "split"), (oracle.FLAG_INTERLEAVED_GLU, "inter"), (oracle.FLAG_BIAS_PER_FTILE, "ftile")):
        c = oracle.cfg(inp.d, inp.f, inp.E, inp.k, flags=flags)
        y, idx, w = oracle.moe_forward(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.host.w1_blocks,
                                       inp.host.w1_scales, inp.b1, inp.host.w2_blocks, inp.host.w2_scales, inp.b2)
        out[f"y_{tag}"] = y
        out["topk_idx"], out["topk_w"] = idx, w
    r = oracle.route(oracle.cfg(inp.d, inp.f, inp.E, inp.k), inp.x, inp.gamma, inp.gate_w, inp.gate_b)
    out["logits"] = r["logits"]
    out["rscale"] = r["rscale"]
    offs, perm, inv = oracle.permute(r["topk_idx"], inp.E)
    out["offsets"], out["perm"], out["inv"] = offs, perm, inv
    deq = oracle.dequant_rows(inp.host.w1_blocks.reshape(-1, inp.d // 2), inp.host.w1_scales.reshape(-1, inp.d // 32),
                              inp.E * 2 * inp.f, inp.d)
    out["w1_dequant_row0_64"] = deq[:64].copy()
    np.savez_compressed(os.path.join(HERE, "tiny_seed0.npz"), x=inp.x, gate_w=inp.gate_w, gate_b=inp.gate_b,
                        w1_blocks=inp.host.w1_blocks, w1_scales=inp.host.w1_scales, w2_blocks=inp.host.w2_blocks,
                        w2_scales=inp.host.w2_scales, b1=inp.b1, b2=inp.b2, **out)
    print("wrote", os.path.join(HERE, "tiny_seed0.npz"))


if __name__ == "__main__":
    main()
