"""Shared helpers of the GPU parity tests."""
import numpy as np

import mxmoe
import oracle
from mxmoe import synth

# Tolerance of the MoE layer output against the f32 oracle (BASELINE north
# star: "within max-abs 2e-2 / rel 1e-2 in bf16"), measured relative to the
# output's own scale because the synthetic weights put |y| near 1e4:
#   max |y - y_ref| / max |y_ref|      <= 2e-2
#   ||y - y_ref||_2 / ||y_ref||_2      <= 1e-2
MAX_ABS_TOL = 2e-2
REL_L2_TOL = 1e-2


def errors(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    max_abs = np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)
    rel = np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)
    return float(max_abs), float(rel)


# (tag, max_abs, rel_l2) of every layer comparison in this session; conftest
# prints them at the end so the margin to the bounds is visible.
MARGINS = []


def assert_close(y, ref, tag=""):
    max_abs, rel = errors(y, ref)
    MARGINS.append((tag, max_abs, rel))
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, f"{tag}: max_abs={max_abs:.3e} rel_l2={rel:.3e}"
    return max_abs, rel


def make_layer(inp: synth.MoeInputs, device=0, **cfg_kw) -> mxmoe.MoeGatedSwiGLU:
    cfg = mxmoe.MoeConfig(inp.d, inp.f, inp.E, inp.k, **cfg_kw)
    layer = cfg.init(device)
    layer.set_router(inp.gamma, inp.gate_w, inp.gate_b)
    layer.set_resident(inp.host, inp.b1, inp.b2)
    return layer


def oracle_forward(inp: synth.MoeInputs, flags=0, x=None):
    c = oracle.cfg(inp.d, inp.f, inp.E, inp.k, flags=flags, ue8_offset=inp.host.w1_desc.ue8_offset)
    xx = inp.x if x is None else x
    return oracle.moe_forward(c, xx, inp.gamma, inp.gate_w, inp.gate_b, inp.host.w1_blocks, inp.host.w1_scales,
                              inp.b1, inp.host.w2_blocks, inp.host.w2_scales, inp.b2)


def to_device_x(inp: synth.MoeInputs, device=0):
    import torch
    if inp.bf16:
        return torch.from_numpy(inp.x).to(torch.bfloat16).to(f"cuda:{device}")
    return torch.from_numpy(inp.x).to(f"cuda:{device}")
