"""Seeded synthetic inputs for the BASELINE configurations.

No public dataset or checkpoint is involved: every tensor is drawn here with
the shapes and value distributions the benchmark configurations state
(activations ~N(0,1), router ~N(0,0.02), E2M1 codes uniform in 0..15,
E8M0 scales uniform in 118..130, biases ~N(0,0.02), RmsNorm gain 1).  bf16
tensors are drawn in f32 and rounded to nearest even; the CPU oracle consumes
the rounded values.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import MoeQuantLayerHost, QuantLinearMxFp4Desc


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round f32 to the nearest bf16 value (ties to even), returned as f32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


@dataclass
class MoeInputs:
    d: int
    f: int
    E: int
    k: int
    n: int
    x: np.ndarray            # [n, d] f32 (bf16-exact when bf16=True)
    gamma: np.ndarray        # [d]
    gate_w: np.ndarray       # [E, d]
    gate_b: np.ndarray       # [E]
    host: MoeQuantLayerHost
    b1: np.ndarray           # [E, 2f]
    b2: np.ndarray           # [E, d]
    bf16: bool

    def x_bf16_bits(self) -> np.ndarray:
        return f32_to_bf16_bits(self.x)


# name -> (d, f, E, k, n, bf16 activations)
CONFIGS = {
    "tiny": (256, 256, 2, 2, 16, False),
    "microbench": (2880, 2880, 1, 1, 8, True),     # configs[1] (T = 1, 2, 4, 8)
    "decode": (2880, 2880, 32, 4, 64, True),       # configs[2]
    "prefill": (2880, 2880, 32, 4, 8192, True),    # configs[3]
    "gptoss120b": (2880, 2880, 128, 4, 4096, True),  # configs[4]
}


def make_inputs(d: int, f: int, E: int, k: int, n: int, bf16: bool, seed: int = 0,
                zipf_router_bias: Optional[float] = None, scale_lo: int = 118, scale_hi: int = 130,
                ue8_offset: int = 0) -> MoeInputs:
    rng = np.random.default_rng(seed)
    rnd = bf16_round if bf16 else (lambda a: np.asarray(a, dtype=np.float32))
    x = rnd(rng.standard_normal((n, d), dtype=np.float32))
    gate_w = rnd(rng.normal(0.0, 0.02, (E, d)).astype(np.float32))
    gate_b = np.zeros(E, dtype=np.float32)
    if zipf_router_bias is not None:
        # logit bias -s * ln(e + 1): expert load roughly Zipf(s)
        gate_b = rnd((-zipf_router_bias * np.log(np.arange(E) + 1.0)).astype(np.float32))
    w1_blocks = rng.integers(0, 256, size=(E, 2 * f, d // 2), dtype=np.uint8)
    w1_scales = (rng.integers(scale_lo, scale_hi + 1, size=(E, 2 * f, d // 32)) + ue8_offset).astype(np.uint8)
    w2_blocks = rng.integers(0, 256, size=(E, d, f // 2), dtype=np.uint8)
    w2_scales = (rng.integers(scale_lo, scale_hi + 1, size=(E, d, f // 32)) + ue8_offset).astype(np.uint8)
    b1 = rnd(rng.normal(0.0, 0.02, (E, 2 * f)).astype(np.float32))
    b2 = rnd(rng.normal(0.0, 0.02, (E, d)).astype(np.float32))
    host = MoeQuantLayerHost(
        QuantLinearMxFp4Desc.for_shape(E, 2 * f, d, ue8_offset), QuantLinearMxFp4Desc.for_shape(E, d, f, ue8_offset),
        w1_blocks, w1_scales, w2_blocks, w2_scales)
    return MoeInputs(d, f, E, k, n, x, np.ones(d, dtype=np.float32), gate_w, gate_b, host, b1, b2, bf16)


def rank_tokens(inp: MoeInputs, rank: int, seed: int = 0) -> MoeInputs:
    """The same layer (router, experts, biases) with this rank's own tokens:
    every expert-parallel rank must hold one shared model, only x differs."""
    from dataclasses import replace
    rng = np.random.default_rng(10_000 + 7919 * rank + seed)
    x = rng.standard_normal(inp.x.shape, dtype=np.float32)
    return replace(inp, x=bf16_round(x) if inp.bf16 else x)


def make_config(name: str, seed: int = 0, n: Optional[int] = None) -> MoeInputs:
    d, f, E, k, n0, bf16 = CONFIGS[name]
    zipf = 1.1 if name == "gptoss120b" else None
    return make_inputs(d, f, E, k, n if n is not None else n0, bf16, seed, zipf_router_bias=zipf)
