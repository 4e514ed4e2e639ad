"""Accuracy of multi-term block-scaled activation operands (analysis tool,
test infrastructure: not on the product path).

The tensor-core expert GEMMs take the MXFP4 weights as stored and represent
each activation operand as a sum of T block-scaled terms: per 32-element
block, term t = code_t x 2^s_t, where 2^s_t is the smallest power of two that
fits the block's largest remaining value into the code format and the
residual after each term is exact.  This script models that on the CPU for
one GPT-OSS-20B-shaped layer (d = f = 2880, 32 experts, top-4, split-half W1,
the seeded synthetic inputs of mxmoe.synth) and reports the layer output
error against the unquantized f64 computation, for E2M1 (kind::mxf4) terms
T = 2, 3, 4 and E4M3 (kind::mxf8f6f4) terms T = 1, 2, with the bounds the
parity tests use: max|dy| / max|y| <= 2e-2 and ||dy|| / ||y|| <= 1e-2.

  python oracle/activation_terms.py [tokens] [seed]
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "burn-extended_b200"))

from mxmoe import synth  # noqa: E402

# E2M1 magnitudes by code (the format's definition; low nibble = even column)
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def dequant(blocks, scales, ue8_offset=0):
    """[E][rows][cols/2] codes + [E][rows][cols/32] E8M0 -> f64 [E][rows][cols]."""
    lo, hi = blocks & 0xF, blocks >> 4
    codes = np.stack([lo, hi], axis=-1).reshape(*blocks.shape[:-1], -1)
    val = E2M1[codes & 7] * np.where(codes & 8, -1.0, 1.0)
    sc = np.exp2(scales.astype(np.float64) - 127 - ue8_offset)
    return val * np.repeat(sc, 32, axis=-1)


def round_e2m1(v):
    """Nearest E2M1 value (ties to the even code), |v| <= 6."""
    a = np.abs(v)
    idx = np.abs(a[..., None] - E2M1).argmin(axis=-1)
    return np.sign(v) * E2M1[idx]


def round_e4m3(v):
    """Nearest E4M3 value (4 significant bits, min normal 2^-6, subnormal step 2^-9, max 448)."""
    a = np.abs(v)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -9)))
    e = np.maximum(e, -6)
    q = 2.0 ** (e - 3)
    return np.sign(v) * np.minimum(np.round(a / q) * q, 448.0)


def terms(x, fmt, T):
    """x [rows][K] -> the sum of T block-scaled terms of format fmt."""
    maxc, rnd = (6.0, round_e2m1) if fmt == "e2m1" else (448.0, round_e4m3)
    r = x.reshape(x.shape[0], -1, 32).astype(np.float64)
    out = np.zeros_like(r)
    for _ in range(T):
        amax = np.abs(r).max(axis=-1, keepdims=True)
        s = np.exp2(np.ceil(np.log2(np.maximum(amax, 1e-300) / maxc)))
        s = np.where(amax > 0, s, 1.0)
        q = rnd(r / s) * s
        out += q
        r = r - q
    return out.reshape(x.shape)


def layer(inp, W1, W2, xq=None, aq=None):
    """y = x + sum_k w * (W2 SwiGLU(W1 x_hat + b1) + b2), optional operand quantizers."""
    x = inp.x.astype(np.float64)
    d, f, k = inp.d, inp.f, inp.k
    rms = 1.0 / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-5)
    xn = x * rms * inp.gamma.astype(np.float64)
    logits = xn @ inp.gate_w.astype(np.float64).T + inp.gate_b.astype(np.float64)
    top = np.argsort(-logits, axis=1, kind="stable")[:, :k]
    tl = np.take_along_axis(logits, top, axis=1)
    w = np.exp(tl - tl.max(axis=1, keepdims=True))
    w /= w.sum(axis=1, keepdims=True)
    y = x.copy()
    for e in range(inp.E):
        tok, slot = np.nonzero(top == e)
        if tok.size == 0:
            continue
        xe = xn[tok]
        if xq:
            xe = xq(xe)
        h = xe @ W1[e].T + inp.b1[e].astype(np.float64)
        g, lin = np.minimum(h[:, :f], 7.0), np.clip(h[:, f:], -7.0, 7.0)
        with np.errstate(over="ignore"):  # exp overflow for very negative g: the product is -0
            act = g / (1.0 + np.exp(-1.702 * g)) * (lin + 1.0)
        if aq:
            act = aq(act)
        ye = act @ W2[e].T + inp.b2[e].astype(np.float64)
        y[tok] += w[tok, slot][:, None] * ye
    return y


def main():
    n = int(sys.argv[1]) if len(sys.argv) > 1 else 256
    seed = int(sys.argv[2]) if len(sys.argv) > 2 else 0
    inp = synth.make_config("prefill", seed=seed, n=n)
    h = inp.host
    W1 = dequant(h.w1_blocks, h.w1_scales)
    W2 = dequant(h.w2_blocks, h.w2_scales)
    ref = layer(inp, W1, W2)
    print(f"{n} tokens, GPT-OSS-20B shape, seed {seed}; bounds: max_rel 2e-2, rel_l2 1e-2")
    print(f"{'operand':<12} {'max|dy|/max|y|':>15} {'rel_l2':>10}  within")
    for fmt, T in (("e4m3", 1), ("e4m3", 2), ("e2m1", 2), ("e2m1", 3), ("e2m1", 4)):
        q = lambda a, fmt=fmt, T=T: terms(a, fmt, T)  # noqa: E731
        y = layer(inp, W1, W2, q, q)
        dy = y - ref
        mr = np.abs(dy).max() / np.abs(ref).max()
        rl = np.linalg.norm(dy) / np.linalg.norm(ref)
        print(f"{fmt} x {T:<5} {mr:15.3e} {rl:10.3e}  {'yes' if mr <= 2e-2 and rl <= 1e-2 else 'no'}")


if __name__ == "__main__":
    main()
