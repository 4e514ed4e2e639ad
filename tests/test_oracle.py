"""CPU checks of the oracle (the checker the CUDA path is compared against).

Pinning: the reference's only known-answer test is the MXFP4 dequant KAT
(tests/mxfp4_dequant_tests.rs:4-25), reproduced verbatim below.  The rest of
the oracle restates src/moe/mod.rs and src/quant/gpu.rs; those tests check it
against independent numpy restatements on small cases and against the frozen
golden vectors of tests/golden/tiny_seed0.npz.
"""
import os

import numpy as np
import pytest

import oracle
from mxmoe import synth

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "tiny_seed0.npz")
LUT = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
               dtype=np.float32)


def test_dequant_known_answer_reference_kat():
    # tests/mxfp4_dequant_tests.rs:4-25
    blocks = np.array([0x10, 0x21], dtype=np.uint8)
    out = oracle.dequant_mxfp4_bytes(blocks, [1, 2], np.array([127], np.uint8), [1])
    assert out.tolist() == [0.0, 0.5, 0.5, 1.0]
    out2 = oracle.dequant_mxfp4_bytes(blocks, [1, 2], np.array([128], np.uint8), [1])
    assert out2.tolist() == [0.0, 1.0, 1.0, 2.0]


def _np_dequant_bytes(blocks, scales, b):
    rows = scales.size
    by = blocks.reshape(rows, b)
    lo, hi = LUT[by & 0xF], LUT[by >> 4]
    out = np.stack([lo, hi], axis=-1).reshape(rows, 2 * b)
    return (out * np.ldexp(np.float32(1.0), scales.astype(np.int32) - 127)[:, None].astype(np.float32)).ravel()


def test_dequant_all_codes_and_scales_bit_exact():
    # every byte value x every E8M0 exponent incl. subnormal range and 255 (inf)
    blocks = np.tile(np.arange(256, dtype=np.uint8), 256)
    scales = np.arange(256, dtype=np.uint8)
    got = oracle.dequant_mxfp4_bytes(blocks, [256, 256], scales, [256])
    with np.errstate(invalid="ignore", over="ignore"):
        want = _np_dequant_bytes(blocks, scales, 256)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    # -0.0 survives (byte 0x08 -> low nibble code 8, output element 16)
    assert np.signbit(got[16]) and got[16] == 0.0


def test_dequant_rows_matches_bytes_view():
    # MoE layout [rows][bpr] with gpr = cols/32 equals the [rows*gpr][16] view
    rng = np.random.default_rng(3)
    rows, cols = 7, 96
    blocks = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(100, 140, (rows, cols // 32), dtype=np.uint8)
    a = oracle.dequant_rows(blocks, scales, rows, cols)
    b = oracle.dequant_mxfp4_bytes(blocks, [rows * cols // 32, 16], scales, [rows * cols // 32])
    assert np.array_equal(a.ravel().view(np.uint32), b.view(np.uint32))


def test_dequant_ue8_offset():
    rng = np.random.default_rng(4)
    blocks = rng.integers(0, 256, (3, 32), dtype=np.uint8)
    scales = rng.integers(118, 131, (3, 2), dtype=np.uint8)
    a = oracle.dequant_rows(blocks, scales, 3, 64)
    b = oracle.dequant_rows(blocks, scales + 14, 3, 64, ue8_offset=14)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("g,l", [(0.0, 0.0), (10.0, 10.0), (-10.0, -10.0), (3.0, -2.0), (-400.0, 400.0),
                                 (7.0, 7.0), (6.999, -7.001)])
def test_swiglu_clamp_matches_formula(g, l):
    # src/quant/gpu.rs:140-145: glu clamped above only, linear both sides
    xg = min(np.float32(g), np.float32(7.0))
    xl = max(np.float32(-7.0), min(np.float32(l), np.float32(7.0)))
    want = np.float32(xg) * np.float32(1.0 / (1.0 + np.exp(-1.702 * xg))) * np.float32(xl + 1.0)
    got = oracle.swiglu(g, l)
    assert abs(got - want) <= 1e-5 * max(1.0, abs(want))


def test_topk_ties_lowest_index_and_softmax():
    logits = np.array([[1.0, 3.0, 3.0, 0.5], [2.0, 2.0, 2.0, 2.0]], np.float32)
    idx, w = oracle.topk_softmax(logits, 2)
    assert idx.tolist() == [[1, 2], [0, 1]]
    assert np.allclose(w, 0.5)
    idx, w = oracle.topk_softmax(np.array([[0.0, 1.0, -1.0]], np.float32), 3)
    assert idx.tolist() == [[1, 0, 2]]
    e = np.exp(np.array([0.0, -1.0, -2.0]))
    assert np.allclose(w[0], e / e.sum(), rtol=1e-6)


def test_permute_canonical_stable():
    rng = np.random.default_rng(5)
    n, k, E = 37, 3, 5
    topk = np.stack([rng.permutation(E)[:k] for _ in range(n)]).astype(np.int32)
    offsets, perm, inv = oracle.permute(topk, E)
    flat = topk.ravel()
    order = np.argsort(flat, kind="stable")
    assert np.array_equal(perm, order)
    assert np.array_equal(inv[perm], np.arange(n * k))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]))


def _np_route(x, gate_w, gate_b, eps=1e-5):
    # independent restatement of the pinned router order (lane chains + butterfly)
    n, d = x.shape
    E = gate_w.shape[0]

    def lane_sum(prod_fn):
        p = np.zeros(32, np.float32)
        for l in range(32):
            acc = np.float32(0)
            for c in range(l, d, 32):
                acc = np.float32(np.fma(*prod_fn(c), acc)) if hasattr(np, "fma") else _fma(*prod_fn(c), acc)
            p[l] = acc
        off = 16
        while off >= 1:
            p[:off] = (p[:off] + p[off:2 * off]).astype(np.float32)
            off //= 2
        return p[0]

    logits = np.zeros((n, E), np.float32)
    for t in range(n):
        xr = x[t]
        ss = lane_sum(lambda c: (xr[c], xr[c]))
        r = np.float32(1.0) / np.float32(np.sqrt(np.float32(np.float32(ss / np.float32(d)) + np.float32(eps))))
        nrm = ((xr * r).astype(np.float32) * np.float32(1.0)).astype(np.float32)
        for e in range(E):
            logits[t, e] = np.float32(lane_sum(lambda c: (nrm[c], gate_w[e, c])) + gate_b[e])
    return logits


def _fma(a, b, c):
    # exact fused multiply-add in float64 then single rounding (exact for f32 inputs)
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def test_router_logits_reproduce_pinned_order():
    inp = synth.make_inputs(64, 64, 4, 2, 3, bf16=True, seed=7)
    c = oracle.cfg(64, 64, 4, 2)
    r = oracle.route(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b)
    want = _np_route(inp.x, inp.gate_w, inp.gate_b)
    assert np.array_equal(r["logits"].view(np.uint32), want.view(np.uint32))


def test_zero_weights_give_residual():
    # tests/moe_basic_tests.rs:31-33: zero-initialised experts => y == x
    d, f, E, k, n = 64, 64, 4, 4, 6
    inp = synth.make_inputs(d, f, E, k, n, bf16=False, seed=1)
    zeros_b = np.zeros_like(inp.host.w1_blocks)
    y, _, _ = oracle.moe_forward(oracle.cfg(d, f, E, k), inp.x, inp.gamma, inp.gate_w, inp.gate_b, zeros_b,
                                 inp.host.w1_scales, np.zeros_like(inp.b1), np.zeros_like(inp.host.w2_blocks),
                                 inp.host.w2_scales, np.zeros_like(inp.b2))
    assert np.array_equal(y, inp.x)


def test_dense_reference_structure_equals_sparse():
    # the reference's dense per-expert loop (src/moe/mod.rs:279-404) computed in numpy
    d, f, E, k, n = 64, 96, 3, 2, 5
    inp = synth.make_inputs(d, f, E, k, n, bf16=False, seed=11)
    c = oracle.cfg(d, f, E, k)
    y, idx, w = oracle.moe_forward(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.host.w1_blocks,
                                   inp.host.w1_scales, inp.b1, inp.host.w2_blocks, inp.host.w2_scales, inp.b2)
    r = oracle.route(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b)
    acc = np.zeros((n, d), np.float64)
    for e in range(E):
        W1 = oracle.dequant_rows(inp.host.w1_blocks[e], inp.host.w1_scales[e], 2 * f, d).astype(np.float64)
        W2 = oracle.dequant_rows(inp.host.w2_blocks[e], inp.host.w2_scales[e], d, f).astype(np.float64)
        h = r["normed"].astype(np.float64) @ W1.T + inp.b1[e]
        g, l = h[:, :f], h[:, f:]
        xg = np.minimum(g, 7.0)
        xl = np.clip(l, -7.0, 7.0)
        act = xg / (1.0 + np.exp(-1.702 * xg)) * (xl + 1.0)
        out = act @ W2.T + inp.b2[e]
        wt = (w * (idx == e)).sum(1)
        acc += out * wt[:, None]
    ref = inp.x + acc
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err < 1e-4, err


def test_golden_fixture_regression():
    z = np.load(GOLDEN)
    inp = synth.make_config("tiny", seed=0)
    assert np.array_equal(z["x"], inp.x) and np.array_equal(z["w1_blocks"], inp.host.w1_blocks)
    c = oracle.cfg(inp.d, inp.f, inp.E, inp.k)
    y, idx, w = oracle.moe_forward(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.host.w1_blocks,
                                   inp.host.w1_scales, inp.b1, inp.host.w2_blocks, inp.host.w2_scales, inp.b2)
    assert np.array_equal(idx, z["topk_idx"])
    assert np.array_equal(y.view(np.uint32), z["y_split"].view(np.uint32))
    # Q2: bias per f tile equals bias once when f <= 256
    assert np.array_equal(z["y_split"], z["y_ftile"])
