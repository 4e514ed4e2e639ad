"""GPU parity of the decode dequant-GEMV path (at most 8 routed pairs in a
forward, e.g. batch 1 at top-4): one fused kernel after the router runs the
expert FFN, the combine and the canonical routing maps.  Checked against the
CPU oracle, against the tensor-core path on the same inputs, and for
bit-identical repeats (direct launch, CUDA-graph capture, replay).

Covers the GPT-OSS-20B and -120B shapes at batch 1, the single-expert
microbench at T = 1..4, several pairs of a token batch on one expert, ragged
and wide K, non-unit RmsNorm gain with f32 input, and the layout flags."""
import numpy as np
import pytest

import oracle
from moe_testutil import assert_close, make_layer, oracle_forward, to_device_x
from mxmoe import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def run(torch, inp, tag, flags=0, **kw):
    want, idx, _ = oracle_forward(inp, flags)
    layer = make_layer(inp, **kw)
    x = to_device_x(inp)
    y = layer.forward(x, out_dtype=torch.float32)
    layer.sync_status()
    r = layer.routing_results(inp.n)
    np.testing.assert_array_equal(r["topk_idx"].cpu().numpy().reshape(inp.n, inp.k), idx)
    # the fused kernel writes the canonical maps itself (no permutation kernel)
    for got, ref in zip((r["offsets"], r["perm"], r["inv"]), oracle.permute(idx, inp.E)):
        np.testing.assert_array_equal(got.cpu().numpy(), ref)
    assert_close(y.cpu().numpy(), want, tag)
    # a second forward (CUDA-graph capture) and a third (replay) are bit-identical
    for _ in range(2):
        y2 = layer.forward(x, out_dtype=torch.float32)
        layer.sync_status()
        assert torch.equal(y, y2)
    layer.close()
    # the tensor-core path on the same inputs agrees within the same bounds
    tc = make_layer(inp, gemv_decode=False, **kw)
    yt = tc.forward(x, out_dtype=torch.float32)
    tc.sync_status()
    assert_close(y.cpu().numpy(), yt.cpu().numpy(), tag + " vs tensor-core path")
    tc.close()


def test_gptoss20b_batch1(torch):
    run(torch, synth.make_config("decode", seed=101, n=1), "dqgemv 20b decode n=1")


def test_gptoss20b_batch2(torch):
    # 8 routed pairs, the most the kernel takes
    run(torch, synth.make_config("decode", seed=102, n=2), "dqgemv 20b decode n=2")


@pytest.mark.parametrize("n,k", [(8, 1), (4, 2)])
def test_eight_pairs_on_one_expert(torch, n, k):
    inp = synth.make_inputs(1024, 512, 4, k, n, True, seed=40 + n)
    inp.gate_b = inp.gate_b.copy()
    inp.gate_b[0] = 50.0
    run(torch, inp, f"dqgemv one expert n={n} k={k}")


def test_gptoss120b_batch1(torch):
    run(torch, synth.make_config("gptoss120b", seed=201, n=1), "dqgemv 120b decode n=1")


@pytest.mark.parametrize("T", [1, 2, 3, 4])
def test_single_expert(torch, T):
    run(torch, synth.make_inputs(2880, 2880, 1, 1, T, True, seed=300 + T), f"dqgemv single expert T={T}")


@pytest.mark.parametrize("n,k", [(4, 1), (2, 2)])
def test_pairs_on_one_expert(torch, n, k):
    # a large router bias sends every token to expert 0 (and k - 1 others)
    inp = synth.make_inputs(1024, 512, 4, k, n, True, seed=n)
    inp.gate_b = inp.gate_b.copy()
    inp.gate_b[0] = 50.0
    run(torch, inp, f"dqgemv one expert n={n} k={k}")


@pytest.mark.parametrize("d,f", [(352, 96), (4096, 1024), (1024, 4096), (2880, 64)])
def test_ragged_and_wide_k(torch, d, f):
    run(torch, synth.make_inputs(d, f, 8, 2, 2, True, seed=d + f), f"dqgemv d={d} f={f}")


def test_f32_input_and_gain(torch):
    inp = synth.make_inputs(768, 640, 16, 4, 1, False, seed=5)
    inp.gamma = (1.0 + 0.5 * np.random.default_rng(3).standard_normal(768)).astype(np.float32)
    run(torch, inp, "dqgemv f32 x, gain")


@pytest.mark.parametrize("flags,kw", [(oracle.FLAG_INTERLEAVED_GLU, dict(interleaved_glu=True)),
                                      (oracle.FLAG_BIAS_PER_FTILE, dict(bias_per_ftile=True)),
                                      (oracle.FLAG_NO_RESIDUAL, dict(residual=False))])
def test_layout_flags_decode(torch, flags, kw):
    inp = synth.make_inputs(512, 384, 4, 2, 2, True, seed=19)
    run(torch, inp, f"dqgemv {kw}", flags, **kw)


def test_bf16_output(torch):
    inp = synth.make_config("decode", seed=7, n=1)
    layer = make_layer(inp)
    x = to_device_x(inp)
    y = layer.forward(x)  # bf16 out
    layer.sync_status()
    want, _, _ = oracle_forward(inp)
    assert_close(y.float().cpu().numpy(), want, "dqgemv bf16 out")
    layer.close()
