"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Bit-exact: dequantized weights, router logits, top-k indices, permutation
maps.  Layer outputs: the tolerance in moe_testutil (max-abs 2e-2 and
relative L2 1e-2 of the output scale)."""
import numpy as np
import pytest

import mxmoe
import oracle
from moe_testutil import assert_close, errors, make_layer, oracle_forward, to_device_x
from mxmoe import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


# ---------------------------------------------------------------- dequant
def test_dequant_kat_gpu(torch):
    # tests/mxfp4_dequant_tests.rs:4-25 through the device entry point
    blocks = torch.tensor([0x10, 0x21], dtype=torch.uint8, device="cuda")
    out = mxmoe.dequant_mxfp4_bytes(blocks, [1, 2], torch.tensor([127], dtype=torch.uint8, device="cuda"), [1])
    assert out.cpu().tolist() == [0.0, 0.5, 0.5, 1.0]
    out = mxmoe.dequant_mxfp4_bytes(blocks, [1, 2], torch.tensor([128], dtype=torch.uint8, device="cuda"), [1])
    assert out.cpu().tolist() == [0.0, 1.0, 1.0, 2.0]


def test_dequant_all_codes_all_scales_bit_exact(torch):
    blocks = np.tile(np.arange(256, dtype=np.uint8), 256)
    scales = np.arange(256, dtype=np.uint8)
    want = oracle.dequant_mxfp4_bytes(blocks, [256, 256], scales, [256])
    got = mxmoe.dequant_mxfp4_bytes(torch.from_numpy(blocks).cuda(), [256, 256], torch.from_numpy(scales).cuda(),
                                    [256]).cpu().numpy()
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_dequant_rows_gptoss_shape_bit_exact(torch):
    inp = synth.make_inputs(2880, 2880, 1, 1, 1, True, seed=2, ue8_offset=14)
    h = inp.host
    want = oracle.dequant_rows(h.w1_blocks.reshape(-1, 1440), h.w1_scales.reshape(-1, 90), 5760, 2880, 14)
    got = mxmoe.dequant_rows(h.w1_desc, torch.from_numpy(h.w1_blocks).cuda(), torch.from_numpy(h.w1_scales).cuda())
    assert np.array_equal(got.cpu().numpy().reshape(5760, 2880).view(np.uint32), want.view(np.uint32))


# ---------------------------------------------------------------- routing
def test_topk_softmax_on_oracle_logits(torch):
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((4096, 128)).astype(np.float32)
    logits[::7, 3] = logits[::7, 5]  # exact ties -> lower index first
    for k in (1, 2, 4, 8):
        want_i, want_w = oracle.topk_softmax(logits, k)
        gi, gw = mxmoe.topk_softmax(torch.from_numpy(logits).cuda(), k)
        assert np.array_equal(gi.cpu().numpy(), want_i)
        assert np.allclose(gw.cpu().numpy(), want_w, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("n,k,E", [(1, 1, 1), (5, 2, 2), (64, 4, 32), (8192, 4, 32), (4096, 4, 128), (3, 4, 8)])
def test_permute_bit_exact(torch, n, k, E):
    rng = np.random.default_rng(n + E)
    topk = np.stack([rng.permutation(E)[:k] for _ in range(n)]).astype(np.int32)
    want = oracle.permute(topk, E)
    got = mxmoe.permute(torch.from_numpy(topk).cuda(), E)
    for w, g in zip(want, got):
        assert np.array_equal(g.cpu().numpy(), w)


@pytest.mark.parametrize("n", [37, 5000])  # one-block and multi-block forms
def test_permute_rejects_ids_out_of_range(torch, n):
    rng = np.random.default_rng(n)
    E = 16
    topk = rng.integers(0, E, size=(n, 2)).astype(np.int32)
    topk[3, 1] = E        # past the last expert
    topk[n - 1, 0] = -4   # negative
    with pytest.raises(mxmoe.MxMoeError) as ei:
        mxmoe.permute(torch.from_numpy(topk).cuda(), E)
    assert ei.value.code == 1  # MXMOE_ERR_INVALID_ARG


def test_permute_all_to_one_expert_and_empty_experts(torch):
    topk = np.zeros((1000, 1), dtype=np.int32) + 5
    want = oracle.permute(topk, 16)
    got = mxmoe.permute(torch.from_numpy(topk).cuda(), 16)
    for w, g in zip(want, got):
        assert np.array_equal(g.cpu().numpy(), w)


@pytest.mark.parametrize("name,n", [("tiny", 16), ("decode", 64), ("gptoss120b", 256), ("prefill", 4500), ("gptoss120b", 4100)])
def test_router_bit_exact(torch, name, n):
    inp = synth.make_config(name, seed=0, n=n)
    layer = make_layer(inp)
    x = to_device_x(inp)
    layer.forward(x)
    rr = layer.routing_results(n)
    c = oracle.cfg(inp.d, inp.f, inp.E, inp.k)
    r = oracle.route(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b)
    assert np.array_equal(rr["logits"].cpu().numpy().reshape(n, inp.E).view(np.uint32), r["logits"].view(np.uint32))
    assert np.array_equal(rr["topk_idx"].cpu().numpy().reshape(n, inp.k), r["topk_idx"])
    assert np.allclose(rr["topk_w"].cpu().numpy().reshape(n, inp.k), r["topk_w"], rtol=2e-6, atol=1e-7)
    offs, perm, inv = oracle.permute(r["topk_idx"], inp.E)
    assert np.array_equal(rr["offsets"].cpu().numpy(), offs)
    assert np.array_equal(rr["perm"].cpu().numpy(), perm)
    assert np.array_equal(rr["inv"].cpu().numpy(), inv)
    layer.close()


def _check_routing(layer, inp, x, n):
    layer.forward(x)
    rr = layer.routing_results(n)
    r = oracle.route(oracle.cfg(inp.d, inp.f, inp.E, inp.k), inp.x, inp.gamma, inp.gate_w, inp.gate_b)
    assert np.array_equal(rr["logits"].cpu().numpy().reshape(n, inp.E).view(np.uint32), r["logits"].view(np.uint32))
    assert np.array_equal(rr["topk_idx"].cpu().numpy().reshape(n, inp.k), r["topk_idx"])
    # canonical maps (pair counts >= 2048 take the multi-block permutation)
    offs, perm, inv = oracle.permute(r["topk_idx"], inp.E)
    assert np.array_equal(rr["offsets"].cpu().numpy(), offs)
    assert np.array_equal(rr["perm"].cpu().numpy(), perm)
    assert np.array_equal(rr["inv"].cpu().numpy(), inv)
    import torch as t
    rs = t.empty(n, dtype=t.float32, device=x.device)
    ti = t.empty(n, inp.k, dtype=t.int32, device=x.device)
    tw = t.empty(n, inp.k, dtype=t.float32, device=x.device)
    layer.route(x, rs, ti, tw)
    assert np.array_equal(rs.cpu().numpy().view(np.uint32), r["rscale"].view(np.uint32))
    assert np.array_equal(ti.cpu().numpy(), r["topk_idx"])


# ragged column chunks (d % 128 != 0), token counts off the block tile, an
# expert count off the 32-expert groups, E = 1, f32 and bf16 activations, and
# both router tilings (n >= 2048 and below)
@pytest.mark.parametrize("d,E,k,n,bf16", [(2880, 32, 4, 2500, True), (96, 40, 2, 2100, False),
                                          (96, 1, 1, 37, True), (352, 72, 8, 300, False),
                                          (2880, 32, 4, 512, True), (2880, 20, 3, 300, False),
                                          (160, 7, 2, 5, False)])
def test_router_bit_exact_shapes(torch, d, E, k, n, bf16):
    inp = synth.make_inputs(d, 128, E, k, n, bf16, seed=d + E + n, zipf_router_bias=0.5)
    layer = make_layer(inp)
    _check_routing(layer, inp, to_device_x(inp), n)
    layer.close()


def test_router_bit_exact_misaligned_x(torch):
    # x starting 2 bytes past a 16-byte boundary: mxmoe_route takes the
    # router's plain-load path instead of cp.async; the full forward, whose
    # row kernels move 16-byte vectors, refuses such x with INVALID_ARG
    n = 70
    inp = synth.make_inputs(256, 128, 8, 2, n, True, seed=5)
    buf = torch.zeros(n * 256 + 8, dtype=torch.bfloat16, device="cuda")
    x = buf[1:1 + n * 256].view(n, 256)
    x.copy_(torch.from_numpy(inp.x).to(torch.bfloat16))
    assert x.data_ptr() % 16 != 0
    layer = make_layer(inp)
    r = oracle.route(oracle.cfg(inp.d, inp.f, inp.E, inp.k), inp.x, inp.gamma, inp.gate_w, inp.gate_b)
    rs = torch.empty(n, dtype=torch.float32, device="cuda")
    ti = torch.empty(n, inp.k, dtype=torch.int32, device="cuda")
    tw = torch.empty(n, inp.k, dtype=torch.float32, device="cuda")
    layer.route(x, rs, ti, tw)
    assert np.array_equal(rs.cpu().numpy().view(np.uint32), r["rscale"].view(np.uint32))
    assert np.array_equal(ti.cpu().numpy(), r["topk_idx"])
    with pytest.raises(mxmoe.MxMoeError) as ei:
        layer.forward(x)
    assert ei.value.code == 1  # MXMOE_ERR_INVALID_ARG
    torch.cuda.synchronize()
    layer.close()


# ---------------------------------------------------------------- layer
@pytest.mark.parametrize("simt", [False, True])
def test_tiny_layer_against_golden(torch, simt):
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "tiny_seed0.npz"))
    inp = synth.make_config("tiny", seed=0)
    layer = make_layer(inp, simt=simt)
    y = layer.forward(to_device_x(inp))
    layer.sync_status()
    assert_close(y.cpu().numpy(), z["y_split"], f"tiny simt={simt}")
    layer.close()


@pytest.mark.parametrize("flags,kw", [(oracle.FLAG_INTERLEAVED_GLU, dict(interleaved_glu=True)),
                                      (oracle.FLAG_BIAS_PER_FTILE, dict(bias_per_ftile=True)),
                                      (oracle.FLAG_NO_RESIDUAL, dict(residual=False))])
def test_layout_flags(torch, flags, kw):
    inp = synth.make_inputs(512, 384, 4, 2, 40, True, seed=9)
    want, _, _ = oracle_forward(inp, flags)
    layer = make_layer(inp, **kw)
    y = layer.forward(to_device_x(inp), out_dtype=torch.float32)
    layer.sync_status()
    assert_close(y.cpu().numpy(), want, str(kw))
    layer.close()


def test_zero_weights_residual_exact(torch):
    # tests/moe_basic_tests.rs:31-33
    inp = synth.make_inputs(256, 256, 4, 4, 6, False, seed=1)
    inp.host.w1_blocks[:] = 0
    inp.host.w2_blocks[:] = 0
    inp.b1[:] = 0
    inp.b2[:] = 0
    layer = make_layer(inp)
    x = to_device_x(inp)
    y = layer.forward(x)
    assert torch.equal(y, x)
    layer.close()


def test_disabled_is_identity(torch):
    inp = synth.make_inputs(256, 256, 2, 2, 8, True, seed=1)
    layer = make_layer(inp, disabled=True)
    x = to_device_x(inp)
    assert torch.equal(layer.forward(x), x)
    layer.close()


@pytest.mark.parametrize("simt", [False, True])
def test_decode_config_against_oracle(torch, simt):
    inp = synth.make_config("decode", seed=0)
    want, _, _ = oracle_forward(inp)
    layer = make_layer(inp, simt=simt)
    y = layer.forward(to_device_x(inp), out_dtype=torch.float32)
    layer.sync_status()
    assert_close(y.cpu().numpy(), want, f"decode simt={simt}")
    layer.close()


@pytest.mark.parametrize("fp4", [True, False])
@pytest.mark.parametrize("shape", [
    (2880, 2880, 32, 4, 64, True, False),    # decode config: 8 pairs per expert (16-pair tiles)
    (2880, 2880, 32, 4, 96, True, False),    # 12 per expert: 16-pair tiles, some experts need two
    (2880, 2880, 32, 4, 190, True, False),   # 23.75 pairs per expert: the last FP4 plan
    (512, 384, 4, 2, 40, False, True),       # f32 input, non-unit RmsNorm gain, 20 pairs per expert
    (1024, 320, 8, 4, 48, True, True),       # K not a multiple of 256 (last stage partial)
])
def test_decode_tile_paths(torch, shape, fp4):
    """Decode-sized batches on the kind::mxf4 tiles (four E2M1 activation
    terms) and on the E4M3 stacked tiles they replace."""
    d, f, E, k, n, bf16, gain = shape
    inp = synth.make_inputs(d, f, E, k, n, bf16, seed=n + E)
    if gain:
        inp.gamma = synth.bf16_round(1.0 + 0.25 * np.random.default_rng(7).standard_normal(d).astype(np.float32))
    want, idx, _ = oracle_forward(inp)
    layer = make_layer(inp, fp4_decode=fp4)
    y = layer.forward(to_device_x(inp), out_dtype=torch.float32)
    layer.sync_status()
    r = layer.routing_results(n)
    np.testing.assert_array_equal(r["topk_idx"].cpu().numpy().reshape(n, k), idx)
    assert_close(y.cpu().numpy(), want, f"{shape} fp4={fp4}")
    layer.close()


@pytest.mark.parametrize("T", [1, 2, 4, 8])
def test_microbench_single_expert(torch, T):
    inp = synth.make_inputs(2880, 2880, 1, 1, T, True, seed=T)
    want, _, _ = oracle_forward(inp)
    layer = make_layer(inp)
    y = layer.forward(to_device_x(inp), out_dtype=torch.float32)
    layer.sync_status()
    assert_close(y.cpu().numpy(), want, f"T={T}")
    layer.close()


def test_prefill_sample_and_properties(torch):
    # full 8192-token prefill on the GPU; the oracle checks a seeded sample of
    # tokens (each token's output depends only on its own row)
    inp = synth.make_config("prefill", seed=0)
    layer = make_layer(inp)
    x = to_device_x(inp)
    y = layer.forward(x, out_dtype=torch.float32)
    layer.sync_status()
    yn = y.cpu().numpy()
    assert np.isfinite(yn).all()
    rng = np.random.default_rng(1)
    sample = np.sort(rng.choice(inp.n, 48, replace=False))
    want, _, _ = oracle_forward(inp, x=inp.x[sample])
    assert_close(yn[sample], want, "prefill sample")
    # deterministic: a second forward is bit-identical
    y2 = layer.forward(x, out_dtype=torch.float32)
    assert torch.equal(y, y2)
    # permutation invariance: reversing tokens reverses outputs exactly
    y3 = layer.forward(x.flip(0).contiguous(), out_dtype=torch.float32)
    assert torch.equal(y3.flip(0), y)
    layer.close()


def test_gptoss120b_skewed_sample(torch):
    inp = synth.make_config("gptoss120b", seed=0, n=1024)
    layer = make_layer(inp)
    y = layer.forward(to_device_x(inp), out_dtype=torch.float32)
    layer.sync_status()
    rr = layer.routing_results(inp.n)
    counts = np.diff(rr["offsets"].cpu().numpy())
    assert counts.max() > 4 * max(1, counts.mean())  # the router bias skews the load
    sample = np.arange(0, inp.n, 32)
    want, _, _ = oracle_forward(inp, x=inp.x[sample])
    assert_close(y.cpu().numpy()[sample], want, "120b sample")
    layer.close()


def test_tc_matches_simt(torch):
    inp = synth.make_inputs(1024, 768, 8, 2, 300, True, seed=4)
    a = make_layer(inp)
    b = make_layer(inp, simt=True)
    x = to_device_x(inp)
    ya = a.forward(x, out_dtype=torch.float32).cpu().numpy()
    yb = b.forward(x, out_dtype=torch.float32).cpu().numpy()
    max_abs, rel = errors(ya, yb)
    assert max_abs < 2e-2 and rel < 1e-2, (max_abs, rel)
    a.close()
    b.close()


def test_forward_host_matches_device(torch):
    inp = synth.make_config("decode", seed=3)
    layer = make_layer(inp)
    x = to_device_x(inp)
    yd = layer.forward(x)
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    layer.forward_host(xh, yh)
    assert torch.equal(yh, yd.cpu())
    layer.close()


def test_forward_host_chunked_matches_device(torch):
    # 4096 tokens: four chunks whose copies overlap the neighbouring forwards
    inp = synth.make_inputs(1024, 512, 8, 4, 4096, True, seed=8)
    layer = make_layer(inp)
    x = to_device_x(inp)
    yd = layer.forward(x, out_dtype=torch.float32)
    xh = x.cpu().pin_memory()
    yh = torch.empty(xh.shape, dtype=torch.float32).pin_memory()
    layer.forward_host(xh, yh)
    assert torch.equal(yh, yd.cpu())
    layer.close()


def _gpu_count():
    try:
        import torch as t
        return t.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_forward_host_two_devices_one_thread(torch):
    # one host thread drives layers on two GPUs: each layer keeps its own
    # device staging buffers and streams
    inp = synth.make_config("decode", seed=5)
    want, _, _ = oracle_forward(inp)
    layers = [make_layer(inp, device=dev) for dev in (0, 1)]
    xh = torch.from_numpy(inp.x).to(torch.bfloat16).pin_memory()
    for _ in range(2):
        for L in layers:
            yh = torch.empty(xh.shape, dtype=torch.float32).pin_memory()
            L.forward_host(xh, yh)
            assert_close(yh.numpy(), want, f"forward_host on device {L.device}")
    for L in layers:
        L.close()


def test_errors_are_reported(torch):
    inp = synth.make_inputs(256, 256, 2, 2, 4, True, seed=1)
    cfg = mxmoe.MoeConfig(256, 256, 2, 2)
    layer = cfg.init(0)
    with pytest.raises(mxmoe.MxMoeError) as ei:
        layer.forward(to_device_x(inp))
    assert ei.value.code == 2  # NOT_READY (reference panics, src/moe/mod.rs:111-113)
    bad = synth.make_inputs(256, 128, 2, 2, 4, True, seed=1)
    with pytest.raises(mxmoe.MxMoeError):
        layer.set_resident(bad.host, bad.b1, bad.b2)
    layer.close()


@pytest.mark.parametrize("name,n", [("decode", 64), ("tiny", 16)])
def test_forward_graph_replay(torch, name, n):
    """Repeated forwards on the same x / out buffers: the first runs directly,
    the second is captured as a CUDA graph, later ones replay it.  New token
    values in x every call must give the oracle's output every call."""
    base = synth.make_config(name, seed=0, n=n)
    layer = make_layer(base)
    x = to_device_x(base)
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    for i in range(4):
        inp = synth.rank_tokens(base, i)
        x.copy_(torch.from_numpy(inp.x).to(x.dtype))
        layer.forward(x, out=y)
        want, _, _ = oracle_forward(inp)
        assert_close(y.cpu().numpy(), want, f"{name} call {i}")
    layer.close()
