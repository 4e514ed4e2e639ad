"""model.bin MoE reader (src/loader/modelbin.rs): header parsing and offset
walk on CPU, and on a GPU a loaded layer's forward against the oracle fed
with the same tensors."""
import os

import numpy as np
import pytest

import mxmoe
from mxmoe import modelbin, synth
from moe_testutil import assert_close, oracle_forward


@pytest.fixture
def torch():
    import torch
    return torch


def layer_tensors(inp: synth.MoeInputs, seed: int) -> modelbin.MoeLayerTensors:
    rng = np.random.default_rng(1000 + seed)
    norm = synth.bf16_round(1.0 + 0.1 * rng.standard_normal(inp.d).astype(np.float32))
    inp.gamma = norm
    bits = synth.f32_to_bf16_bits
    h = inp.host
    return modelbin.MoeLayerTensors(bits(norm), bits(inp.gate_w), bits(inp.gate_b), h.w1_blocks, h.w1_scales,
                                    bits(inp.b1), h.w2_blocks, h.w2_scales, bits(inp.b2))


def write_file(path, d, f, E, k, n_layers=2, n=16, **shape_kw):
    """Two (or more) synthetic layers; returns (per-layer inputs, payload offsets)."""
    inps, layers = [], []
    for l in range(n_layers):
        inp = synth.make_inputs(d, f, E, k, n, True, seed=l)
        layers.append(layer_tensors(inp, l))
        inps.append(inp)
    shape = modelbin.ModelBinShape(d, f, E, k, **shape_kw)
    payloads = modelbin.write_modelbin(str(path), shape, layers)
    return inps, payloads


def test_header_and_offsets(tmp_path):
    p = tmp_path / "model.bin"
    _, payloads = write_file(p, 64, 96, 3, 2, n_layers=3, num_text=13, num_special=3, regex=b"[a-z]+\0",
                             token_blob=b"xyzzy\0", swiglu_limit=6.5, rms_eps=2e-5, head_dim=8, num_heads=3,
                             num_kv_heads=1)
    h = modelbin.parse_modelbin(str(p))
    assert (h["num_blocks"], h["num_experts"], h["num_active_experts"], h["embedding_dim"], h["mlp_dim"]) == \
        (3, 3, 2, 64, 96)
    assert (h["head_dim"], h["num_heads"], h["num_kv_heads"]) == (8, 3, 1)
    assert (h["num_text_tokens"], h["num_special_tokens"]) == (13, 3)
    assert h["swiglu_limit"] == pytest.approx(6.5) and h["rms_eps"] == pytest.approx(2e-5)
    assert h["dense_offset"] % 16384 == 0 and h["file_bytes"] == os.path.getsize(p)
    # the reader's offset walk lands exactly on each layer's expert payload
    assert [h["moe_offset"] + l * h["moe_layer_stride"] for l in range(3)] == payloads


def test_bad_files_are_rejected(tmp_path):
    p = tmp_path / "model.bin"
    write_file(p, 64, 96, 2, 1)
    raw = p.read_bytes()
    bad = tmp_path / "bad_magic.bin"
    bad.write_bytes(b"GPT-OSS v0.9" + raw[12:])
    with pytest.raises(mxmoe.MxMoeError, match="magic"):
        modelbin.parse_modelbin(str(bad))
    with pytest.raises(mxmoe.MxMoeError, match="cannot open"):
        modelbin.parse_modelbin(str(tmp_path / "missing.bin"))
    short = tmp_path / "short.bin"
    short.write_bytes(raw[:-1])
    # the header still parses; loading the last layer finds its payload cut off
    assert modelbin.parse_modelbin(str(short))["num_blocks"] == 2
    with pytest.raises(mxmoe.MxMoeError, match="past the end"):
        modelbin.load_moe_layer(str(short), 1)
    with pytest.raises(mxmoe.MxMoeError, match="out of range"):
        modelbin.load_moe_layer(str(p), 2)
    with pytest.raises(mxmoe.MxMoeError, match="outside num_experts"):
        modelbin.load_moe_layer(str(p), 0, experts=(1, 2))


@pytest.mark.gpu
@pytest.mark.parametrize("d,f,E,k,n", [(256, 256, 4, 2, 16), (2880, 2880, 4, 2, 96)])
def test_loaded_layer_matches_oracle(torch, tmp_path, d, f, E, k, n):
    """Every layer of the file, loaded by the C reader (scales stored +14,
    bf16 router and biases), reproduces the oracle on the writer's tensors."""
    p = tmp_path / "model.bin"
    inps, _ = write_file(p, d, f, E, k, n_layers=2, n=n)
    for l, inp in enumerate(inps):
        layer = modelbin.load_moe_layer(str(p), l)
        assert (layer.cfg.d_model, layer.cfg.num_experts, layer.cfg.experts_per_token) == (d, E, k)
        x = torch.from_numpy(inp.x).to(torch.bfloat16).cuda()
        y = layer.forward(x, out_dtype=torch.float32)
        want, idx, _ = oracle_forward(inp)
        r = layer.routing_results(n)
        np.testing.assert_array_equal(r["topk_idx"].cpu().numpy().reshape(n, k), idx)
        assert_close(y.cpu().numpy(), want, f"layer {l}")
        layer.close()


@pytest.mark.gpu
def test_sharded_load_matches_full_load(torch, tmp_path):
    """A shard load reads only its experts: forward_local on the shard equals
    the full layer's pairs routed to those experts."""
    d, f, E, k, n = 256, 256, 4, 2, 32
    p = tmp_path / "model.bin"
    write_file(p, d, f, E, k, n_layers=1, n=n)
    full = modelbin.load_moe_layer(str(p), 0)
    part = modelbin.load_moe_layer(str(p), 0, experts=(2, 2))
    g = torch.Generator().manual_seed(3)
    xr = torch.randn(n, d, generator=g).to(torch.bfloat16).cuda()
    rscale = torch.ones(n, dtype=torch.float32, device="cuda")
    weight = torch.ones(n, dtype=torch.float32, device="cuda")
    expert = torch.tensor([2 + (i % 2) for i in range(n)], dtype=torch.int32, device="cuda")
    a = torch.empty(n, d, dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    full.forward_local(xr, rscale, expert, weight, a)
    part.forward_local(xr, rscale, expert, weight, b)
    torch.cuda.synchronize()
    assert_close(b.cpu().numpy(), a.cpu().numpy(), "shard vs full")
    full.close()
    part.close()
