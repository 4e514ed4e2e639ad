"""GPT-OSS safetensors MoE loader (src/loader/gpt_oss.rs:369-423 with the
interleaved W1 rows of real checkpoints): header and error handling on CPU,
and on a GPU a layer loaded from a (multi-file) checkpoint against the
oracle run with the interleaved layout."""
import json
import struct

import numpy as np
import pytest

import mxmoe
import oracle
from mxmoe import safetensors as st
from mxmoe import synth
from moe_testutil import assert_close, oracle_forward


@pytest.fixture
def torch():
    import torch
    return torch


def checkpoint_tensors(inp: synth.MoeInputs, layer: int, float_dtype: str = "BF16"):
    """One layer's tensors under the GPT-OSS checkpoint names and shapes."""
    E, d, f = inp.E, inp.d, inp.f
    rng = np.random.default_rng(500 + layer)
    inp.gamma = synth.bf16_round(1.0 + 0.1 * rng.standard_normal(d).astype(np.float32))

    def fl(a):
        if float_dtype == "F32":
            return np.ascontiguousarray(a, dtype=np.float32)
        return ("BF16", synth.f32_to_bf16_bits(a))

    h = inp.host
    p = f"block.{layer}.mlp."
    return {
        p + "norm.scale": fl(inp.gamma),
        p + "gate.weight": fl(inp.gate_w),
        p + "gate.bias": fl(inp.gate_b),
        p + "mlp1_weight.blocks": h.w1_blocks.reshape(E, 2 * f, d // 32, 16),
        p + "mlp1_weight.scales": h.w1_scales.reshape(E, 2 * f, d // 32),
        p + "mlp1_bias": fl(inp.b1),
        p + "mlp2_weight.blocks": h.w2_blocks.reshape(E, d, f // 32, 16),
        p + "mlp2_weight.scales": h.w2_scales.reshape(E, d, f // 32),
        p + "mlp2_bias": fl(inp.b2),
    }


def make_checkpoint(tmp_path, d=64, f=96, E=3, k=2, n=16, n_layers=2, n_files=1, float_dtype="BF16"):
    inps, tensors = [], {}
    for l in range(n_layers):
        inp = synth.make_inputs(d, f, E, k, n, True, seed=20 + l)
        tensors.update(checkpoint_tensors(inp, l, float_dtype))
        inps.append(inp)
    names = list(tensors)
    paths = []
    for i in range(n_files):
        p = str(tmp_path / f"model-{i:05d}-of-{n_files:05d}.safetensors")
        st.write_safetensors(p, {nm: tensors[nm] for nm in names[i::n_files]},
                             metadata={"format": "pt", "note": "quote \" and \\u0041 escapes"})
        paths.append(p)
    return inps, paths


def test_writer_round_trip(tmp_path):
    _, paths = make_checkpoint(tmp_path)
    hdr = st.read_header(paths)
    assert hdr["block.1.mlp.mlp1_weight.blocks"]["shape"] == [3, 192, 2, 16]
    assert hdr["block.0.mlp.gate.weight"]["dtype"] == "BF16"


def test_bad_checkpoints_are_rejected(tmp_path):
    _, paths = make_checkpoint(tmp_path)
    with pytest.raises(mxmoe.MxMoeError, match="not found"):
        st.load_gptoss_moe_layer(paths, 2)
    with pytest.raises(mxmoe.MxMoeError, match="cannot open"):
        st.load_gptoss_moe_layer([str(tmp_path / "missing.safetensors")], 0)
    with pytest.raises(mxmoe.MxMoeError, match="config says"):
        mxmoe.lib()  # loads the library before the failing call below
        import ctypes
        arr = (ctypes.c_char_p * 1)(paths[0].encode())
        c = mxmoe._lib.Config(128, 0, 0, 2, 1.702, 7.0, 1e-5, 0, 0)
        h = ctypes.c_void_p()
        mxmoe.check(mxmoe.lib().mxmoe_safetensors_load_layer(arr, 1, 0, ctypes.byref(c), 0, 0, None,
                                                             ctypes.byref(h)))
    with pytest.raises(mxmoe.MxMoeError, match="outside num_experts"):
        st.load_gptoss_moe_layer(paths, 0, experts=(2, 2))

    # a wrong shape, a wrong dtype, a truncated data section, a broken header
    d, f, E = 64, 96, 3
    inp = synth.make_inputs(d, f, E, 2, 4, True, seed=1)
    good = checkpoint_tensors(inp, 0)
    bad = dict(good)
    bad["block.0.mlp.mlp2_weight.scales"] = np.zeros((E, d, f // 32 + 1), np.uint8)
    p = str(tmp_path / "bad_shape.safetensors")
    st.write_safetensors(p, bad)
    with pytest.raises(mxmoe.MxMoeError, match="has shape"):
        st.load_gptoss_moe_layer(p, 0)
    bad = dict(good)
    bad["block.0.mlp.mlp1_bias"] = ("F16", np.zeros((E, 2 * f), np.uint16))
    st.write_safetensors(p, bad)
    with pytest.raises(mxmoe.MxMoeError, match="dtype F16"):
        st.load_gptoss_moe_layer(p, 0)
    st.write_safetensors(p, good)
    raw = open(p, "rb").read()
    with open(p, "wb") as fh:
        fh.write(raw[:-7])
    with pytest.raises(mxmoe.MxMoeError, match="past the end"):
        st.load_gptoss_moe_layer(p, 0)
    hdr = json.dumps({"block.0.mlp.norm.scale": {"dtype": "BF16", "shape": [64]}}).encode()
    with open(p, "wb") as fh:
        fh.write(struct.pack("<Q", len(hdr)) + hdr)
    with pytest.raises(mxmoe.MxMoeError, match="lacks dtype, shape or data_offsets"):
        st.load_gptoss_moe_layer(p, 0)
    with open(p, "wb") as fh:
        fh.write(struct.pack("<Q", 1 << 40) + b"{}")
    with pytest.raises(mxmoe.MxMoeError, match="does not fit"):
        st.load_gptoss_moe_layer(p, 0)


@pytest.mark.gpu
@pytest.mark.parametrize("d,f,E,k,n,n_files,float_dtype", [
    (256, 256, 4, 2, 16, 1, "BF16"),
    (256, 256, 4, 2, 40, 3, "F32"),
    (2880, 2880, 4, 2, 96, 2, "BF16"),
])
def test_checkpoint_layer_matches_oracle(torch, tmp_path, d, f, E, k, n, n_files, float_dtype):
    """Each layer of the checkpoint, loaded with interleaved W1 rows and
    packed scales (bias 127), reproduces the oracle's interleaved layout."""
    inps, paths = make_checkpoint(tmp_path, d, f, E, k, n, n_layers=2, n_files=n_files, float_dtype=float_dtype)
    for l, inp in enumerate(inps):
        layer = st.load_gptoss_moe_layer(paths, l, experts_per_token=k)
        assert (layer.cfg.d_model, layer.cfg.ffn_hidden, layer.cfg.num_experts) == (d, f, E)
        assert layer.cfg.interleaved_glu
        x = torch.from_numpy(inp.x).to(torch.bfloat16).cuda()
        y = layer.forward(x, out_dtype=torch.float32)
        want, idx, _ = oracle_forward(inp, flags=oracle.FLAG_INTERLEAVED_GLU)
        r = layer.routing_results(n)
        np.testing.assert_array_equal(r["topk_idx"].cpu().numpy().reshape(n, k), idx)
        assert_close(y.cpu().numpy(), want, f"layer {l}")
        # the split-half reading of the same rows is a different function
        other, _, _ = oracle_forward(inp)
        with pytest.raises(AssertionError):
            assert_close(y.cpu().numpy(), other)
        layer.close()


@pytest.mark.gpu
def test_checkpoint_shard_matches_full(torch, tmp_path):
    d, f, E, k, n = 256, 256, 4, 2, 32
    _, paths = make_checkpoint(tmp_path, d, f, E, k, n, n_layers=1)
    full = st.load_gptoss_moe_layer(paths, 0, experts_per_token=k)
    part = st.load_gptoss_moe_layer(paths, 0, experts_per_token=k, experts=(1, 2))
    g = torch.Generator().manual_seed(5)
    xr = torch.randn(n, d, generator=g).to(torch.bfloat16).cuda()
    ones = torch.ones(n, dtype=torch.float32, device="cuda")
    expert = torch.tensor([1 + (i % 2) for i in range(n)], dtype=torch.int32, device="cuda")
    a = torch.empty(n, d, dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    full.forward_local(xr, ones, expert, ones, a)
    part.forward_local(xr, ones, expert, ones, b)
    torch.cuda.synchronize()
    assert_close(b.cpu().numpy(), a.cpu().numpy(), "shard vs full")
    full.close()
    part.close()
