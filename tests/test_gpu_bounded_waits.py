"""Failure detection on the GPU without a GPU fault: a forward withholds one
device-side signal (mxmoe_set_fault_injection, a host-side switch), the
consumer's bounded wait runs out after 1 ms, the kernel records
MXMOE_ERR_TIMEOUT and returns, and the next forward on the same layer is
correct again.  Covers the tensor-core GEMM's mbarrier waits (kind::mxf4
decode tiles and E4M3 tokens-as-A tiles) and the dequant-GEMV's W1 -> W2
wait."""
import re

import pytest

import mxmoe
from moe_testutil import assert_close, make_layer, oracle_forward, to_device_x
from mxmoe import synth

pytestmark = pytest.mark.gpu

MXMOE_ERR_TIMEOUT = 6


@pytest.mark.parametrize("name,shape", [
    ("gemv", (512, 512, 8, 4, 1)),        # batch 1: the fused dequant-GEMV
    ("mxf4 tiles", (1024, 512, 8, 4, 40)),  # decode batch: kind::mxf4 tensor-core tiles
    ("e4m3 tiles", (1024, 512, 8, 2, 600)),  # larger batch: E4M3 tokens-as-A tiles
])
def test_withheld_signal_times_out_then_recovers(name, shape):
    import torch
    d, f, E, k, n = shape
    inp = synth.make_inputs(d, f, E, k, n, True, seed=n)
    want, _, _ = oracle_forward(inp)
    layer = make_layer(inp)
    x = to_device_x(inp)
    y = layer.forward(x, out_dtype=torch.float32)  # a clean forward first
    layer.sync_status()
    layer.inject_fault()
    layer.forward(x, out_dtype=torch.float32)
    with pytest.raises(mxmoe.MxMoeError) as ei:
        layer.sync_status()
    assert ei.value.code == MXMOE_ERR_TIMEOUT, (name, ei.value)
    if name == "gemv":  # block 0 withheld its arrival: one short of the grid
        m = re.search(r"saw (\d+) of (\d+) block arrivals", str(ei.value))
        assert m and int(m.group(1)) == int(m.group(2)) - 1, str(ei.value)
    # the context is healthy and the layer computes correctly again, twice
    # (direct launch, then the graph-captured replay path)
    for i in range(3):
        y = layer.forward(x, out_dtype=torch.float32)
        layer.sync_status()
        assert_close(y.cpu().numpy(), want, f"{name} after timeout, call {i}")
    layer.close()
