"""GPU parity of the streaming multi-query attention step (mxmqa_* over the C
ABI) against the float64 CPU oracle (oracle/attention_oracle.py, which follows
src/attention/streaming_mqa.rs:239-435).

Every case runs a multi-step decode through the cache: a prompt chunk, then
single tokens and small chunks past the cache capacity, so eviction with sink
tokens (the ring head advance) is exercised, under Full and Window(w), with
quiet softmax, pre-scaled QK, module and per-call sinks, an additive bias,
RoPE per token and per head (the reference's own indexing), NTK/YaRN scaling,
bf16 weights, bf16 activations, and the GPT-OSS attention shape.  Tolerance:
f32 compute against f64, |got - want| <= 2e-4 + 2e-4 |want| (f32 output);
bf16 output adds its rounding, 1e-2 + 1e-2 |want|."""
import numpy as np
import pytest

import attention_oracle as ao

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def bf16_round(a):
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def make(p: ao.MqaParams, bf16_w=False, rope_cfg=None):
    from mxmoe.attention import RopeConfig, StreamingMultiQueryAttentionConfig
    cfg = StreamingMultiQueryAttentionConfig(p.d_model, p.n_heads, p.kv_heads, p.head_dim,
                                             quiet_softmax=p.quiet_softmax, pre_scaled_qk=p.pre_scaled_qk,
                                             rope_by_head=p.rope_by_head)
    m = cfg.init(0)
    m.set_weights(p.wq, p.bq, p.wk, p.bk, p.wv, p.bv, p.wo, p.bo, bf16=bf16_w)
    if p.sinks is not None:
        m.set_sinks(p.sinks)
    if p.rope is not None:
        m.set_rope(RopeConfig(**(rope_cfg or {k: v for k, v in p.rope.items()})))
    return m


def run_steps(torch, p, chunks, batch, cache_len, sink, window, seed=0, x_bf16=False, out_bf16=False, bf16_w=False,
              bias=False, call_sinks=False):
    from mxmoe.attention import AttnWindow, StreamingMqaCache, StreamingMqaParams
    rng = np.random.default_rng(seed)
    m = make(p, bf16_w=bf16_w)
    cache = StreamingMqaCache(m, batch, cache_len, sink)
    oc = ao.MqaCache(batch, cache_len, p.kv_heads, p.head_dim, sink)
    win = AttnWindow.full() if window is None else AttnWindow.of(window)
    pos = 0
    worst = 0.0
    for step, T in enumerate(chunks):
        x = rng.standard_normal((batch, T, p.d_model)).astype(np.float32)
        if x_bf16:
            x = bf16_round(x)
        xt = torch.from_numpy(x).cuda()
        if x_bf16:
            xt = xt.to(torch.bfloat16)
        # the window length the step sees, for the bias shape
        le = min(oc.local_end_index + T, cache_len) if oc.local_end_index + T > cache_len else oc.local_end_index + T
        active = le if window is None else sink + min(window, max(le - sink, 0))
        b_np = rng.standard_normal((batch, p.n_heads, T, active)).astype(np.float32) * 0.5 if bias else None
        s_np = rng.standard_normal(p.n_heads).astype(np.float32) if call_sinks else None
        prm = StreamingMqaParams(pos, win,
                                 sinks=torch.from_numpy(s_np).cuda() if call_sinks else None,
                                 attn_bias=torch.from_numpy(b_np).cuda() if bias else None)
        y = m.forward_streaming(xt, cache, prm, out_dtype=torch.bfloat16 if out_bf16 else torch.float32)
        want = ao.forward_streaming(p, x, oc, pos, window, sinks=s_np, attn_bias=b_np)
        got = y.float().cpu().numpy()
        tol_a, tol_r = (1e-2, 1e-2) if out_bf16 else (2e-4, 2e-4)
        err = np.abs(got - want) - tol_r * np.abs(want)
        worst = max(worst, float(err.max()))
        assert err.max() <= tol_a, f"step {step} (T={T}, pos={pos}): max excess {err.max():.3e}"
        assert cache.state() == (oc.global_end_index, oc.local_end_index)
        pos += T
    return worst


DECODE = [5, 1, 1, 3, 1, 1, 1, 4, 1, 2, 1, 1, 1, 1, 6, 1]


@pytest.mark.parametrize("window", [None, 6])
@pytest.mark.parametrize("sink", [0, 2])
def test_decode_eviction(torch, window, sink):
    p = ao.random_params(64, 8, 2, 16, seed=11, rope={"theta": 10000.0})
    run_steps(torch, p, DECODE, batch=2, cache_len=12, sink=sink, window=window, seed=1)


def test_reference_shapes_and_quiet(torch):
    """The reference tests' shapes: d_model 32 / 16, 4 heads over 2 KV heads."""
    p = ao.random_params(32, 4, 2, 8, seed=12)
    run_steps(torch, p, [12], batch=2, cache_len=64, sink=0, window=None, seed=2)
    run_steps(torch, p, [4, 4, 4, 4], batch=1, cache_len=64, sink=0, window=16, seed=3)
    q = ao.random_params(16, 4, 2, 4, seed=13, quiet_softmax=True)
    run_steps(torch, q, [8, 1, 1], batch=1, cache_len=32, sink=0, window=8, seed=4)


def test_module_and_call_sinks(torch):
    p = ao.random_params(64, 8, 4, 8, seed=14, sinks=True)
    run_steps(torch, p, DECODE, batch=1, cache_len=10, sink=1, window=5, seed=5)
    p.sinks = np.zeros((4, 2), np.float32)
    run_steps(torch, p, [8, 1, 1], batch=1, cache_len=32, sink=0, window=8, seed=6)
    run_steps(torch, p, DECODE, batch=2, cache_len=12, sink=2, window=None, seed=7, call_sinks=True)


def test_quiet_pre_scaled_bias(torch):
    p = ao.random_params(64, 8, 2, 16, seed=15, quiet_softmax=True, pre_scaled_qk=True, sinks=True)
    run_steps(torch, p, DECODE, batch=2, cache_len=12, sink=2, window=6, seed=8, bias=True)


@pytest.mark.parametrize("by_head", [False, True])
def test_rope_modes_and_yarn(torch, by_head):
    yarn = {"theta": 10000.0, "scaling_factor": 32.0, "initial_context": 4096.0, "ntk_alpha": 1.0,
            "ntk_beta": 32.0}
    p = ao.random_params(64, 4, 2, 64, seed=16, rope=yarn, rope_by_head=by_head)
    run_steps(torch, p, [3, 1, 1, 1, 2, 1], batch=1, cache_len=8, sink=0, window=None, seed=9)


def test_bf16_weights_and_activations(torch):
    p = ao.random_params(64, 8, 2, 16, seed=17, bf16=True, rope={"theta": 10000.0})
    run_steps(torch, p, DECODE, batch=2, cache_len=12, sink=2, window=6, seed=10, bf16_w=True, x_bf16=True)
    run_steps(torch, p, [4, 1, 1], batch=1, cache_len=12, sink=0, window=None, seed=11, bf16_w=True,
              out_bf16=True)


def test_gpt_oss_shape(torch):
    """GPT-OSS attention: d_model 2880, 64 query heads over 8 KV heads, head_dim
    64, learned sinks, RoPE base 150000 with YaRN x32, a 128-token window."""
    yarn = {"theta": 150000.0, "scaling_factor": 32.0, "initial_context": 4096.0, "ntk_alpha": 1.0,
            "ntk_beta": 32.0}
    p = ao.random_params(2880, 64, 8, 64, seed=18, sinks=True, bf16=True, rope=yarn)
    run_steps(torch, p, [150, 1, 1, 4, 1], batch=1, cache_len=160, sink=0, window=128, seed=12, bf16_w=True)


def test_errors_leave_cache_untouched(torch):
    from mxmoe._lib import MxMoeError
    from mxmoe.attention import AttnWindow, StreamingMqaCache, StreamingMqaParams
    p = ao.random_params(32, 4, 2, 8, seed=19)
    m = make(p)
    c = StreamingMqaCache(m, 1, 16, 4)
    x = torch.ones(1, 2, 32, device="cuda")
    with pytest.raises(MxMoeError):  # Window with fewer tokens than sink_tokens
        m.forward_streaming(x, c, StreamingMqaParams(0, AttnWindow.of(8)))
    assert c.state() == (0, 0)
    m.forward_streaming(x, c, StreamingMqaParams(0, AttnWindow.full()))
    m.forward_streaming(torch.ones(1, 3, 32, device="cuda"), c, StreamingMqaParams(2, AttnWindow.of(8)))
    assert c.state() == (5, 5)
    with pytest.raises(MxMoeError):  # start_pos going backwards
        m.forward_streaming(x, c, StreamingMqaParams(0, AttnWindow.full()))
    with pytest.raises(MxMoeError):  # batch mismatch
        m.forward_streaming(torch.ones(2, 1, 32, device="cuda"), c, StreamingMqaParams(5, AttnWindow.full()))
    assert c.state() == (5, 5)
    c.reset()
    assert c.state() == (0, 0)
