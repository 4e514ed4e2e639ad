"""CPU checks of the streaming multi-query attention oracle: the properties the
reference's own tests assert (tests/attention_mqa_streaming_tests.rs:15-178),
plus the cache bookkeeping (eviction with sink tokens, the roll of
src/attention/cache_ops.rs:74-117) that the CUDA path replaces with a ring
offset, and the argument errors the C ABI reports.  No GPU needed."""
import numpy as np
import pytest

import attention_oracle as ao


def _x(rng, b, t, d):
    # burn's Distribution::Default is U[0, 1)
    return rng.random((b, t, d))


def test_window_matches_full():
    """streaming_mqa_window_matches_full: Window(t) over a t-token prompt == Full."""
    rng = np.random.default_rng(1)
    p = ao.random_params(32, 4, 2, 8, seed=1)
    x = _x(rng, 2, 12, 32)
    full = ao.forward_streaming(p, x, ao.MqaCache(2, 64, 2, 8, 0), 0, None)
    win = ao.forward_streaming(p, x, ao.MqaCache(2, 64, 2, 8, 0), 0, 12)
    assert full.shape == (2, 12, 32)
    np.testing.assert_allclose(full, win, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("rope", [None, {"theta": 10000.0}])
def test_chunks_consistent(rope):
    """streaming_mqa_with_chunks_consistent: a 16-token prompt in chunks of 4.
    There is no causal mask inside a chunk, so only the last chunk sees the
    same keys as the one-shot pass and matches it; chunk k matches a one-shot
    pass over the prompt's first 4(k + 1) tokens.  (The reference test only
    bounds the whole difference loosely, rel 0.5 / abs 0.2, for that reason.)"""
    rng = np.random.default_rng(2)
    p = ao.random_params(32, 4, 2, 8, seed=2, rope=rope)
    x = _x(rng, 1, 16, 32)
    full = ao.forward_streaming(p, x, ao.MqaCache(1, 64, 2, 8, 0), 0, 16)
    c = ao.MqaCache(1, 64, 2, 8, 0)
    outs = [ao.forward_streaming(p, x[:, s:s + 4], c, s, 16) for s in range(0, 16, 4)]
    chunked = np.concatenate(outs, axis=1)
    np.testing.assert_allclose(chunked[:, 12:], full[:, 12:], rtol=1e-10, atol=1e-10)
    for k in range(4):
        e = 4 * (k + 1)
        pre = ao.forward_streaming(p, x[:, :e], ao.MqaCache(1, 64, 2, 8, 0), 0, 16)
        np.testing.assert_allclose(outs[k], pre[:, e - 4:], rtol=1e-10, atol=1e-10)


def test_quiet_softmax_executes_and_damps():
    """streaming_mqa_quiet_softmax_executes, and the extra e^-m term makes the
    weights sum below one."""
    rng = np.random.default_rng(3)
    p = ao.random_params(16, 4, 2, 4, seed=3, quiet_softmax=True)
    out = ao.forward_streaming(p, _x(rng, 1, 8, 16), ao.MqaCache(1, 32, 2, 4, 0), 0, 8)
    assert out.shape == (1, 8, 16)
    w = ao.softmax(np.array([[0.3, -1.0, 2.0]]), quiet=True)
    assert 0.0 < w.sum() < 1.0


def test_module_sinks_used():
    """streaming_mqa_uses_module_sinks_when_set: zero sinks [kv_heads, groups]
    add one e^0 column to every softmax, equal to passing them per call."""
    rng = np.random.default_rng(4)
    x = _x(rng, 1, 8, 16)
    p = ao.random_params(16, 4, 2, 4, seed=4)
    plain = ao.forward_streaming(p, x, ao.MqaCache(1, 32, 2, 4, 0), 0, 8)
    p.sinks = np.zeros((2, 2), np.float32)
    mod = ao.forward_streaming(p, x, ao.MqaCache(1, 32, 2, 4, 0), 0, 8)
    p.sinks = None
    per_call = ao.forward_streaming(p, x, ao.MqaCache(1, 32, 2, 4, 0), 0, 8, sinks=np.zeros(4))
    assert mod.shape == (1, 8, 16)
    np.testing.assert_allclose(mod, per_call, rtol=1e-12, atol=1e-12)
    assert np.abs(mod - plain).max() > 1e-3


def _ring_slot(l, sink, cap, head):
    return l if l < sink else sink + (l - sink + head) % (cap - sink)


@pytest.mark.parametrize("sink,chunks", [(0, [3, 1, 1, 2, 1, 1, 1, 4, 1, 1]), (2, [5, 1, 1, 3, 1, 1, 1, 4, 1, 2, 1]),
                                          (3, [1] * 20)])
def test_ring_offset_equals_roll(sink, chunks):
    """The CUDA path keeps the non-sink part of the cache as a ring and turns
    the roll into a head advance (slot = sink + (l - sink + head) % (cap -
    sink)).  Replay the oracle's bookkeeping and check every cached logical
    position reads the same K through the ring as through the rolled buffer."""
    rng = np.random.default_rng(5)
    p = ao.random_params(16, 4, 2, 4, seed=5)
    cap = 10
    c = ao.MqaCache(1, cap, 2, 4, sink)
    ring = np.zeros_like(c.k)
    head, local_end, glob, pos = 0, 0, 0, 0
    for T in chunks:
        x = _x(rng, 1, T, 16)
        ao.forward_streaming(p, x, c, pos, None)
        # the same bookkeeping as mxmqa_forward_streaming
        cur = pos + T
        delta = cur - glob
        need = local_end + delta
        if need > cap:
            ev = need - cap
            avail = max(local_end - sink, 0)
            if not (avail == 0 or ev >= avail):
                head = (head + ev) % (cap - sink)
            local_end = max(local_end - ev, 0)
        local_end += delta
        glob = cur
        ls = local_end - T
        for t in range(T):
            ring[:, _ring_slot(ls + t, sink, cap, head)] = c.k[:, ls + t]
        assert (c.local_end_index, c.global_end_index) == (local_end, glob)
        for l in range(local_end):
            np.testing.assert_array_equal(ring[:, _ring_slot(l, sink, cap, head)], c.k[:, l])
        pos = cur


def test_rolling_window_equals_fresh_window():
    """With no sink tokens, a small rolling cache under Window(w) gives the
    same decode outputs as an uncapped cache under the same window."""
    rng = np.random.default_rng(6)
    p = ao.random_params(16, 4, 2, 4, seed=6, rope={"theta": 10000.0})
    small, big = ao.MqaCache(1, 6, 2, 4, 0), ao.MqaCache(1, 64, 2, 4, 0)
    pos = 0
    for T in [3, 1, 1, 1, 2, 1, 1, 1, 1, 1, 1]:
        x = _x(rng, 1, T, 16)
        a = ao.forward_streaming(p, x, small, pos, 4)
        b = ao.forward_streaming(p, x, big, pos, 4)
        np.testing.assert_allclose(a, b, rtol=1e-12, atol=1e-12)
        pos += T


def test_window_below_sink_refused_without_state_change():
    p = ao.random_params(16, 4, 2, 4, seed=7)
    c = ao.MqaCache(1, 16, 2, 4, 4)
    x = np.ones((1, 2, 16))
    with pytest.raises(ValueError):
        ao.forward_streaming(p, x, c, 0, 8)
    assert (c.global_end_index, c.local_end_index) == (0, 0)
    ao.forward_streaming(p, x, c, 0, None)  # Full is fine
    ao.forward_streaming(p, np.ones((1, 2, 16)), c, 2, 8)


def test_rope_yarn_tables():
    """NTK/YaRN interpolation as src/rope/mod.rs:34-46 writes it: the ramp is
    0 below `low` (those frequencies are divided by the factor) and 1 above
    `high` (left alone), which with its index convention divides the HIGH
    frequencies; cos/sin are scaled by 0.1 ln s + 1."""
    th0, c0 = ao.rope_theta({"theta": 150000.0}, 64)
    th, c = ao.rope_theta({"theta": 150000.0, "scaling_factor": 32.0, "initial_context": 4096.0,
                           "ntk_alpha": 1.0, "ntk_beta": 32.0}, 64)
    assert c0 == 1.0 and abs(c - (0.1 * np.log(32.0) + 1.0)) < 1e-6
    np.testing.assert_allclose(th[0], th0[0] / 32.0, rtol=1e-6)
    assert th[-1] == th0[-1]
    assert np.all(th <= th0)
