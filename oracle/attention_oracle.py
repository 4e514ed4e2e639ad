"""CPU restatement of the reference's streaming multi-query attention step --
test infrastructure only (the checker of the CUDA path, never the product).

Follows, step by step:
  forward_streaming           src/attention/streaming_mqa.rs:239-435
  StreamingMqaCache           src/attention/streaming_mqa.rs:132-203
  evict_and_roll_mqa          src/attention/cache_ops.rs:74-117 (a real left
                              roll of the non-sink slice, as the reference does)
  compute_scores / softmax    src/attention/core.rs:7-35 (dropout off)
  apply_sinks_then_softmax    src/attention/core.rs:37-55
  AttnWindow                  src/attention/streaming.rs:14-19
  RoPE                        burn's RotaryEncoding (interleaved pairs,
                              theta_i = base^(-2i/d)), with the NTK/YaRN
                              inverse-frequency interpolation and cos/sin
                              concentration of src/rope/mod.rs:11-50.
Third-party pieces (burn 0c13f844, not vendored) restated from their published
definitions: softmax(x) = e^(x - m) / sum e^(x - m); quiet_softmax(x) =
e^(x - m) / (e^(-m) + sum e^(x - m)) with m = max x; RotaryEncoding::apply
rotates pairs (x[2i], x[2i+1]) by position * theta_i along dimension -2 of its
input.  The reference calls it on [B, T, heads, d_k] tensors
(streaming_mqa.rs:267-300), so its rotation index is start + head; rope_by_head
selects that, the default uses start + token.
Parity is "unpinned" against the reference binary (the crate cannot be built
here); the reference's own MQA tests (tests/attention_mqa_streaming_tests.rs)
are properties, ported in tests/test_attention_oracle.py.
Computed in float64.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np


@dataclass
class MqaParams:
    d_model: int
    n_heads: int
    kv_heads: int
    head_dim: int
    wq: np.ndarray  # [d_model][n_heads * head_dim] (Burn Linear layout)
    bq: np.ndarray
    wk: np.ndarray  # [d_model][kv_heads * head_dim]
    bk: np.ndarray
    wv: np.ndarray
    bv: np.ndarray
    wo: np.ndarray  # [n_heads * head_dim][d_model]
    bo: np.ndarray
    quiet_softmax: bool = False
    pre_scaled_qk: bool = False
    sinks: Optional[np.ndarray] = None  # [kv_heads][groups] module sinks
    rope: Optional[dict] = None         # theta, scaling_factor, initial_context, ntk_alpha, ntk_beta
    rope_by_head: bool = False


@dataclass
class MqaCache:
    batch: int
    cache_len: int
    kv_heads: int
    head_dim: int
    sink_tokens: int
    k: np.ndarray = field(init=False)
    v: np.ndarray = field(init=False)
    global_end_index: int = 0
    local_end_index: int = 0

    def __post_init__(self):
        shape = (self.batch, self.cache_len, self.kv_heads, self.head_dim)
        self.k = np.zeros(shape, dtype=np.float64)
        self.v = np.zeros(shape, dtype=np.float64)


def rope_theta(rope: dict, rope_dim: int):
    """Inverse frequencies and the cos/sin concentration (burn
    RotaryEncodingConfig::init + src/rope/mod.rs:11-50), in f32 like the
    reference's tables."""
    base = np.float32(rope.get("theta", 10000.0))
    i = np.arange(rope_dim // 2, dtype=np.float32)
    th = (np.float32(1.0) / np.power(base, (np.float32(2.0) * i) / np.float32(rope_dim))).astype(np.float32)
    s = rope.get("scaling_factor", 1.0)
    conc = 1.0
    if s > 1.0:
        d_model = np.float32(rope_dim * 2.0)
        d_half = d_model / np.float32(2.0)
        log_base = np.float32(np.log(base))
        two_pi = np.float32(2.0 * np.pi)
        low = d_half * np.float32(np.log(rope["initial_context"] / (rope["ntk_beta"] * two_pi))) / log_base
        high = d_half * np.float32(np.log(rope["initial_context"] / (rope["ntk_alpha"] * two_pi))) / log_base
        assert 0 < low < high < d_half - 1
        idx = np.log(th).astype(np.float32) * (-d_model / np.float32(2.0) / log_base)
        ramp = np.clip((idx - low) / (high - low), 0.0, 1.0).astype(np.float32)
        th = ((th / np.float32(s)) * (np.float32(1.0) - ramp) + th * ramp).astype(np.float32)
        conc = float(np.float32(0.1) * np.float32(np.log(s)) + np.float32(1.0))
    return th, conc


def apply_rope(x: np.ndarray, start: int, rope: dict, by_head: bool) -> np.ndarray:
    """x [B, T, H, dk] -> rotated copy (pairs 2i, 2i+1 of the even part)."""
    B, T, H, dk = x.shape
    rd = dk & ~1
    if rd == 0:
        return x
    th, conc = rope_theta(rope, rd)
    out = x.copy()
    idx = np.arange(H) if by_head else np.arange(T)
    pos = (start + idx).astype(np.float32)
    ang = (pos[:, None] * th[None, :]).astype(np.float32).astype(np.float64)  # [P, rd/2]
    cs, sn = np.cos(ang) * conc, np.sin(ang) * conc
    a = x[..., 0:rd:2]
    b = x[..., 1:rd:2]
    if by_head:
        cs_, sn_ = cs[None, None, :, :], sn[None, None, :, :]
    else:
        cs_, sn_ = cs[None, :, None, :], sn[None, :, None, :]
    out[..., 0:rd:2] = a * cs_ - b * sn_
    out[..., 1:rd:2] = b * cs_ + a * sn_
    return out


def evict_and_roll(cache: MqaCache, num_evicted: int):
    sink = cache.sink_tokens
    avail = max(cache.local_end_index - sink, 0)
    if avail == 0 or num_evicted >= avail:
        cache.local_end_index = max(cache.local_end_index - num_evicted, 0)
        return
    for buf in (cache.k, cache.v):
        sub = buf[:, sink:cache.local_end_index].copy()
        buf[:, sink:sink + avail] = np.roll(sub, -num_evicted, axis=1)
    cache.local_end_index = max(cache.local_end_index - num_evicted, 0)


def softmax(x, quiet):
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    den = e.sum(axis=-1, keepdims=True)
    if quiet:
        den = den + np.exp(-m)
    return e / den


def forward_streaming(p: MqaParams, x: np.ndarray, cache: MqaCache, start_pos: int, window: Optional[int],
                      sinks: Optional[np.ndarray] = None, attn_bias: Optional[np.ndarray] = None) -> np.ndarray:
    """x [B, T, d_model] -> [B, T, d_model]; window None = AttnWindow::Full."""
    x = np.asarray(x, dtype=np.float64)
    B, T, _ = x.shape
    nH, kvH, dk = p.n_heads, p.kv_heads, p.head_dim
    groups = nH // kvH
    q = (x @ p.wq + p.bq).reshape(B, T, nH, dk)
    k = (x @ p.wk + p.bk).reshape(B, T, kvH, dk)
    v = (x @ p.wv + p.bv).reshape(B, T, kvH, dk)
    if p.rope is not None:
        q = apply_rope(q, start_pos, p.rope, p.rope_by_head)
        k = apply_rope(k, start_pos, p.rope, p.rope_by_head)
    # cache update (streaming_mqa.rs:313-346)
    current_end = start_pos + T
    assert current_end >= cache.global_end_index
    sink, cap = cache.sink_tokens, cache.cache_len
    delta = max(current_end - cache.global_end_index, 0)
    need = cache.local_end_index + delta
    le = max(cache.local_end_index - (need - cap), 0) + delta if need > cap else need
    if window is not None and le < sink:
        # fewer cached tokens than sink_tokens: the reference's reshape panics;
        # refused here before the cache changes, as the CUDA path does
        raise ValueError("windowed attention needs at least sink_tokens cached tokens")
    if need > cap:
        evict_and_roll(cache, need - cap)
    cache.local_end_index += delta
    local_end = cache.local_end_index
    local_start = local_end - T
    assert local_start >= 0
    cache.k[:, local_start:local_end] = k
    cache.v[:, local_start:local_end] = v
    cache.global_end_index = current_end
    if window is None:
        active = local_end
    else:
        active = sink + min(window, max(local_end - sink, 0))
    start = max(local_end - active, 0)
    kw = np.repeat(cache.k[:, start:local_end], groups, axis=2)  # [B, Tk, nH, dk]
    vw = np.repeat(cache.v[:, start:local_end], groups, axis=2)
    scale_dk = 1 if p.pre_scaled_qk else dk
    scores = np.einsum("bthd,bkhd->bhtk", q, kw) / np.sqrt(scale_dk)
    if attn_bias is not None:
        scores = scores + np.asarray(attn_bias, dtype=np.float64)
    s = sinks if sinks is not None else p.sinks
    if s is not None:
        col = np.broadcast_to(np.asarray(s, dtype=np.float64).reshape(1, nH, 1, 1), (B, nH, T, 1))
        w = softmax(np.concatenate([scores, col], axis=-1), p.quiet_softmax)[..., :active]
    else:
        w = softmax(scores, p.quiet_softmax)
    ctx = np.einsum("bhtk,bkhd->bthd", w, vw).reshape(B, T, nH * dk)
    return ctx @ p.wo + p.bo


def random_params(d_model, n_heads, kv_heads, head_dim, seed=0, sinks=False, bf16=False, **kw) -> MqaParams:
    """Seeded weights ~N(0, 1/sqrt(fan_in)), biases ~N(0, 0.02); bf16-exact when asked."""
    rng = np.random.default_rng(seed)

    def r(shape, sc):
        a = rng.standard_normal(shape).astype(np.float32) * np.float32(sc)
        if bf16:
            u = a.view(np.uint32).astype(np.uint64)
            u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
            a = u.astype(np.uint32).view(np.float32)
        return a

    jq, jk = n_heads * head_dim, kv_heads * head_dim
    p = MqaParams(d_model, n_heads, kv_heads, head_dim,
                  r((d_model, jq), d_model ** -0.5), r((jq,), 0.02),
                  r((d_model, jk), d_model ** -0.5), r((jk,), 0.02),
                  r((d_model, jk), d_model ** -0.5), r((jk,), 0.02),
                  r((jq, d_model), jq ** -0.5), r((d_model,), 0.02), **kw)
    if sinks:
        p.sinks = rng.standard_normal((kv_heads, n_heads // kv_heads)).astype(np.float32)
    return p
