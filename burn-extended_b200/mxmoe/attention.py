"""Host-side mirror of burn-extended's streaming multi-query attention over the
C ABI (`mxmqa_*` in include/mxmoe.h).

Names and argument meaning follow the reference:
  StreamingMultiQueryAttentionConfig   src/attention/streaming_mqa.rs:12-42 (init :94-131)
  StreamingMultiQueryAttention         :44-74 (forward_streaming :239-435)
  StreamingMqaCache                    :132-203
  StreamingMqaParams                   :205-218
  AttnWindow                           src/attention/streaming.rs:14-19
Weights are given as Burn stores Linear layers ([d_in][d_out] + bias).  All
compute runs in libmxmoe.so on the GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from ._lib import BF16, F32, MqaConfig, MqaRope, check, lib

FLAG_QUIET_SOFTMAX = 0x1
FLAG_PRE_SCALED_QK = 0x2
FLAG_ROPE_BY_HEAD = 0x4


class AttnWindow:
    """AttnWindow::Full / AttnWindow::Window(n)."""

    def __init__(self, window: Optional[int] = None):
        self.window = window

    @staticmethod
    def full() -> "AttnWindow":
        return AttnWindow(None)

    @staticmethod
    def of(n: int) -> "AttnWindow":
        return AttnWindow(int(n))

    def code(self) -> int:
        return 0 if self.window is None else self.window


@dataclass
class RopeConfig:
    """burn RotaryEncodingConfig plus the NTK/YaRN scaling of src/rope/mod.rs."""
    max_seq_len: int = 131072
    theta: float = 10000.0
    scaling_factor: float = 1.0
    initial_context: float = 4096.0
    ntk_alpha: float = 1.0
    ntk_beta: float = 32.0


@dataclass
class StreamingMqaParams:
    start_pos: int
    window: AttnWindow
    sinks: Optional[object] = None      # device tensor [n_heads] f32 (this call only)
    attn_bias: Optional[object] = None  # device tensor [B, n_heads, T, active] f32


@dataclass
class StreamingMultiQueryAttentionConfig:
    d_model: int
    n_heads: int
    num_key_value_heads: int
    head_dim: int
    dropout: float = 0.0
    quiet_softmax: bool = False
    learned_sinks: bool = False
    pre_scaled_qk: bool = False
    rope_by_head: bool = False  # reproduce the reference's head-indexed RoPE call

    def init(self, device: int = 0) -> "StreamingMultiQueryAttention":
        if self.dropout != 0.0:
            raise ValueError("inference only: dropout must be 0")
        return StreamingMultiQueryAttention(self, device)


class StreamingMultiQueryAttention:
    def __init__(self, cfg: StreamingMultiQueryAttentionConfig, device: int = 0):
        flags = (FLAG_QUIET_SOFTMAX if cfg.quiet_softmax else 0) | (FLAG_PRE_SCALED_QK if cfg.pre_scaled_qk else 0) \
            | (FLAG_ROPE_BY_HEAD if cfg.rope_by_head else 0)
        c = MqaConfig(cfg.d_model, cfg.n_heads, cfg.num_key_value_heads, cfg.head_dim, flags, device)
        h = ctypes.c_void_p()
        check(lib().mxmqa_create(ctypes.byref(c), ctypes.byref(h)))
        self.cfg, self.device, self._h = cfg, device, h

    def set_weights(self, wq, bq, wk, bk, wv, bv, wo, bo, bf16: bool = False):
        """Burn Linear layout: w [d_in][d_out] (numpy f32 values; bf16=True
        uploads them as bf16, which must then be bf16-exact)."""
        def arr(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype=np.float32)
            if bf16:
                return (a.view(np.uint32) >> 16).astype(np.uint16)
            return a
        ws = [arr(a) for a in (wq, bq, wk, bk, wv, bv, wo, bo)]
        self._keep = ws
        ptrs = [None if a is None else a.ctypes.data for a in ws]
        check(lib().mxmqa_set_weights(self._h, *ptrs, BF16 if bf16 else F32, None))

    def set_sinks(self, sinks: Optional[np.ndarray]):
        """Learned sinks [kv_heads][groups] (None removes them)."""
        if sinks is None:
            check(lib().mxmqa_set_sinks(self._h, None))
            return
        s = np.ascontiguousarray(sinks, dtype=np.float32).reshape(-1)
        check(lib().mxmqa_set_sinks(self._h, s.ctypes.data))

    def set_rope(self, rope: Optional[RopeConfig]):
        if rope is None:
            check(lib().mxmqa_set_rope(self._h, None))
            return
        r = MqaRope(rope.max_seq_len, rope.theta, rope.scaling_factor, rope.initial_context, rope.ntk_alpha,
                    rope.ntk_beta)
        check(lib().mxmqa_set_rope(self._h, ctypes.byref(r)))

    def forward_streaming(self, x, cache: "StreamingMqaCache", params: StreamingMqaParams, out_dtype=None):
        """x: torch CUDA tensor [B, T, d_model] (f32 or bf16) -> [B, T, d_model]."""
        import torch
        B, T, d = x.shape
        xc = x.contiguous()
        y = torch.empty(xc.shape, dtype=out_dtype or xc.dtype, device=xc.device)

        def dt(t):
            return F32 if t.dtype == torch.float32 else BF16

        sinks = params.sinks.data_ptr() if params.sinks is not None else None
        bias = params.attn_bias.contiguous().data_ptr() if params.attn_bias is not None else None
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().mxmqa_forward_streaming(self._h, cache._h, xc.data_ptr(), dt(xc), B, T, params.start_pos,
                                            params.window.code(), sinks, bias, y.data_ptr(), dt(y), stream))
        return y

    def close(self):
        if getattr(self, "_h", None):
            lib().mxmqa_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StreamingMqaCache:
    """StreamingMqaCache::new(device, batch, cache_len, kv_heads, head_dim, sink_tokens)."""

    def __init__(self, attn: StreamingMultiQueryAttention, batch: int, cache_len: int, sink_tokens: int = 0):
        h = ctypes.c_void_p()
        check(lib().mxmqa_cache_create(attn._h, batch, cache_len, sink_tokens, ctypes.byref(h)))
        self._h = h
        self.batch, self.cache_len, self.sink_tokens = batch, cache_len, sink_tokens

    def reset(self):
        check(lib().mxmqa_cache_reset(self._h))

    def state(self):
        g, l = ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().mxmqa_cache_state(self._h, ctypes.byref(g), ctypes.byref(l)))
        return int(g.value), int(l.value)

    def __len__(self):
        return self.state()[1]

    def close(self):
        if getattr(self, "_h", None):
            lib().mxmqa_cache_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
