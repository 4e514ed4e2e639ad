"""model.bin (GPT-OSS v1.0 container) MoE loading over the C ABI.

  parse_modelbin   src/loader/modelbin.rs:153-156 (parse_headers :75-151)
  load_moe_layer   the MoE part of load_modelbin_into (:158-462): router from
                   layers.{l}.mlp.norm / mlp.gate, experts from the layer's
                   MXFP4 payload (ue8_offset 14), bf16 biases
  write_modelbin   a writer of the same container (the layout
                   src/bin/gptoss_export.rs emits) for synthetic layers; the
                   dense attention / embedding tensors it writes are filler of
                   the right sizes, since only the MoE part is read back here

All parsing and loading runs in libmxmoe.so (csrc/modelbin.cpp); this module
only forwards arguments and wraps the resulting layer handle.
"""
from __future__ import annotations

import ctypes
import os
import struct
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from . import MoeConfig, MoeGatedSwiGLU
from ._lib import ModelBinHeader, check, lib

MAGIC = b"GPT-OSS v1.0"
UE8_OFFSET = 14          # src/loader/modelbin.rs:452-453
SWIGLU_ALPHA = 1.702     # src/activation/mod.rs:6
_PAGE = 16384
_SECTION = 16


def parse_modelbin(path: str) -> dict:
    """Header fields of a model.bin plus the derived byte offsets
    (dense_offset, moe_offset, moe_layer_stride, file_bytes)."""
    h = ModelBinHeader()
    check(lib().mxmoe_modelbin_info(os.fsencode(path), ctypes.byref(h)))
    return {name: getattr(h, name) for name, _ in ModelBinHeader._fields_}


def load_moe_layer(path: str, layer: int, device: int = 0, *, interleaved_glu: bool = False,
                   bias_per_ftile: bool = False, residual: bool = True, simt: bool = False,
                   experts: Optional[Sequence[int]] = None, stream=None) -> MoeGatedSwiGLU:
    """MoE layer `layer` of the model.bin at `path`, resident on `device`.

    `experts` = (begin, count) loads only that contiguous expert shard (the
    router stays global), so an expert-parallel rank reads its own share of
    the file.  W1 rows are read as split-half [glu; lin] unless
    interleaved_glu, as MoeConfig documents."""
    hdr = parse_modelbin(path)
    cfg = MoeConfig(hdr["embedding_dim"], hdr["mlp_dim"], hdr["num_experts"], hdr["num_active_experts"],
                    swiglu_alpha=SWIGLU_ALPHA, swiglu_limit=hdr["swiglu_limit"], rms_eps=hdr["rms_eps"],
                    interleaved_glu=interleaved_glu, bias_per_ftile=bias_per_ftile, residual=residual, simt=simt)
    begin, count = (0, 0) if experts is None else (int(experts[0]), int(experts[1]))
    if experts is not None and count <= 0:
        raise ValueError("experts = (begin, count) needs count >= 1")
    s = None
    if stream is not None:
        s = stream.cuda_stream
    h = ctypes.c_void_p()
    check(lib().mxmoe_modelbin_load_layer(os.fsencode(path), layer, device, cfg.flags(), begin, count, s,
                                          ctypes.byref(h)))
    return MoeGatedSwiGLU._adopt(cfg, device, h)


# --------------------------------------------------------------------------
# writer
# --------------------------------------------------------------------------

@dataclass
class MoeLayerTensors:
    """One layer's MoE tensors as they sit in the file.  bf16 tensors are
    uint16 bit patterns; scales are true E8M0 exponents (the writer adds the
    file's +14)."""
    norm: np.ndarray          # [d] bf16 bits
    gate_w: np.ndarray        # [E, d] bf16 bits
    gate_b: np.ndarray        # [E] bf16 bits
    w1_blocks: np.ndarray     # [E, 2f, ceil(d/2)] u8
    w1_scales: np.ndarray     # [E, 2f, ceil(d/32)] u8
    b1: np.ndarray            # [E, 2f] bf16 bits
    w2_blocks: np.ndarray     # [E, d, ceil(f/2)] u8
    w2_scales: np.ndarray     # [E, d, ceil(f/32)] u8
    b2: np.ndarray            # [E, d] bf16 bits


@dataclass
class ModelBinShape:
    d: int
    f: int
    E: int
    k: int
    head_dim: int = 16
    num_heads: int = 2
    num_kv_heads: int = 1
    num_text: int = 8
    num_special: int = 2
    swiglu_limit: float = 7.0
    rms_eps: float = 1e-5
    context_length: int = 4096
    attention_window: int = 128
    regex: bytes = b"\\w+\0"
    token_blob: bytes = b"abc\0"


class _Out:
    def __init__(self, fh):
        self.fh = fh

    def tell(self) -> int:
        return self.fh.tell()

    def pad(self, align: int):
        r = self.tell() % align
        if r:
            self.fh.write(b"\0" * (align - r))

    def write(self, b):
        self.fh.write(b if isinstance(b, (bytes, bytearray)) else np.ascontiguousarray(b).tobytes())


def write_modelbin(path: str, shape: ModelBinShape, layers: List[MoeLayerTensors], seed: int = 0) -> List[int]:
    """Writes a GPT-OSS v1.0 container holding `layers`' MoE tensors; the
    dense attention, embedding and norm tensors are seeded bf16 filler.
    Returns the byte offset of each layer's expert payload."""
    rng = np.random.default_rng(seed)
    d, f, E = shape.d, shape.f, shape.E
    included = shape.num_text + shape.num_special
    qkv_rows = shape.head_dim * (shape.num_heads + 2 * shape.num_kv_heads)

    def filler(n):
        return rng.integers(0, 1 << 16, size=n, dtype=np.uint16)

    with open(path, "wb") as fh:
        o = _Out(fh)
        o.write(MAGIC + b"\0" * 4)
        o.write(bytes(range(16)))                                   # model uuid
        o.write(struct.pack("<6I", shape.context_length, len(layers), E, shape.k, d, f))
        o.write(struct.pack("<f", shape.swiglu_limit))
        o.write(struct.pack("<4I", shape.head_dim, shape.num_heads, shape.num_kv_heads, shape.attention_window))
        o.write(struct.pack("<6f", 150000.0, 32.0, 0.0, 1.0, 1.0, shape.rms_eps))
        o.write(bytes(range(16, 32)))                               # layout uuid
        o.write(bytes(range(32, 48)))                               # tokenizer uuid
        o.write(struct.pack("<4I", shape.num_special, shape.num_text, len(shape.regex), len(shape.token_blob)))
        o.write(bytes(16 * shape.num_special))
        o.write(shape.regex)
        o.write(shape.token_blob)
        o.pad(_PAGE)
        o.write(filler(included * d))                              # embedding
        for L in layers:
            o.pad(_SECTION); o.write(filler(d))                     # attention norm
            o.pad(_SECTION); o.write(filler(qkv_rows * d)); o.write(filler(qkv_rows))
            o.pad(_SECTION); o.write(filler(shape.num_heads))       # sinks
            o.pad(_SECTION); o.write(filler(d * shape.num_heads * shape.head_dim)); o.write(filler(d))
            o.pad(_SECTION); o.write(L.norm.astype(np.uint16))
            o.pad(_SECTION); o.write(L.gate_w.astype(np.uint16)); o.write(L.gate_b.astype(np.uint16))
        o.pad(_SECTION); o.write(filler(d))                         # final norm
        o.pad(_SECTION); o.write(filler(included * d))              # unembedding
        payloads = []
        for L in layers:
            o.pad(_PAGE)
            payloads.append(o.tell())
            for e in range(E):
                o.pad(_SECTION); o.write(L.w1_blocks[e].astype(np.uint8))
                o.pad(_SECTION); o.write((L.w1_scales[e].astype(np.int32) + UE8_OFFSET).astype(np.uint8))
                o.pad(_SECTION); o.write(L.b1[e].astype(np.uint16))
                o.pad(_SECTION); o.write(L.w2_blocks[e].astype(np.uint8))
                o.pad(_SECTION); o.write((L.w2_scales[e].astype(np.int32) + UE8_OFFSET).astype(np.uint8))
                o.pad(_SECTION); o.write(L.b2[e].astype(np.uint16))
    return payloads
