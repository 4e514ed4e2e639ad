"""GPT-OSS safetensors MoE loading over the C ABI.

  load_gptoss_moe_layer   load_gptoss_moe (src/loader/gpt_oss.rs:369-423) for
                          one layer, into the layer itself, packed MXFP4
                          uploaded as is, W1 rows read interleaved
  write_safetensors       a writer of the container format (u64 header
                          length, JSON header, data) for tests and exports

Parsing and loading run in libmxmoe.so (csrc/safetensors.cpp).
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
from typing import Dict, Optional, Sequence, Tuple, Union

import numpy as np

from . import MoeConfig, MoeGatedSwiGLU
from ._lib import Config, check, lib

_DTYPES = {np.dtype(np.uint8): "U8", np.dtype(np.int8): "I8", np.dtype(np.float32): "F32",
           np.dtype(np.float16): "F16"}


def load_gptoss_moe_layer(paths: Union[str, Sequence[str]], layer: int, experts_per_token: int = 4,
                          device: int = 0, *, swiglu_alpha: float = 1.702, swiglu_limit: float = 7.0,
                          rms_eps: float = 1e-5, bias_per_ftile: bool = False, residual: bool = True,
                          simt: bool = False, experts: Optional[Sequence[int]] = None,
                          stream=None) -> MoeGatedSwiGLU:
    """MoE layer `layer` of a GPT-OSS checkpoint (one file or the list of its
    shards) as a device-resident MoeGatedSwiGLU.  d_model, ffn_hidden and
    num_experts come from the tensor shapes; `experts` = (begin, count)
    loads one contiguous expert shard."""
    if isinstance(paths, (str, os.PathLike)):
        paths = [paths]
    enc = [os.fsencode(p) for p in paths]
    arr = (ctypes.c_char_p * len(enc))(*enc)
    cfg = MoeConfig(0, 0, 0, experts_per_token, swiglu_alpha=swiglu_alpha, swiglu_limit=swiglu_limit,
                    rms_eps=rms_eps, interleaved_glu=True, bias_per_ftile=bias_per_ftile, residual=residual,
                    simt=simt)
    c = Config(0, 0, 0, experts_per_token, swiglu_alpha, swiglu_limit, rms_eps, cfg.flags(), device)
    begin, count = (0, 0) if experts is None else (int(experts[0]), int(experts[1]))
    if experts is not None and count <= 0:
        raise ValueError("experts = (begin, count) needs count >= 1")
    s = stream.cuda_stream if stream is not None else None
    h = ctypes.c_void_p()
    check(lib().mxmoe_safetensors_load_layer(arr, len(enc), layer, ctypes.byref(c), begin, count, s,
                                             ctypes.byref(h)))
    return MoeGatedSwiGLU._adopt(_config_of(h, cfg), device, h)


def _config_of(h: ctypes.c_void_p, cfg: MoeConfig) -> MoeConfig:
    """cfg with the shapes the library took from the checkpoint."""
    c = Config()
    check(lib().mxmoe_get_config(h, ctypes.byref(c)))
    cfg.d_model, cfg.ffn_hidden, cfg.num_experts = c.d_model, c.ffn_hidden, c.num_experts
    return cfg


def read_header(paths: Union[str, Sequence[str]]) -> Dict[str, dict]:
    """The tensor records of one or more safetensors files (name -> record)."""
    if isinstance(paths, (str, os.PathLike)):
        paths = [paths]
    out = {}
    for p in paths:
        with open(p, "rb") as fh:
            (n,) = struct.unpack("<Q", fh.read(8))
            hdr = json.loads(fh.read(n))
        out.update({k: v for k, v in hdr.items() if k != "__metadata__"})
    return out


def write_safetensors(path: str, tensors: Dict[str, Union[np.ndarray, Tuple[str, np.ndarray]]],
                      metadata: Optional[Dict[str, str]] = None):
    """Writes `tensors` (name -> array, or name -> ("BF16", uint16 bit array))
    in the safetensors container, data in insertion order, the header padded
    with spaces to a multiple of 8 bytes."""
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = dict(metadata)
    for name, t in tensors.items():
        if isinstance(t, tuple):
            dt, a = t
        else:
            a = t
            dt = _DTYPES[np.dtype(a.dtype)]
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)
