"""ctypes wrapper of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs as the checker.  The shipped library
never calls it.  See mxmoe_oracle.h for which parts are pinned by the
reference's own known-answer tests and which are "parity unpinned".
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(_HERE, "_build", "liboracle.so")

FLAG_INTERLEAVED_GLU = 0x1
FLAG_BIAS_PER_FTILE = 0x2
FLAG_NO_RESIDUAL = 0x4


class OrcCfg(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_uint32), ("ffn_hidden", ctypes.c_uint32), ("num_experts", ctypes.c_uint32),
                ("experts_per_token", ctypes.c_uint32), ("swiglu_alpha", ctypes.c_float),
                ("swiglu_limit", ctypes.c_float), ("rms_eps", ctypes.c_float), ("flags", ctypes.c_uint32),
                ("ue8_offset", ctypes.c_int32)]


_lib = None


def build():
    src = os.path.join(_HERE, "mxmoe_oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB)
    return _lib


def _p(a):
    return a.ctypes.data if a is not None else None


def cfg(d, f, E, k, alpha=1.702, limit=7.0, eps=1e-5, flags=0, ue8_offset=0):
    return OrcCfg(d, f, E, k, alpha, limit, eps, flags, ue8_offset)


def dequant_mxfp4_bytes(blocks, blocks_shape, scales, scales_shape):
    """src/loader/mxfp4.rs:57-79."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    rows = int(np.prod(scales_shape)) if len(scales_shape) else 1
    b = int(blocks_shape[-1])
    out = np.empty(rows * b * 2, dtype=np.float32)
    L = lib()
    L.orc_dequant_mxfp4_bytes.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                          ctypes.c_void_p]
    L.orc_dequant_mxfp4_bytes(_p(blocks), rows, b, _p(scales), _p(out))
    return out


def dequant_rows(blocks, scales, rows, cols, ue8_offset=0):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    L = lib()
    L.orc_dequant_rows.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_size_t] * 4 + [
        ctypes.c_int, ctypes.c_void_p]
    L.orc_dequant_rows(_p(blocks), _p(scales), rows, cols, (cols + 1) // 2, (cols + 31) // 32, ue8_offset, _p(out))
    return out


def route(c: OrcCfg, x, gamma, gate_w, gate_b):
    n = x.shape[0]
    x = np.ascontiguousarray(x, dtype=np.float32)
    normed = np.empty_like(x)
    rscale = np.empty(n, dtype=np.float32)
    logits = np.empty((n, c.num_experts), dtype=np.float32)
    idx = np.empty((n, c.experts_per_token), dtype=np.int32)
    w = np.empty((n, c.experts_per_token), dtype=np.float32)
    L = lib()
    L.orc_route.argtypes = [ctypes.POINTER(OrcCfg), ctypes.c_size_t] + [ctypes.c_void_p] * 9
    L.orc_route(ctypes.byref(c), n, _p(x), _p(np.ascontiguousarray(gamma, np.float32)),
                _p(np.ascontiguousarray(gate_w, np.float32)), _p(np.ascontiguousarray(gate_b, np.float32)),
                _p(normed), _p(rscale), _p(logits), _p(idx), _p(w))
    return dict(normed=normed, rscale=rscale, logits=logits, topk_idx=idx, topk_w=w)


def topk_softmax(logits, k):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    n, E = logits.shape
    idx = np.empty((n, k), dtype=np.int32)
    w = np.empty((n, k), dtype=np.float32)
    L = lib()
    L.orc_topk_softmax.argtypes = [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_void_p]
    L.orc_topk_softmax(n, E, k, _p(logits), _p(idx), _p(w))
    return idx, w


def permute(topk_idx, E):
    topk_idx = np.ascontiguousarray(topk_idx, dtype=np.int32)
    n, k = topk_idx.shape
    offsets = np.empty(E + 1, dtype=np.int32)
    perm = np.empty(n * k, dtype=np.int32)
    inv = np.empty(n * k, dtype=np.int32)
    L = lib()
    L.orc_permute.argtypes = [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32] + [ctypes.c_void_p] * 4
    L.orc_permute(n, k, E, _p(topk_idx), _p(offsets), _p(perm), _p(inv))
    return offsets, perm, inv


def swiglu(g, l, alpha=1.702, limit=7.0):
    L = lib()
    L.orc_swiglu.argtypes = [ctypes.c_float] * 4
    L.orc_swiglu.restype = ctypes.c_float
    return L.orc_swiglu(g, l, alpha, limit)


def moe_forward(c: OrcCfg, x, gamma, gate_w, gate_b, w1_blocks, w1_scales, b1, w2_blocks, w2_scales, b2,
                nthreads=0):
    n = x.shape[0]
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    idx = np.empty((n, c.experts_per_token), dtype=np.int32)
    w = np.empty((n, c.experts_per_token), dtype=np.float32)
    L = lib()
    L.orc_moe_forward.argtypes = [ctypes.POINTER(OrcCfg), ctypes.c_size_t] + [ctypes.c_void_p] * 13 + [ctypes.c_int]
    arrs = [np.ascontiguousarray(a, dtype=t) for a, t in (
        (gamma, np.float32), (gate_w, np.float32), (gate_b, np.float32), (w1_blocks, np.uint8),
        (w1_scales, np.uint8), (b1, np.float32), (w2_blocks, np.uint8), (w2_scales, np.uint8), (b2, np.float32))]
    L.orc_moe_forward(ctypes.byref(c), n, _p(x), *[_p(a) for a in arrs], _p(y), _p(idx), _p(w), nthreads)
    return y, idx, w


def moe_experts(c: OrcCfg, x, normed, topk_idx, topk_w, w1_blocks, w1_scales, b1, w2_blocks, w2_scales, b2,
                nthreads=0):
    n = x.shape[0]
    y = np.empty((n, c.d_model), dtype=np.float32)
    L = lib()
    L.orc_moe_experts.argtypes = [ctypes.POINTER(OrcCfg), ctypes.c_size_t] + [ctypes.c_void_p] * 11 + [ctypes.c_int]
    arrs = [np.ascontiguousarray(a, dtype=t) for a, t in (
        (x, np.float32), (normed, np.float32), (topk_idx, np.int32), (topk_w, np.float32), (w1_blocks, np.uint8),
        (w1_scales, np.uint8), (b1, np.float32), (w2_blocks, np.uint8), (w2_scales, np.uint8), (b2, np.float32))]
    L.orc_moe_experts(ctypes.byref(c), n, *[_p(a) for a in arrs], _p(y), nthreads)
    return y


def num_threads():
    L = lib()
    L.orc_num_threads.restype = ctypes.c_int
    return L.orc_num_threads()
