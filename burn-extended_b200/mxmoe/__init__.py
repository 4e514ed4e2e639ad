"""Host-side mirror of burn-extended's `moe` / `quant` API over the B200 C ABI.

Names, argument meaning and error behaviour follow the reference crate:
  MoeConfig            src/moe/mod.rs:22-33   (init -> MoeGatedSwiGLU, :60-91)
  MoeGatedSwiGLU       src/moe/mod.rs:35-57   (set_resident :95-97, forward :99-115)
  QuantLinearMxFp4Desc src/quant/mod.rs:3-11
  MoeQuantLayerHost    src/quant/mod.rs:13-21
  dequant_mxfp4_bytes  src/loader/mxfp4.rs:57-79
The reference panics on a missing resident buffer (src/moe/mod.rs:111-113);
here every failure raises MxMoeError.  All compute runs in libmxmoe.so on the
GPU; PyTorch only provides device memory and streams.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from ._lib import (BF16, F32, FLAG_BIAS_PER_FTILE, FLAG_DISABLED, FLAG_INTERLEAVED_GLU, FLAG_NO_FP4, FLAG_NO_GEMV,
                   FLAG_NO_RESIDUAL, FLAG_SIMT, Config, MxMoeError, QuantDesc, check, exported_symbols, last_error, lib)

__all__ = [
    "MoeConfig", "MoeGatedSwiGLU", "QuantLinearMxFp4Desc", "MoeQuantLayerHost", "dequant_mxfp4_bytes",
    "dequant_rows", "topk_softmax", "permute", "MxMoeError", "lib", "exported_symbols", "F32", "BF16",
]


def _torch():
    import torch
    return torch


def _stream_ptr(stream=None, device=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return s.cuda_stream


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise MxMoeError(1, f"unsupported dtype {t.dtype} (float32 or bfloat16)")


@dataclass
class QuantLinearMxFp4Desc:
    """quant::QuantLinearMxFp4Desc (src/quant/mod.rs:3-11)."""
    experts: int
    rows: int
    cols: int
    bpr: int
    gpr: int
    ue8_offset: int = 0

    @staticmethod
    def for_shape(experts: int, rows: int, cols: int, ue8_offset: int = 0) -> "QuantLinearMxFp4Desc":
        return QuantLinearMxFp4Desc(experts, rows, cols, (cols + 1) // 2, (cols + 31) // 32, ue8_offset)

    def c(self) -> QuantDesc:
        return QuantDesc(self.experts, self.rows, self.cols, self.bpr, self.gpr, self.ue8_offset)


@dataclass
class MoeQuantLayerHost:
    """quant::MoeQuantLayerHost (src/quant/mod.rs:13-21): packed bytes on the host."""
    w1_desc: QuantLinearMxFp4Desc
    w2_desc: QuantLinearMxFp4Desc
    w1_blocks: np.ndarray
    w1_scales: np.ndarray
    w2_blocks: np.ndarray
    w2_scales: np.ndarray


@dataclass
class MoeConfig:
    """moe::MoeConfig (src/moe/mod.rs:22-33) plus the layout switches the
    reference leaves implicit (split-half vs interleaved W1 rows, per-f-tile
    W2 bias) and the RmsNorm epsilon."""
    d_model: int
    ffn_hidden: int
    num_experts: int
    experts_per_token: int
    swiglu_alpha: float = 1.702
    swiglu_limit: float = 7.0
    disabled: bool = False
    verbose: bool = False
    rms_eps: float = 1e-5
    interleaved_glu: bool = False
    bias_per_ftile: bool = False
    residual: bool = True
    simt: bool = False
    fp4_decode: bool = True  # kind::mxf4 tiles for decode batches (FLAG_NO_FP4 when False)
    gemv_decode: bool = True  # CUDA-core dequant-GEMV for tiny batches (FLAG_NO_GEMV when False)

    def flags(self) -> int:
        f = 0
        if self.interleaved_glu:
            f |= FLAG_INTERLEAVED_GLU
        if self.bias_per_ftile:
            f |= FLAG_BIAS_PER_FTILE
        if not self.residual:
            f |= FLAG_NO_RESIDUAL
        if self.disabled:
            f |= FLAG_DISABLED
        if self.simt:
            f |= FLAG_SIMT
        if not self.fp4_decode:
            f |= FLAG_NO_FP4
        if not self.gemv_decode:
            f |= FLAG_NO_GEMV
        return f

    def init(self, device: int = 0) -> "MoeGatedSwiGLU":
        """MoeConfig::init (src/moe/mod.rs:60-91)."""
        return MoeGatedSwiGLU(self, device)


class MoeGatedSwiGLU:
    """moe::MoeGatedSwiGLU (src/moe/mod.rs:35-57) backed by one mxmoe_layer."""

    def __init__(self, cfg: MoeConfig, device: int = 0):
        self.cfg = cfg
        self.device = device
        c = Config(cfg.d_model, cfg.ffn_hidden, cfg.num_experts, cfg.experts_per_token, cfg.swiglu_alpha,
                   cfg.swiglu_limit, cfg.rms_eps, cfg.flags(), device)
        h = ctypes.c_void_p()
        check(lib().mxmoe_create(ctypes.byref(c), ctypes.byref(h)))
        self._h = h
        self._keep = []

    @classmethod
    def _adopt(cls, cfg: MoeConfig, device: int, handle: ctypes.c_void_p) -> "MoeGatedSwiGLU":
        """Wraps a layer the library already created (the model.bin loader)."""
        self = cls.__new__(cls)
        self.cfg, self.device, self._h, self._keep = cfg, device, handle, []
        return self

    # -- parameters --------------------------------------------------------
    def set_router(self, norm_gamma: np.ndarray, gate_w: np.ndarray, gate_b: np.ndarray):
        """RmsNorm gain [d] and gate Linear weight [E, d] / bias [E] (f32)."""
        g = np.ascontiguousarray(norm_gamma, dtype=np.float32)
        w = np.ascontiguousarray(gate_w, dtype=np.float32)
        b = np.ascontiguousarray(gate_b, dtype=np.float32)
        E, d = self.cfg.num_experts, self.cfg.d_model
        if g.shape != (d,) or w.shape != (E, d) or b.shape != (E,):
            raise MxMoeError(1, f"router shapes {g.shape} {w.shape} {b.shape}, want ({d},) ({E},{d}) ({E},)")
        check(lib().mxmoe_set_router(self._h, g.ctypes.data, w.ctypes.data, b.ctypes.data, F32, None))

    def set_expert_shard(self, begin: int, count: int):
        check(lib().mxmoe_set_expert_shard(self._h, begin, count))

    def set_resident(self, host: MoeQuantLayerHost, mlp1_bias: np.ndarray, mlp2_bias: np.ndarray):
        """MoeQuantLayerResident::new + set_resident (src/quant/gpu.rs:31-53,
        src/moe/mod.rs:95-97); biases are the mlp1_bias [E, 2f] / mlp2_bias
        [E, d] params (:42, :45), given in f32."""
        arrs = [np.ascontiguousarray(a, dtype=np.uint8) for a in
                (host.w1_blocks, host.w1_scales, host.w2_blocks, host.w2_scales)]
        b1 = np.ascontiguousarray(mlp1_bias, dtype=np.float32)
        b2 = np.ascontiguousarray(mlp2_bias, dtype=np.float32)
        d1, d2 = host.w1_desc.c(), host.w2_desc.c()
        check(lib().mxmoe_upload_experts(self._h, ctypes.byref(d1), arrs[0].ctypes.data, arrs[1].ctypes.data,
                                         ctypes.byref(d2), arrs[2].ctypes.data, arrs[3].ctypes.data,
                                         b1.ctypes.data, b2.ctypes.data, F32, None))

    def reserve(self, max_tokens: int):
        check(lib().mxmoe_reserve(self._h, max_tokens))

    # -- forward -----------------------------------------------------------
    def forward(self, x, out_dtype=None, stream=None, out=None):
        """MoeGatedSwiGLU::forward (src/moe/mod.rs:99-115) on a CUDA tensor
        [..., d] (float32 or bfloat16); returns y of the same shape (written
        into `out` when given: repeated calls on the same x and out buffers
        replay a captured CUDA graph)."""
        torch = _torch()
        if not x.is_cuda:
            raise MxMoeError(1, "forward takes a CUDA tensor; use forward_host for host buffers")
        xc = x.contiguous()
        n = xc.numel() // self.cfg.d_model
        if out is not None:
            if out.shape != xc.shape or not out.is_contiguous():
                raise MxMoeError(1, "out must be a contiguous tensor of x's shape")
            y = out
        else:
            y = torch.empty(xc.shape, dtype=out_dtype or xc.dtype, device=xc.device)
        check(lib().mxmoe_forward(self._h, xc.data_ptr(), _dtype_code(xc), y.data_ptr(), _dtype_code(y), n,
                                  _stream_ptr(stream, self.device)))
        return y

    def forward_host(self, x_host, y_host, stream=None):
        """Host-buffer forward (pinned torch tensors or numpy arrays);
        synchronizes and checks the device status."""
        n = x_host.numel() // self.cfg.d_model if hasattr(x_host, "numel") else x_host.size // self.cfg.d_model
        xd = _dtype_code(x_host) if hasattr(x_host, "dtype") and hasattr(x_host, "data_ptr") else (
            F32 if x_host.dtype == np.float32 else BF16)
        yd = _dtype_code(y_host) if hasattr(y_host, "data_ptr") else (F32 if y_host.dtype == np.float32 else BF16)
        xp = x_host.data_ptr() if hasattr(x_host, "data_ptr") else x_host.ctypes.data
        yp = y_host.data_ptr() if hasattr(y_host, "data_ptr") else y_host.ctypes.data
        check(lib().mxmoe_forward_host(self._h, xp, xd, yp, yd, n, _stream_ptr(stream, self.device)))

    STAGES = ("router", "permute", "quantize", "w1_gemm", "w2_gemm", "combine")

    def inject_fault(self, mode: int = 1):
        """Test hook (mxmoe_set_fault_injection): the next forward withholds
        one device-side signal so that a bounded wait runs out (1 ms) and
        sync_status raises MxMoeError(MXMOE_ERR_TIMEOUT).  No GPU fault."""
        check(lib().mxmoe_set_fault_injection(self._h, mode))

    def set_profiling(self, enable: bool = True):
        check(lib().mxmoe_set_profiling(self._h, 1 if enable else 0))

    def last_profile(self) -> dict:
        """Per-stage milliseconds of the last forward (CUDA events on its stream)."""
        arr = (ctypes.c_float * 8)()
        cnt = ctypes.c_int()
        check(lib().mxmoe_last_profile(self._h, arr, 8, ctypes.byref(cnt)))
        return {name: float(arr[i]) for i, name in enumerate(self.STAGES[:cnt.value])}

    def sync_status(self, stream=None):
        check(lib().mxmoe_sync_status(self._h, _stream_ptr(stream, self.device)))

    def routing_results(self, n_tokens: int) -> dict:
        """Copies of the last forward's routing tensors (for parity checks)."""
        torch = _torch()
        ptrs = [ctypes.c_void_p() for _ in range(6)]
        check(lib().mxmoe_routing_results(self._h, *[ctypes.byref(p) for p in ptrs]))
        E, k = self.cfg.num_experts, self.cfg.experts_per_token
        P = n_tokens * k
        out = {}
        specs = [("topk_idx", P, torch.int32), ("topk_w", P, torch.float32), ("offsets", E + 1, torch.int32),
                 ("perm", P, torch.int32), ("inv", P, torch.int32), ("logits", n_tokens * E, torch.float32)]
        torch.cuda.synchronize(self.device)
        for (name, count, dt), p in zip(specs, ptrs):
            t = torch.empty(count, dtype=dt, device=f"cuda:{self.device}")
            if count:
                _copy_device(t, p.value, count * t.element_size())
            out[name] = t
        return out

    # -- expert parallel ---------------------------------------------------
    def route(self, x, rscale, topk_idx, topk_w, offsets=None, perm=None, inv=None, stream=None):
        n = x.numel() // self.cfg.d_model
        ptr = lambda t: t.data_ptr() if t is not None else None
        check(lib().mxmoe_route(self._h, x.data_ptr(), _dtype_code(x), n, rscale.data_ptr(), topk_idx.data_ptr(),
                                topk_w.data_ptr(), ptr(offsets), ptr(perm), ptr(inv), _stream_ptr(stream, self.device)))

    def forward_local(self, xr, rscale, expert, weight, out, stream=None):
        """Expert FFN of this layer's shard for dispatched pairs (out: f32 or bf16)."""
        n = expert.numel()
        if n == 0:
            return
        check(lib().mxmoe_forward_local(self._h, xr.data_ptr(), _dtype_code(xr), rscale.data_ptr(),
                                        expert.data_ptr(), weight.data_ptr(), n, out.data_ptr(), _dtype_code(out),
                                        _stream_ptr(stream, self.device)))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().mxmoe_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_cudart = None


def _copy_device(dst, src_ptr: int, nbytes: int):
    """Device-to-device copy from a library-owned buffer into a torch tensor."""
    global _cudart
    if _cudart is None:
        lib()  # loads libcudart.so.12 as a dependency
        _cudart = ctypes.CDLL("libcudart.so.12")
        _cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        _cudart.cudaMemcpy.restype = ctypes.c_int
    res = _cudart.cudaMemcpy(dst.data_ptr(), src_ptr, nbytes, 3)  # cudaMemcpyDeviceToDevice
    if res != 0:
        raise MxMoeError(3, f"cudaMemcpy failed ({res})")


def gather_pairs(x, k: int, perm, rscale, topk_idx, topk_w, out_x, out_meta, stream=None):
    """Dispatch packing: out_x[q] = x[perm[q] // k], out_meta[q] = (rscale, expert, weight) as int32 words."""
    n = rscale.numel()
    check(lib().mxmoe_gather_pairs(x.data_ptr(), _dtype_code(x), n, x.shape[-1], k, perm.data_ptr(),
                                   rscale.data_ptr(), topk_idx.data_ptr(), topk_w.data_ptr(), out_x.data_ptr(),
                                   out_meta.data_ptr(), _stream_ptr(stream)))


def combine(x, k: int, topk_idx, inv, pair_out, y, residual: bool = True, stream=None):
    n = y.numel() // y.shape[-1]
    if n == 0:
        return
    check(lib().mxmoe_combine(x.data_ptr() if x is not None else None, _dtype_code(x) if x is not None else 0, n,
                              y.shape[-1], k, topk_idx.data_ptr(), inv.data_ptr(),
                              pair_out.data_ptr() if pair_out.numel() else None, _dtype_code(pair_out),
                              1 if residual else 0, y.data_ptr(), _dtype_code(y), _stream_ptr(stream)))


def dequant_mxfp4_bytes(blocks, blocks_shape, scales, scales_shape):
    """loader::mxfp4::dequant_mxfp4_bytes (src/loader/mxfp4.rs:57-79) on the
    GPU.  blocks / scales: CUDA uint8 tensors; returns a float32 CUDA tensor
    with the blocks' shape and last dim doubled."""
    torch = _torch()
    rows = int(np.prod(scales_shape)) if len(scales_shape) else 1
    b = int(blocks_shape[-1])
    out = torch.empty(rows * b * 2, dtype=torch.float32, device=blocks.device)
    check(lib().mxmoe_dequant_mxfp4_bytes(blocks.data_ptr(), rows, b, scales.data_ptr(), out.data_ptr(),
                                          _stream_ptr()))
    return out


def dequant_rows(desc: QuantLinearMxFp4Desc, blocks, scales):
    """Dequantizes MoE weights [experts, rows, cols] on the GPU (f32)."""
    torch = _torch()
    out = torch.empty(desc.experts * desc.rows * desc.cols, dtype=torch.float32, device=blocks.device)
    d = desc.c()
    check(lib().mxmoe_dequant_rows(ctypes.byref(d), blocks.data_ptr(), scales.data_ptr(), out.data_ptr(),
                                   _stream_ptr()))
    return out.view(desc.experts, desc.rows, desc.cols)


def topk_softmax(logits, k: int):
    torch = _torch()
    n, E = logits.shape
    idx = torch.empty(n, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(n, k, dtype=torch.float32, device=logits.device)
    check(lib().mxmoe_topk_softmax(logits.contiguous().data_ptr(), n, E, k, idx.data_ptr(), w.data_ptr(),
                                   _stream_ptr()))
    return idx, w


def permute(topk_idx, num_experts: int):
    torch = _torch()
    n, k = topk_idx.shape
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=topk_idx.device)
    perm = torch.empty(n * k, dtype=torch.int32, device=topk_idx.device)
    inv = torch.empty(n * k, dtype=torch.int32, device=topk_idx.device)
    check(lib().mxmoe_permute(topk_idx.contiguous().data_ptr(), n, k, num_experts, offsets.data_ptr(),
                              perm.data_ptr(), inv.data_ptr(), _stream_ptr()))
    return offsets, perm, inv
