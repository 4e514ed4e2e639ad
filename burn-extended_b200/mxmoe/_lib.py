"""ctypes binding of include/mxmoe.h (libmxmoe.so, built in-tree by build.py).

Loading fails loudly: there is no CPU fallback for any entry point.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmxmoe.so")

MXMOE_OK = 0
STATUS_NAMES = {
    0: "OK", 1: "INVALID_ARG", 2: "NOT_READY", 3: "CUDA", 4: "OOM",
    5: "UNSUPPORTED", 6: "TIMEOUT", 7: "TOO_LARGE",
}
F32, BF16 = 0, 1

FLAG_INTERLEAVED_GLU = 0x1
FLAG_BIAS_PER_FTILE = 0x2
FLAG_NO_RESIDUAL = 0x4
FLAG_DISABLED = 0x8
FLAG_SIMT = 0x10
FLAG_NO_GRAPHS = 0x20
FLAG_NO_FP4 = 0x40
FLAG_NO_GEMV = 0x80


class MxMoeError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"mxmoe error {STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_uint32), ("ffn_hidden", ctypes.c_uint32),
        ("num_experts", ctypes.c_uint32), ("experts_per_token", ctypes.c_uint32),
        ("swiglu_alpha", ctypes.c_float), ("swiglu_limit", ctypes.c_float),
        ("rms_eps", ctypes.c_float), ("flags", ctypes.c_uint32), ("device", ctypes.c_int32),
    ]


class ModelBinHeader(ctypes.Structure):
    """mxmoe_modelbin_header: model.bin header fields and derived offsets."""
    _fields_ = [
        ("context_length", ctypes.c_uint32), ("num_blocks", ctypes.c_uint32),
        ("num_experts", ctypes.c_uint32), ("num_active_experts", ctypes.c_uint32),
        ("embedding_dim", ctypes.c_uint32), ("mlp_dim", ctypes.c_uint32),
        ("swiglu_limit", ctypes.c_float), ("head_dim", ctypes.c_uint32),
        ("num_heads", ctypes.c_uint32), ("num_kv_heads", ctypes.c_uint32),
        ("attention_window", ctypes.c_uint32), ("rms_eps", ctypes.c_float),
        ("num_text_tokens", ctypes.c_uint32), ("num_special_tokens", ctypes.c_uint32),
        ("dense_offset", ctypes.c_uint64), ("moe_offset", ctypes.c_uint64),
        ("moe_layer_stride", ctypes.c_uint64), ("file_bytes", ctypes.c_uint64),
    ]


class QuantDesc(ctypes.Structure):
    _fields_ = [
        ("experts", ctypes.c_uint64), ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64),
        ("bpr", ctypes.c_uint64), ("gpr", ctypes.c_uint64), ("ue8_offset", ctypes.c_int32),
    ]


class MqaConfig(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_uint32), ("n_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("device", ctypes.c_int32)]


class MqaRope(ctypes.Structure):
    _fields_ = [("max_seq_len", ctypes.c_uint32), ("theta", ctypes.c_float), ("scaling_factor", ctypes.c_float),
                ("initial_context", ctypes.c_float), ("ntk_alpha", ctypes.c_float), ("ntk_beta", ctypes.c_float)]


_vp = ctypes.c_void_p
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_i32 = ctypes.c_int
_SIGS = {
    "mxmoe_abi_version": ([], _i32),
    "mxmoe_build_info": ([], ctypes.c_char_p),
    "mxmoe_last_error": ([ctypes.c_char_p, ctypes.c_size_t], _i32),
    "mxmoe_create": ([ctypes.POINTER(Config), ctypes.POINTER(_vp)], _i32),
    "mxmoe_destroy": ([_vp], _i32),
    "mxmoe_get_config": ([_vp, ctypes.POINTER(Config)], _i32),
    "mxmoe_fp4_operands": ([_vp, _vp, ctypes.POINTER(_u32)], _i32),
    "mxmoe_set_router": ([_vp, _vp, _vp, _vp, _i32, _vp], _i32),
    "mxmoe_upload_experts": ([_vp, ctypes.POINTER(QuantDesc), _vp, _vp, ctypes.POINTER(QuantDesc), _vp, _vp,
                              _vp, _vp, _i32, _vp], _i32),
    "mxmoe_reserve": ([_vp, _u32], _i32),
    "mxmoe_forward": ([_vp, _vp, _i32, _vp, _i32, _u32, _vp], _i32),
    "mxmoe_forward_host": ([_vp, _vp, _i32, _vp, _i32, _u32, _vp], _i32),
    "mxmoe_routing_results": ([_vp] + [ctypes.POINTER(_vp)] * 6, _i32),
    "mxmoe_dequant_mxfp4_bytes": ([_vp, _u64, _u64, _vp, _vp, _vp], _i32),
    "mxmoe_dequant_rows": ([ctypes.POINTER(QuantDesc), _vp, _vp, _vp, _vp], _i32),
    "mxmoe_topk_softmax": ([_vp, _u32, _u32, _u32, _vp, _vp, _vp], _i32),
    "mxmoe_permute": ([_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp], _i32),
    "mxmoe_permute_noalloc": ([_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp], _i32),
    "mxmoe_sync_status": ([_vp, _vp], _i32),
    "mxmoe_set_expert_shard": ([_vp, _u32, _u32], _i32),
    "mxmoe_set_profiling": ([_vp, _i32], _i32),
    "mxmoe_set_fault_injection": ([_vp, _u32], _i32),
    "mxmqa_create": ([ctypes.POINTER(MqaConfig), ctypes.POINTER(_vp)], _i32),
    "mxmqa_destroy": ([_vp], _i32),
    "mxmqa_set_weights": ([_vp] + [_vp] * 8 + [_i32, _vp], _i32),
    "mxmqa_set_sinks": ([_vp, _vp], _i32),
    "mxmqa_set_rope": ([_vp, ctypes.POINTER(MqaRope)], _i32),
    "mxmqa_cache_create": ([_vp, _u32, _u32, _u32, ctypes.POINTER(_vp)], _i32),
    "mxmqa_cache_reset": ([_vp], _i32),
    "mxmqa_cache_state": ([_vp, ctypes.POINTER(_u64), ctypes.POINTER(_u64)], _i32),
    "mxmqa_cache_destroy": ([_vp], _i32),
    "mxmqa_forward_streaming": ([_vp, _vp, _vp, _i32, _u32, _u32, _u64, _u32, _vp, _vp, _vp, _i32, _vp], _i32),
    "mxmoe_last_profile": ([_vp, ctypes.POINTER(ctypes.c_float), _i32, ctypes.POINTER(_i32)], _i32),
    "mxmoe_route": ([_vp, _vp, _i32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp], _i32),
    "mxmoe_gather_pairs": ([_vp, _i32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp], _i32),
    "mxmoe_forward_local": ([_vp, _vp, _i32, _vp, _vp, _vp, _u32, _vp, _i32, _vp], _i32),
    "mxmoe_combine": ([_vp, _i32, _u32, _u32, _u32, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _vp], _i32),
    "mxmoe_ipc_alloc": ([ctypes.c_size_t, _i32, ctypes.POINTER(_vp), _vp], _i32),
    "mxmoe_ipc_free": ([_vp, _i32], _i32),
    "mxmoe_ipc_open": ([_vp, _i32, ctypes.POINTER(_vp)], _i32),
    "mxmoe_ipc_close": ([_vp, _i32], _i32),
    "mxmoe_dispatch_pairs": ([_vp, _i32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp,
                              _u32, _vp, _vp], _i32),
    "mxmoe_forward_local_meta": ([_vp, _vp, _i32, _vp, _u32, _vp, _u32, _u32, _u32, _vp], _i32),
    "mxmoe_ep_reserve": ([_vp, _u32, _u32, _vp], _i32),
    "mxmoe_ep_dispatch": ([_vp, _vp, _i32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _vp, _vp], _i32),
    "mxmoe_ep_experts": ([_vp, _i32, _vp, _u32, _vp], _i32),
    "mxmoe_ep_attach": ([_vp, _u32, _u32, _vp, _vp, _vp, _vp, _vp], _i32),
    "mxmoe_ep_forward": ([_vp, _vp, _i32, _u32, _vp, _i32, _vp], _i32),
    "mxmoe_ep_buffers": ([_vp, _vp], _i32),
    "mxmoe_ep_plan_replicas": ([_vp, _u32, _u32, _vp], _i32),
    "mxmoe_ep_balanced_placement": ([_vp, _u32, _u32, _vp], _i32),
    "mxmoe_modelbin_info": ([ctypes.c_char_p, ctypes.POINTER(ModelBinHeader)], _i32),
    "mxmoe_safetensors_load_layer": ([ctypes.POINTER(ctypes.c_char_p), _u32, _u32, ctypes.POINTER(Config), _u32, _u32,
                                      _vp, ctypes.POINTER(_vp)], _i32),
    "mxmoe_modelbin_load_layer": ([ctypes.c_char_p, _u32, _i32, _u32, _u32, _u32, _vp, ctypes.POINTER(_vp)], _i32),
}

IPC_HANDLE_BYTES = 64
RETURN_FROM_EPILOGUE = 0x1

_lib = None


def lib():
    """Loads libmxmoe.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python burn-extended_b200/build.py` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS.keys())


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().mxmoe_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int):
    if code != MXMOE_OK:
        raise MxMoeError(code, last_error())
