"""C-ABI checks that need no GPU: the library loads, exports every entry
point include/mxmoe.h declares, and rejects bad arguments before touching the
device."""
import ctypes
import os
import re

import pytest

import mxmoe
from mxmoe import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mxmoe.h")


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"MXMOE_API\s+(?:const\s+)?\w+\**\s+\**(mx(?:moe|mqa)_\w+)\s*\(", txt)))


def test_header_declares_expected_entry_points():
    syms = header_symbols()
    assert len(syms) >= 20
    for s in ("mxmoe_create", "mxmoe_forward", "mxmoe_upload_experts", "mxmoe_dequant_mxfp4_bytes",
              "mxmoe_forward_local", "mxmoe_combine"):
        assert s in syms


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    for s in header_symbols():
        assert hasattr(L, s), s
    # and the Python binding covers exactly the header
    assert sorted(_lib.exported_symbols()) == header_symbols()


def test_abi_version_and_info():
    L = _lib.lib()
    assert L.mxmoe_abi_version() == 1
    assert b"sm_100a" in L.mxmoe_build_info()


def test_create_rejects_bad_config_without_device():
    L = _lib.lib()
    h = ctypes.c_void_p()
    bad = _lib.Config(0, 256, 2, 2, 1.702, 7.0, 1e-5, 0, 0)
    assert L.mxmoe_create(ctypes.byref(bad), ctypes.byref(h)) == 1
    assert "zero dimension" in _lib.last_error()
    bad = _lib.Config(250, 256, 2, 2, 1.702, 7.0, 1e-5, 0, 0)
    assert L.mxmoe_create(ctypes.byref(bad), ctypes.byref(h)) == 5
    bad = _lib.Config(256, 256, 4, 9, 1.702, 7.0, 1e-5, 0, 0)
    assert L.mxmoe_create(ctypes.byref(bad), ctypes.byref(h)) == 5
    assert L.mxmoe_create(None, ctypes.byref(h)) == 1
    assert not h.value


def test_null_and_shape_checks():
    L = _lib.lib()
    assert L.mxmoe_destroy(None) == 0
    assert L.mxmoe_forward(None, None, 0, None, 0, 0, None) == 1
    assert L.mxmoe_topk_softmax(None, 4, 2, 3, None, None, None) == 5  # k > E
    assert L.mxmoe_permute(None, 4, 2, 0, None, None, None, None) == 5  # E == 0
    d = _lib.QuantDesc(1, 4, 64, 1, 1, 0)  # bpr too small
    assert L.mxmoe_dequant_rows(ctypes.byref(d), None, None, None, None) in (1,)


def test_python_mirror_flags():
    c = mxmoe.MoeConfig(256, 256, 2, 2, interleaved_glu=True, bias_per_ftile=True, residual=False, simt=True)
    assert c.flags() == (_lib.FLAG_INTERLEAVED_GLU | _lib.FLAG_BIAS_PER_FTILE | _lib.FLAG_NO_RESIDUAL |
                         _lib.FLAG_SIMT)
    d = mxmoe.QuantLinearMxFp4Desc.for_shape(32, 5760, 2880, 14)
    assert (d.bpr, d.gpr) == (1440, 90)


def test_error_raises_in_python():
    with pytest.raises(mxmoe.MxMoeError):
        mxmoe.MoeConfig(0, 256, 2, 2).init(0)
