"""The C++ mirror of the reference API (include/mxmoe.hpp): it compiles
against the C ABI, reports argument errors as exceptions (the reference
panics), and on a GPU reproduces the golden tiny-layer output."""
import os
import subprocess

import numpy as np
import pytest

from moe_testutil import assert_close

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "burn-extended_b200", "mxmoe")
SRC = os.path.join(ROOT, "burn-extended_b200", "examples", "moe_forward.cpp")


@pytest.fixture(scope="module")
def exe(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("cpp") / "moe_forward")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), SRC, "-o", out,
                    "-L", LIBDIR, "-lmxmoe", f"-Wl,-rpath,{LIBDIR}"], check=True)
    return out


def test_cpp_mirror_compiles_and_validates(exe):
    r = subprocess.run([exe, "--check-errors"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "errors caught: 2" in r.stdout


@pytest.mark.gpu
def test_cpp_mirror_tiny_forward_matches_golden(exe, tmp_path):
    z = np.load(os.path.join(ROOT, "tests", "golden", "tiny_seed0.npz"))
    E, f2, half_d = z["w1_blocks"].shape
    d, f, n, k = half_d * 2, f2 // 2, z["x"].shape[0], z["topk_idx"].shape[1]
    (tmp_path / "meta.txt").write_text(f"{d} {f} {E} {k} {n} 0\n")
    for name in ("x", "gate_w", "gate_b", "b1", "b2"):
        z[name].astype(np.float32).tofile(tmp_path / f"{name}.f32")
    np.ones(d, np.float32).tofile(tmp_path / "gamma.f32")
    for name in ("w1_blocks", "w1_scales", "w2_blocks", "w2_scales"):
        z[name].astype(np.uint8).tofile(tmp_path / f"{name}.u8")
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    y = np.fromfile(tmp_path / "y.f32", dtype=np.float32).reshape(n, d)
    assert_close(y, z["y_split"], "C++ mirror tiny")
