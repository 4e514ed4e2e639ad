"""The expert-parallel step through the C ABI alone (mxmoe_ep_attach /
mxmoe_ep_forward), from a C++ host program: two and four ranks, each a layer
holding its share of the experts on its own thread and stream, meet through
a host barrier; every rank's output over several steps (one with a rank that
has no tokens) is checked against the full single-GPU layer.  The ranks share
one GPU; no kernel waits on another rank."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "burn-extended_b200", "mxmoe")
SRC = os.path.join(ROOT, "burn-extended_b200", "examples", "ep_forward.cpp")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def exe(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("cpp_ep") / "ep_forward")
    subprocess.run(["g++", "-std=c++17", "-O1", "-pthread", "-I", os.path.join(ROOT, "include"), "-I",
                    os.path.join(CUDA, "include"), SRC, "-o", out, "-L", LIBDIR, "-lmxmoe", "-L",
                    os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{LIBDIR}"], check=True)
    return out


def test_ep_program_compiles(exe):
    assert os.path.exists(exe)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_ep_forward_through_c_abi(exe, world):
    r = subprocess.run([exe, str(world), "48", "3"], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ep_forward ok" in r.stdout
