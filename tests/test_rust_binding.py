"""The Rust FFI crate (rust/burn-extended-cuda-sys, shipped as source: no Rust
toolchain on this image) against include/mxmoe.h: the same entry points with
the same number of parameters, and #[repr(C)] structs with the header's
fields in the header's order and types."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mxmoe.h")
SYS = os.path.join(ROOT, "rust", "burn-extended-cuda-sys", "src", "lib.rs")

C_TO_RUST = {"uint32_t": "u32", "int32_t": "i32", "uint64_t": "u64", "float": "f32"}


def header_functions():
    s = open(HEADER).read()
    out = {}
    for m in re.finditer(r"MXMOE_API\s+[\w\s\*]+?\b(mx(?:moe|mqa)_\w+)\s*\(([^;]*?)\);", s, re.S):
        args = " ".join(m.group(2).split())
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def rust_functions():
    s = open(SYS).read()
    block = s[s.index('extern "C" {'):s.index("pub mod cudart")]
    out = {}
    for m in re.finditer(r"pub fn (mx(?:moe|mqa)_\w+)\s*\(([^)]*)\)", block, re.S):
        args = [a for a in " ".join(m.group(2).split()).split(",") if a.strip()]
        out[m.group(1)] = len(args)
    return out


def header_struct(name):
    s = open(HEADER).read()
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), s, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return [(t, n) for t, n in re.findall(r"(\w+)\s+(\w+);", body)]


def rust_struct(name):
    s = open(SYS).read()
    body = re.search(r"pub struct %s \{(.*?)\}" % name, s, re.S).group(1)
    return re.findall(r"pub (\w+): (\w+),", body)


def test_same_entry_points():
    h, r = header_functions(), rust_functions()
    assert set(h) == set(r), (set(h) ^ set(r))
    for name, n in h.items():
        assert r[name] == n, (name, n, r[name])


def test_structs_match_header():
    for name in ("mxmoe_config", "mxmoe_quant_desc", "mxmoe_modelbin_header", "mxmqa_config", "mxmqa_rope"):
        hs, rs = header_struct(name), rust_struct(name)
        assert [n for _, n in hs] == [n for n, _ in rs], name
        for (ct, n), (_, rt) in zip(hs, rs):
            assert C_TO_RUST[ct] == rt, (name, n, ct, rt)
