"""The Rust side of the boundary (rust/ffi.rs, rust/build.rs, rust/status.rs) cannot be compiled
here (no cargo), so its declarations are checked against the C header and the library's exports:
every function rust/ffi.rs declares is declared in include/candle_moe.h with the same number of
parameters, the library exports it, and the two drop-in symbols keep the argument list the
reference crate's src/lib.rs passes (16 and 8 parameters)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "candle-moe_b200", "libcandle_moe_b200.so")


def _rust_fns():
    src = open(os.path.join(ROOT, "rust", "ffi.rs")).read()
    body = src[src.index('unsafe extern "C"'):]
    out = {}
    for m in re.finditer(r"pub\(crate\) fn (\w+)\s*\(([^)]*)\)", body):
        params = [p for p in m.group(2).split(",") if p.strip()]
        out[m.group(1)] = len(params)
    return out


def _header_fns():
    src = open(os.path.join(ROOT, "include", "candle_moe.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(\w+)\s*\(([^;{]*?)\)\s*;", src):
        name, args = m.group(1), m.group(2).strip()
        out[name] = 0 if args in ("", "void") else len(args.split(","))
    return out


def test_rust_declarations_match_the_header():
    rust, hdr = _rust_fns(), _header_fns()
    assert rust, "no declarations found in rust/ffi.rs"
    for name, n in rust.items():
        assert name in hdr, f"{name} is not declared in include/candle_moe.h"
        assert hdr[name] == n, f"{name}: {n} parameters in rust/ffi.rs, {hdr[name]} in the header"
    assert rust["fused_moe"] == 16 and rust["topk_softmax"] == 8


def test_rust_declarations_are_exported():
    if not os.path.exists(LIB):
        pytest.skip("library not built")
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for name in _rust_fns():
        assert name in exported, name


def test_build_rs_links_the_prebuilt_library_only():
    src = open(os.path.join(ROOT, "rust", "build.rs")).read()
    src = re.sub(r"//[^\n]*", "", src)  # code only
    assert "rustc-link-lib=dylib=candle_moe_b200" in src
    assert "bindgen_cuda" not in src and "nvcc" not in src
