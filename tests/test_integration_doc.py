"""INTEGRATION.md documents how the Rust crate builds and binds the library.
Its build.rs recipe must compile exactly the sources build.py compiles, with
build.py's flags, and its `extern "C"` block must declare exactly the
functions include/tqfs.h declares, each with the same number of parameters."""
import os
import re

from turboqwenfare_b200 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rust_blocks():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    return re.findall(r"```rust\n(.*?)```", text, flags=re.S)


def _header_prototypes():
    out = {}
    for hdr in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not hdr.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", hdr)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for name, args in re.findall(r"\b(tqfs_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
            args = args.strip()
            out[name] = 0 if args in ("", "void") else len(args.split(","))
    return out


def _rust_externs():
    out = {}
    for block in _rust_blocks():
        for m in re.finditer(r"pub fn (tqfs_\w+)\s*\((.*?)\)\s*(->[^;]*)?;", block, flags=re.S):
            args = m.group(2).strip().rstrip(",")
            out[m.group(1)] = 0 if not args else len(args.split(","))
    return out


def test_build_recipe_compiles_every_source_with_the_library_flags():
    build_rs = next(b for b in _rust_blocks() if "nvcc" in b)
    listed = re.search(r"let sources = \[(.*?)\];", build_rs, flags=re.S).group(1)
    assert sorted(re.findall(r'"(\w+\.cu)"', listed)) == sorted(B.SOURCES)
    for flag in B.flags():
        if flag == "-I" or flag.startswith("/"):
            continue  # include path: the crate names its own
        assert f'"{flag}"' in build_rs, flag
    assert '"-shared"' in build_rs


def test_extern_block_declares_every_header_function():
    header = _header_prototypes()
    rust = _rust_externs()
    assert len(header) >= 25
    assert sorted(rust) == sorted(header)
    for name, n in header.items():
        assert rust[name] == n, f"{name}: header has {n} parameters, INTEGRATION.md {rust[name]}"
