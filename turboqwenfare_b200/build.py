"""Builds libtqfsample.so in-tree for sm_100a with nvcc.

The library is plain CUDA C++ behind the C ABI in include/tqfs.h; it does not
link PyTorch. Output: turboqwenfare_b200/lib/libtqfsample.so (git-ignored,
shipped with the source tree to GPU hosts).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libtqfsample.so")
SOURCES = ["api.cu", "stream.cu", "general.cu", "penalties.cu", "noalloc.cu", "mtp.cu", "decode.cu", "lmhead.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def flags(verbose: bool = False) -> list[str]:
    f = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in os.listdir(CSRC)] + [os.path.join(ROOT, "include", "tqfs.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles every source to an object in parallel, then links the shared
    library (no device linking: no device code crosses translation units)."""
    if not force and not needs_build():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    objs, procs = [], []
    for s in SOURCES:
        obj = os.path.join(LIB_DIR, s.replace(".cu", ".o"))
        objs.append(obj)
        cmd = [nvcc()] + flags(verbose) + ["-c", "-o", obj, os.path.join(CSRC, s)]
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    failed = []
    for s, p in procs:
        out, err = p.communicate()
        if p.returncode != 0:
            failed.append(s)
            sys.stderr.write(out + err)
        elif verbose:
            sys.stderr.write(err)
    if failed:
        raise RuntimeError(f"nvcc failed on {', '.join(failed)}")
    tmp = LIB + ".tmp"
    res = subprocess.run([nvcc()] + ARCH + ["-shared", "-o", tmp] + objs, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed linking libtqfsample.so")
    for obj in objs:
        os.remove(obj)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
