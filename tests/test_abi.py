"""The C-ABI library loads on a CPU-only host and exports every entry point
include/tqfs.h declares; host-side helpers (no device work) match the oracle."""
import ctypes
import os
import re

import numpy as np
import pytest

import turboqwenfare_b200._native as N
from turboqwenfare_b200.params import PARAMS_DTYPE

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for hdr in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not hdr.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", hdr)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^[A-Za-z_][\w\s\*]*?\b(tqfs_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(N.LIB_PATH if os.path.exists(N.LIB_PATH) else N.lib()._name)
    decl = declared_functions()
    assert len(decl) >= 15
    missing = [n for n in decl if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(N.EXPORTS) == decl, "the Python binding must bind exactly the declared set"


def test_params_layout_matches_header():
    assert ctypes.sizeof(N.Params) == 40 == PARAMS_DTYPE.itemsize
    for name, _ in N.Params._fields_:
        assert getattr(N.Params, name).offset == PARAMS_DTYPE.fields[name][1], name


def test_status_strings_and_version():
    L = N.lib()
    assert L.tqfs_version() >= 1
    assert L.tqfs_status_string(0) == b"ok"
    assert L.tqfs_status_string(6) == b"unsupported"


def test_create_without_a_device_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = ctypes.c_void_p()
    assert N.lib().tqfs_create(0, ctypes.byref(h)) == N.ERR_NO_DEVICE
    assert not h


def test_host_xoshiro_matches_oracle_and_reference_kat():
    import oracle as O
    from turboqwenfare_b200 import Xoshiro256PlusPlus
    r = Xoshiro256PlusPlus([1, 1, 1, 1])
    assert r.next_u64() == 16_777_217
    for seed in (0, 1, 42, 2**63 + 5, 2**64 - 1):
        a = Xoshiro256PlusPlus.from_seed(seed)
        b = O.xoshiro_from_seed(seed)
        assert (a.state == b).all()
        for _ in range(50):
            assert a.next_u64() == O.xoshiro_next_u64(b)
        assert a.next_f32() == O.xoshiro_next_f32(b)


def test_xoshiro_against_an_independent_restatement():
    """SplitMix64 seeding + xoshiro256++ restated in arbitrary-precision Python."""
    from turboqwenfare_b200 import Xoshiro256PlusPlus
    M = 2**64 - 1

    def seed(s):
        z, out = s, []
        for _ in range(4):
            z = (z + 0x9E3779B97F4A7C15) & M
            x = z
            x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M
            x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M
            out.append(x ^ (x >> 31))
        return out

    def rotl(x, k):
        return ((x << k) | (x >> (64 - k))) & M

    def nxt(s):
        r = (rotl((s[0] + s[3]) & M, 23) + s[0]) & M
        t = (s[1] << 17) & M
        s[2] ^= s[0]; s[3] ^= s[1]; s[1] ^= s[2]; s[0] ^= s[3]; s[2] ^= t; s[3] = rotl(s[3], 45)
        return r

    for sd in (7, 20260819):
        py = seed(sd)
        lib = Xoshiro256PlusPlus.from_seed(sd)
        assert list(map(int, lib.state)) == py
        for _ in range(20):
            assert lib.next_u64() == nxt(py)
