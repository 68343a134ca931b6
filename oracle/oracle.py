"""CPU ORACLE wrapper — test infrastructure only.

ctypes access to oracle/_build/liboracle.so, the C++ restatement of
TurboQwenFare's sampler (src/sampling/mod.rs:84-331,
src/runtime/decode.rs:48-64, src/runtime/mtp.rs:92-104). Only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline / reference arm import
this module, and only as the checker; the product library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

PARAMS_DTYPE = np.dtype(
    [
        ("temperature", "<f4"),
        ("top_p", "<f4"),
        ("top_k", "<u4"),
        ("min_p", "<f4"),
        ("repeat_penalty", "<f4"),
        ("frequency_penalty", "<f4"),
        ("presence_penalty", "<f4"),
        ("flags", "<u4"),
        ("repeat_last_n", "<u8"),
    ],
    align=True,
)
assert PARAMS_DTYPE.itemsize == 40


class OrcParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("top_k", ctypes.c_uint32),
        ("min_p", ctypes.c_float),
        ("repeat_penalty", ctypes.c_float),
        ("frequency_penalty", ctypes.c_float),
        ("presence_penalty", ctypes.c_float),
        ("flags", ctypes.c_uint32),
        ("repeat_last_n", ctypes.c_uint64),
    ]


class OrcDebug(ctypes.Structure):
    _fields_ = [
        ("n_after_topk", ctypes.c_int64),
        ("n_after_topp", ctypes.c_int64),
        ("n_after_minp", ctypes.c_int64),
        ("total", ctypes.c_float),
        ("total2", ctypes.c_float),
        ("target", ctypes.c_float),
        ("consumed", ctypes.c_int32),
        ("topk_tie", ctypes.c_int32),
        ("drawn_index", ctypes.c_int64),
        ("cdf_margin", ctypes.c_double),
        ("topp_margin", ctypes.c_double),
        ("kept_tokens", ctypes.POINTER(ctypes.c_uint32)),
        ("kept_probs", ctypes.POINTER(ctypes.c_float)),
        ("kept_cap", ctypes.c_int64),
    ]


_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (g++ only, no GPU)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    u64p = P(ctypes.c_uint64)
    L.orc_xoshiro_from_seed.argtypes = [ctypes.c_uint64, u64p]
    L.orc_xoshiro_next_u64.argtypes = [u64p]
    L.orc_xoshiro_next_u64.restype = ctypes.c_uint64
    L.orc_xoshiro_next_f32.argtypes = [u64p]
    L.orc_xoshiro_next_f32.restype = ctypes.c_float
    L.orc_top_logit_candidates.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    L.orc_apply_penalties.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, P(OrcParams)]
    L.orc_sample.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, P(OrcParams),
                             ctypes.c_void_p, u64p, P(OrcDebug)]
    L.orc_sample.restype = ctypes.c_uint32
    L.orc_sample_dense.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                   P(OrcParams), ctypes.c_void_p, u64p, ctypes.c_void_p, P(OrcDebug)]
    L.orc_sample_dense.restype = ctypes.c_uint32
    L.orc_sample_batch.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    L.orc_verify_pair.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    L.orc_verify_pair.restype = ctypes.c_int
    L.orc_mtp_verify.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                 ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    L.orc_mtp_verify.restype = ctypes.c_int
    L.orc_filtered_distribution.argtypes = [ctypes.c_void_p, ctypes.c_int64, P(OrcParams), ctypes.c_void_p]
    _lib = L
    return L


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def to_orc(p) -> OrcParams:
    """Accepts a numpy PARAMS_DTYPE record or any object with the fields."""
    o = OrcParams()
    for name, _ in OrcParams._fields_:
        v = p[name] if isinstance(p, np.void) else getattr(p, name)
        setattr(o, name, type(getattr(o, name))(v))
    return o


# ---- xoshiro256++ -----------------------------------------------------------
def xoshiro_from_seed(seed: int) -> np.ndarray:
    st = np.zeros(4, dtype=np.uint64)
    lib().orc_xoshiro_from_seed(ctypes.c_uint64(seed & (2**64 - 1)), st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)))
    return st


def xoshiro_next_u64(st: np.ndarray) -> int:
    return int(lib().orc_xoshiro_next_u64(st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))))


def xoshiro_next_f32(st: np.ndarray) -> float:
    return float(lib().orc_xoshiro_next_f32(st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))))


# ---- sampler ------------------------------------------------------------------
def top_logit_candidates(logits) -> list[tuple[int, float]]:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    t = np.zeros(4, np.uint32)
    v = np.zeros(4, np.float32)
    lib().orc_top_logit_candidates(_ptr(x), x.size, _ptr(t), _ptr(v))
    return [(int(t[i]), float(v[i])) for i in range(4)]


def apply_penalties(values, history, params) -> np.ndarray:
    x = np.array(values, dtype=np.float32)
    h = np.ascontiguousarray(history, dtype=np.uint32)
    op = to_orc(params)
    lib().orc_apply_penalties(_ptr(x), x.size, _ptr(h), h.size, ctypes.byref(op))
    return x


@dataclass
class SampleResult:
    token: int
    debug: OrcDebug
    probs: np.ndarray | None = None


def sample(logits, history, params, u: float | None = None, rng_state: np.ndarray | None = None,
           dense: bool = False) -> SampleResult:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    h = np.ascontiguousarray(history if history is not None else [], dtype=np.uint32)
    op = to_orc(params)
    dbg = OrcDebug()
    uu = None if u is None else np.array([u], dtype=np.float32)
    st = rng_state if rng_state is not None else np.zeros(4, np.uint64)
    stp = st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
    if dense:
        probs = np.zeros(x.size, np.float32)
        tok = lib().orc_sample_dense(_ptr(x), x.size, _ptr(h), h.size, ctypes.byref(op), _ptr(uu), stp,
                                     _ptr(probs), ctypes.byref(dbg))
        return SampleResult(int(tok), dbg, probs)
    tok = lib().orc_sample(_ptr(x), x.size, _ptr(h), h.size, ctypes.byref(op), _ptr(uu), stp, ctypes.byref(dbg))
    return SampleResult(int(tok), dbg)


def sample_batch(logits: np.ndarray, params: np.ndarray, hist: np.ndarray | None = None,
                 hist_off: np.ndarray | None = None, uniforms: np.ndarray | None = None,
                 rng_states: np.ndarray | None = None, vocab: int | None = None,
                 threads: int = 0) -> np.ndarray:
    """logits: rows x ld (float32 or uint16 bf16 bits)."""
    rows, ld = logits.shape
    n = ld if vocab is None else vocab
    dtype = 0 if logits.dtype == np.float32 else 1
    logits = np.ascontiguousarray(logits)
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    out = np.zeros(rows, np.int32)
    h = None if hist is None else np.ascontiguousarray(hist, dtype=np.int32)
    ho = None if hist_off is None else np.ascontiguousarray(hist_off, dtype=np.int64)
    uu = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float32)
    rs = rng_states
    lib().orc_sample_batch(_ptr(logits), dtype, rows, n, ld, _ptr(h), _ptr(ho), _ptr(params), _ptr(uu),
                           _ptr(rs), _ptr(out), threads)
    return out


def verify_pair(target_prediction: int, draft_token: int) -> int:
    return int(lib().orc_verify_pair(target_prediction, draft_token))


def mtp_verify(target: np.ndarray, draft: np.ndarray, drafts: np.ndarray, params: np.ndarray,
               uniforms: np.ndarray, vocab: int | None = None, threads: int = 0):
    """target: seqs x (L+1) x ld f32, draft: seqs x L x ld f32."""
    seqs, L1, ld = target.shape
    L = L1 - 1
    n = ld if vocab is None else vocab
    target = np.ascontiguousarray(target, dtype=np.float32)
    draft = np.ascontiguousarray(draft, dtype=np.float32)
    drafts = np.ascontiguousarray(drafts, dtype=np.uint32)
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    uniforms = np.ascontiguousarray(uniforms, dtype=np.float32)
    acc = np.zeros(seqs, np.int32)
    tok = np.zeros(seqs, np.int32)
    mask = np.zeros((seqs, L), np.uint8)
    rc = lib().orc_mtp_verify(_ptr(target), _ptr(draft), seqs, L, n, ld, _ptr(drafts), _ptr(params),
                              _ptr(uniforms), _ptr(acc), _ptr(tok), _ptr(mask), threads)
    if rc != 0:
        raise ValueError("oracle MTP verify rejects rows with active penalties")
    return acc, tok, mask


def filtered_distribution(logits, params) -> np.ndarray:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    q = np.zeros(x.size, np.float32)
    op = to_orc(params)
    lib().orc_filtered_distribution(_ptr(x), x.size, ctypes.byref(op), _ptr(q))
    return q
