"""ctypes binding of libtqfsample.so (the C ABI in include/tqfs.h).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

LIB_PATH = _build.LIB

# status codes (include/tqfs.h)
OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED_DTYPE = 2
ERR_CUDA = 3
ERR_NCCL = 4
ERR_TIMEOUT = 5
ERR_UNSUPPORTED = 6
ERR_NO_DEVICE = 7
ERR_OUT_OF_MEMORY = 8

DTYPE_F32 = 0
DTYPE_BF16 = 1

ROW_OK = 0
ROW_ERR_WINDOW = 1
ROW_ERR_UNSUPPORTED = 2
ROW_ERR_EMPTY = 4
ROW_ERR_TIMEOUT = 8

PARAM_HAS_MIN_P = 1

# Every symbol include/tqfs.h declares; tests check the library exports them.
EXPORTS = [
    "tqfs_version", "tqfs_status_string", "tqfs_create", "tqfs_destroy", "tqfs_last_error",
    "tqfs_set_timing", "tqfs_get_timing", "tqfs_stream_plan", "tqfs_debug_stall_row", "tqfs_xoshiro_from_seed", "tqfs_xoshiro_next_u64",
    "tqfs_xoshiro_next_f32", "tqfs_sample", "tqfs_sample_host", "tqfs_top_logit_candidates",
    "tqfs_apply_penalties", "tqfs_mtp_verify", "tqfs_shard_record_words", "tqfs_shard_export",
    "tqfs_shard_merge", "tqfs_nccl_unique_id", "tqfs_nccl_comm_init", "tqfs_nccl_comm_init_timeout", "tqfs_nccl_comm_destroy",
    "tqfs_nccl_wait",
    "tqfs_sample_vocab_sharded", "tqfs_sample_static", "tqfs_decode_begin", "tqfs_decode_append", "tqfs_mtp_commit", "tqfs_rng_draw", "tqfs_lm_head_logits", "tqfs_lm_head_sample", "tqfs_sampler_new", "tqfs_sampler_is_greedy", "tqfs_sampler_select", "tqfs_sampler_get_state",
    "tqfs_sampler_free",
]


class TqfsError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"tqfs status {status}: {message}")
        self.status = status


class Params(ctypes.Structure):
    """tqfs_params (40 bytes)."""
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


class Candidate(ctypes.Structure):
    _fields_ = [("token", ctypes.c_uint32), ("logit", ctypes.c_float)]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads the in-tree library (building it first if nvcc is present)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        try:
            _build.build()
        except Exception as exc:  # no nvcc: nothing to fall back to
            raise ImportError(f"libtqfsample.so is missing and could not be built: {exc}") from exc
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64
    u64p = ctypes.POINTER(ctypes.c_uint64)
    L.tqfs_version.restype = i32
    L.tqfs_status_string.argtypes = [i32]
    L.tqfs_status_string.restype = ctypes.c_char_p
    L.tqfs_create.argtypes = [i32, ctypes.POINTER(vp)]
    L.tqfs_destroy.argtypes = [vp]
    L.tqfs_last_error.argtypes = [vp]
    L.tqfs_last_error.restype = ctypes.c_char_p
    L.tqfs_set_timing.argtypes = [vp, i32]
    L.tqfs_get_timing.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int64)]
    L.tqfs_debug_stall_row.argtypes = [vp, i32, u64]
    L.tqfs_stream_plan.argtypes = [i32, i32, i32, ctypes.POINTER(i32), ctypes.POINTER(i32)]
    L.tqfs_xoshiro_from_seed.argtypes = [u64, u64p]
    L.tqfs_xoshiro_from_seed.restype = None
    L.tqfs_xoshiro_next_u64.argtypes = [u64p]
    L.tqfs_xoshiro_next_u64.restype = u64
    L.tqfs_xoshiro_next_f32.argtypes = [u64p]
    L.tqfs_xoshiro_next_f32.restype = ctypes.c_float
    L.tqfs_sample.argtypes = [vp, vp, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_sample_host.argtypes = [vp, vp, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_top_logit_candidates.argtypes = [vp, vp, i32, i32, i32, i64, vp, vp]
    L.tqfs_apply_penalties.argtypes = [vp, vp, i32, i32, i32, i64, vp, vp, vp, vp, vp]
    L.tqfs_sample_static.argtypes = [vp, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_mtp_verify.argtypes = [vp, vp, vp, i32, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_shard_record_words.argtypes = []
    L.tqfs_shard_export.argtypes = [vp, vp, i32, i32, i32, i64, i32, i32, vp, vp, vp, vp, vp]
    L.tqfs_shard_merge.argtypes = [vp, vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_nccl_unique_id.argtypes = [vp]
    L.tqfs_nccl_comm_init.argtypes = [vp, i32, i32, vp, ctypes.POINTER(vp)]
    L.tqfs_nccl_comm_destroy.argtypes = [vp]
    L.tqfs_nccl_comm_init_timeout.argtypes = [vp, i32, i32, vp, i32, ctypes.POINTER(vp)]
    L.tqfs_nccl_wait.argtypes = [vp, vp, vp, i32]
    L.tqfs_sample_vocab_sharded.argtypes = [vp, vp, i32, vp, i32, i32, i32, i64, i32, i32, vp, vp, vp, vp, vp,
                                            vp, vp, vp]
    L.tqfs_decode_begin.argtypes = [i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_decode_append.argtypes = [i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_mtp_commit.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_rng_draw.argtypes = [i32, i32, vp, vp, vp]
    L.tqfs_lm_head_logits.argtypes = [vp, vp, i32, i32, i32, i64, i64, vp, i64, vp, vp]
    L.tqfs_lm_head_sample.argtypes = [vp, vp, vp, i32, i32, i32, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp]
    L.tqfs_sampler_new.argtypes = [vp, ctypes.POINTER(Params), i32, u64, ctypes.POINTER(vp)]
    L.tqfs_sampler_is_greedy.argtypes = [vp]
    L.tqfs_sampler_select.argtypes = [vp, vp, i64, vp, i64, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32)]
    L.tqfs_sampler_get_state.argtypes = [vp, u64p]
    L.tqfs_sampler_free.argtypes = [vp]
    for name in EXPORTS:
        if not hasattr(L, name):
            raise ImportError(f"libtqfsample.so lacks {name}")
    _lib = L
    return L


def check(status: int, handle=None) -> None:
    if status != OK:
        msg = lib().tqfs_status_string(status).decode()
        if handle is not None:
            detail = lib().tqfs_last_error(handle)
            if detail:
                msg += f" ({detail.decode()})"
        raise TqfsError(status, msg)


class Handle:
    """Owns one tqfs_handle for one CUDA device."""

    def __init__(self, device: int = 0):
        self.ptr = ctypes.c_void_p()
        check(lib().tqfs_create(device, ctypes.byref(self.ptr)))
        self.device = device

    def close(self) -> None:
        if self.ptr:
            lib().tqfs_destroy(self.ptr)
            self.ptr = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, status: int) -> None:
        check(status, self.ptr)


_handles: dict[int, Handle] = {}


def stream_plan(rows: int, vocab: int, dtype: int = DTYPE_F32) -> tuple[int, int]:
    """(units per row, chunks per unit) the stream kernel uses for a batch on
    the current device."""
    u, c = ctypes.c_int(), ctypes.c_int()
    check(lib().tqfs_stream_plan(rows, vocab, dtype, ctypes.byref(u), ctypes.byref(c)))
    return u.value, c.value


def default_handle(device: int = 0) -> Handle:
    h = _handles.get(device)
    if h is None:
        h = _handles[device] = Handle(device)
    return h
