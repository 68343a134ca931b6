"""Host-side mirror of TurboQwenFare's sampling API over libtqfsample.

Same names, argument meaning and error behaviour as the Rust crate:
  Sampler.new / is_greedy / select      src/sampling/mod.rs:41-74
  Xoshiro256PlusPlus.from_seed/next_u64  src/sampling/mod.rs:274-331
  top_logit_candidates                   src/runtime/decode.rs:48-64
plus the batched device entry point `sample_batch` the decode loop of a
batched server calls once per step (one launch for all rows).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _native as N
from .params import PARAMS_DTYPE, SamplingParams, pack


class Xoshiro256PlusPlus:
    """xoshiro256++ seeded by SplitMix64 (src/sampling/mod.rs:274-331)."""

    def __init__(self, state):
        self.state = np.array(state, dtype=np.uint64)

    @classmethod
    def from_seed(cls, seed: int) -> "Xoshiro256PlusPlus":
        st = np.zeros(4, np.uint64)
        N.lib().tqfs_xoshiro_from_seed(seed & (2**64 - 1), st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)))
        return cls(st)

    def next_u64(self) -> int:
        return int(N.lib().tqfs_xoshiro_next_u64(self.state.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))))

    def next_f32(self) -> float:
        return float(N.lib().tqfs_xoshiro_next_f32(self.state.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))))


@dataclass(frozen=True)
class LogitCandidate:
    token: int
    logit: float


def _params_struct(p: SamplingParams) -> N.Params:
    r = p.record()
    s = N.Params()
    for name, _ in N.Params._fields_:
        setattr(s, name, type(getattr(s, name))(r[name]))
    return s


class Sampler:
    """Drop-in `Sampler`: `Sampler.new(&params)`, `.is_greedy()`, `.select(..)`.

    The greedy arm returns the caller's argmax without touching the logits
    (src/sampling/mod.rs:68-73); the stochastic arm runs on the GPU with the
    xoshiro256++ stream held by the library for the whole generation.
    """

    def __init__(self, params: SamplingParams, device: int = 0):
        self._h = N.default_handle(device)
        self._ptr = ctypes.c_void_p()
        ps = _params_struct(params)
        has_seed = params.seed is not None
        seed = (params.seed or 0) & (2**64 - 1)
        self._h.check(N.lib().tqfs_sampler_new(self._h.ptr, ctypes.byref(ps), int(has_seed), seed,
                                              ctypes.byref(self._ptr)))

    @classmethod
    def new(cls, params: SamplingParams, device: int = 0) -> "Sampler":
        return cls(params, device)

    def is_greedy(self) -> bool:
        return bool(N.lib().tqfs_sampler_is_greedy(self._ptr))

    def select(self, logits, history: Sequence[int], greedy_token: int) -> int:
        out = ctypes.c_uint32()
        if self.is_greedy():
            self._h.check(N.lib().tqfs_sampler_select(self._ptr, None, 0, None, 0, greedy_token, ctypes.byref(out)))
            return int(out.value)
        x = np.ascontiguousarray(logits, dtype=np.float32)
        h = np.ascontiguousarray(np.asarray(history, dtype=np.int64).astype(np.uint32))
        self._h.check(N.lib().tqfs_sampler_select(
            self._ptr, x.ctypes.data_as(ctypes.c_void_p), x.size,
            h.ctypes.data_as(ctypes.c_void_p) if h.size else None, h.size, greedy_token & 0xFFFFFFFF,
            ctypes.byref(out)))
        return int(out.value)

    def rng_state(self) -> np.ndarray:
        st = np.zeros(4, np.uint64)
        self._h.check(N.lib().tqfs_sampler_get_state(self._ptr, st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))))
        return st

    def __del__(self):
        try:
            if self._ptr:
                N.lib().tqfs_sampler_free(self._ptr)
                self._ptr = ctypes.c_void_p()
        except Exception:
            pass


# ---- device batch API (torch tensors as device memory) ------------------------

def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def params_tensor(params, rows: int, device):
    import torch
    arr = params if isinstance(params, np.ndarray) else pack(params, rows)
    if arr.dtype != PARAMS_DTYPE or arr.shape[0] != rows:
        raise ValueError("params must be one tqfs_params row per logits row")
    raw = torch.from_numpy(arr.view(np.uint8).copy())
    return raw.to(device)


@dataclass
class BatchResult:
    tokens: "object"
    status: "object"
    top4: "object" = None
    probs: "object" = None


def sample_batch(logits, params, history=None, history_offsets=None, uniforms=None, rng_state=None,
                 vocab: Optional[int] = None, want_top4: bool = False, want_probs: bool = False,
                 handle: Optional[N.Handle] = None) -> BatchResult:
    """One launch of the batched sampler over device tensors.

    logits: (rows, ld) float32 or bfloat16 CUDA tensor; params: packed
    tqfs_params rows (numpy PARAMS_DTYPE array, a SamplingParams, a list of
    them, or a uint8 CUDA tensor already packed); history: int32 CUDA tensor
    of concatenated histories with int64 `history_offsets` (rows+1);
    uniforms: float32 (rows,) or None to draw from `rng_state` (uint64/int64
    (rows, 4) tensor, advanced in place).
    """
    import torch
    rows, ld = logits.shape
    dev = logits.device
    h = handle or N.default_handle(dev.index or 0)
    dtype = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}.get(logits.dtype)
    if dtype is None:
        raise N.TqfsError(N.ERR_UNSUPPORTED_DTYPE, str(logits.dtype))
    if not (isinstance(params, torch.Tensor) and params.dtype == torch.uint8):
        params = params_tensor(params, rows, dev)
    tokens = torch.empty(rows, dtype=torch.int32, device=dev)
    status = torch.empty(rows, dtype=torch.int32, device=dev)
    top4 = torch.empty((rows, 4, 2), dtype=torch.int32, device=dev) if want_top4 else None
    probs = torch.empty((rows, ld), dtype=torch.float32, device=dev) if want_probs else None
    n = ld if vocab is None else vocab
    h.check(N.lib().tqfs_sample(
        h.ptr, _ptr(logits), dtype, rows, n, ld, _ptr(history), _ptr(history_offsets), _ptr(params),
        _ptr(uniforms), _ptr(rng_state), _ptr(tokens), _ptr(top4), _ptr(probs), _ptr(status), _stream(dev)))
    return BatchResult(tokens, status, top4, probs)


def top_logit_candidates(logits, handle: Optional[N.Handle] = None):
    """`top_logit_candidates` on the GPU. A 1-D host array returns a list of
    4 LogitCandidate (as the reference); a (rows, V) CUDA tensor returns a
    (rows, 4) list of tensors (tokens int64, logits float32)."""
    import torch
    single = not isinstance(logits, torch.Tensor) or logits.dim() == 1
    x = torch.as_tensor(np.ascontiguousarray(logits, dtype=np.float32)) if not isinstance(logits, torch.Tensor) else logits
    if single:
        x = x.reshape(1, -1)
    if not x.is_cuda:
        x = x.cuda()
    x = x.contiguous()
    rows, ld = x.shape
    h = handle or N.default_handle(x.device.index or 0)
    dtype = N.DTYPE_F32 if x.dtype == torch.float32 else N.DTYPE_BF16
    out = torch.empty((rows, 4, 2), dtype=torch.int32, device=x.device)
    h.check(N.lib().tqfs_top_logit_candidates(h.ptr, x.data_ptr(), dtype, rows, ld, ld, out.data_ptr(),
                                              _stream(x.device)))
    toks = out[..., 0].to(torch.int64) & 0xFFFFFFFF
    vals = out[..., 1].view(torch.float32)
    if single:
        torch.cuda.current_stream(x.device).synchronize()
        t = toks[0].cpu().tolist()
        v = vals[0].cpu().tolist()
        return [LogitCandidate(int(t[i]), float(v[i])) for i in range(4)]
    return toks, vals


def apply_penalties(values, history, params: SamplingParams, handle: Optional[N.Handle] = None) -> np.ndarray:
    """`apply_penalties` (src/sampling/mod.rs:114-148) of one host row on the
    GPU; returns the penalised f32 values (inspection and tests)."""
    import torch
    x = torch.as_tensor(np.ascontiguousarray(values, dtype=np.float32)).reshape(1, -1).cuda()
    hist = np.ascontiguousarray(np.asarray(history, dtype=np.int64).astype(np.int32))
    h = handle or N.default_handle(x.device.index or 0)
    ht = torch.from_numpy(hist).cuda() if hist.size else torch.zeros(1, dtype=torch.int32, device=x.device)
    off = torch.tensor([0, hist.size], dtype=torch.int64, device=x.device)
    pt = params_tensor(pack([params]), 1, x.device)
    out = torch.empty_like(x)
    n = x.shape[1]
    h.check(N.lib().tqfs_apply_penalties(h.ptr, x.data_ptr(), N.DTYPE_F32, 1, n, n, ht.data_ptr(),
                                         off.data_ptr(), pt.data_ptr(), out.data_ptr(), _stream(x.device)))
    return out[0].cpu().numpy()
