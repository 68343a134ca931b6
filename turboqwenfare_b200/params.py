"""`SamplingParams` and its packed device layout.

Mirrors `SamplingParams` and its `Default` (src/runtime/request.rs:46-90).
Host-only fields (seed, stop_sequences, max_output_tokens) stay on the
host; `pack` produces the 40-byte `tqfs_params` rows the kernels read.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

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

HAS_MIN_P = 1
USIZE_MAX = 2**64 - 1


@dataclass
class SamplingParams:
    """src/runtime/request.rs:46-72. `temperature == 0.0` means greedy."""

    temperature: float = 0.0
    top_p: float = 1.0
    top_k: Optional[int] = None
    min_p: Optional[float] = None
    seed: Optional[int] = None
    repeat_penalty: float = 1.0
    repeat_last_n: int = 64
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    stop_sequences: list = field(default_factory=list)
    max_output_tokens: Optional[int] = None

    def record(self) -> np.void:
        """The row as a `tqfs_params` record (top_k None -> 0)."""
        r = np.zeros((), dtype=PARAMS_DTYPE)
        r["temperature"] = np.float32(self.temperature)
        r["top_p"] = np.float32(self.top_p)
        r["top_k"] = 0 if self.top_k is None else int(self.top_k) & 0xFFFFFFFF
        r["min_p"] = np.float32(0.0 if self.min_p is None else self.min_p)
        r["flags"] = 0 if self.min_p is None else HAS_MIN_P
        r["repeat_penalty"] = np.float32(self.repeat_penalty)
        r["repeat_last_n"] = min(int(self.repeat_last_n), USIZE_MAX)
        r["frequency_penalty"] = np.float32(self.frequency_penalty)
        r["presence_penalty"] = np.float32(self.presence_penalty)
        return r[()]


def pack(params: Sequence[SamplingParams] | SamplingParams, rows: int | None = None) -> np.ndarray:
    """Packs one SamplingParams per row (or one broadcast to `rows`)."""
    if isinstance(params, SamplingParams):
        out = np.empty(rows or 1, dtype=PARAMS_DTYPE)
        out[:] = params.record()
        return out
    out = np.empty(len(params), dtype=PARAMS_DTYPE)
    for i, p in enumerate(params):
        out[i] = p.record()
    return out
