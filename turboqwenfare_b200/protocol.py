"""Protocol request fields -> `SamplingParams`, as the reference's servers map them.

The reference normalises two wire protocols onto one `SamplingParams`
(src/runtime/request.rs:46-90) before the sampler sees a request; the device
path must receive exactly what those mappings produce:

  openai_sampling   `apply_sampling` (src/server/openai/mod.rs:276-315) with
                    the chat-completions field choice at :441-451
  ollama_sampling   `OllamaOptions::into_sampling`
                    (src/server/ollama/mod.rs:211-263)

The semantics the device path depends on: `top_k` 0 means "off" (None);
Ollama's `repeat_last_n` -1 means the whole context (usize::MAX, which the
kernels bound by the history length); Ollama's `seed` -1 means no seed;
absent OpenAI temperature is greedy (0.0). Out-of-range values are refused
with the reference's messages (`ProtocolError`), never clamped.
"""
from __future__ import annotations

import math
from typing import Any, Mapping, Optional

from .params import USIZE_MAX, SamplingParams

U32_MAX = 2**32 - 1
MAX_OPENAI_STOP = 4


class ProtocolError(ValueError):
    """A request the reference answers with 400 (the message is its own)."""


def _range(name: str, value: float, low: float, high: float) -> float:
    """`range` / `bounded` (openai/mod.rs:317-324, ollama/mod.rs:266-273)."""
    v = float(value)
    if not math.isfinite(v) or v < low or v > high:
        raise ProtocolError(f"{name} must be a finite value between {low:g} and {high:g}")
    return v


def _stop_list(stop: Any) -> list:
    if stop is None:
        return []
    if isinstance(stop, str):
        return [stop]
    if isinstance(stop, list):
        if not all(isinstance(s, str) for s in stop):
            raise ProtocolError("stop entries must be strings")
        return list(stop)
    raise ProtocolError("stop must be a string or an array of strings")


def openai_sampling(request: Mapping[str, Any]) -> SamplingParams:
    """A chat-completions request body (parsed JSON) -> SamplingParams."""
    p = SamplingParams()
    t = request.get("temperature")
    p.temperature = 0.0 if t is None else _range("temperature", t, 0.0, 2.0)
    if request.get("top_p") is not None:
        p.top_p = _range("top_p", request["top_p"], 0.0, 1.0)
    if request.get("top_k") is not None:
        k = int(request["top_k"])
        if k < 0 or k > U32_MAX:
            raise ProtocolError("top_k must be an unsigned 32-bit integer")
        p.top_k = k if k > 0 else None
    if request.get("min_p") is not None:
        p.min_p = _range("min_p", request["min_p"], 0.0, 1.0)
    p.seed = request.get("seed")
    if request.get("frequency_penalty") is not None:
        p.frequency_penalty = _range("frequency_penalty", request["frequency_penalty"], -2.0, 2.0)
    if request.get("presence_penalty") is not None:
        p.presence_penalty = _range("presence_penalty", request["presence_penalty"], -2.0, 2.0)
    maximum = request.get("max_completion_tokens")
    if maximum is None:
        maximum = request.get("max_tokens")
    if maximum is not None:
        if int(maximum) == 0:
            raise ProtocolError("max output tokens must be at least 1")
        p.max_output_tokens = int(maximum)
    stops = _stop_list(request.get("stop"))
    if len(stops) > MAX_OPENAI_STOP:
        raise ProtocolError(f"at most {MAX_OPENAI_STOP} stop sequences are supported")
    p.stop_sequences = [s for s in stops if s]
    return p


def ollama_sampling(options: Optional[Mapping[str, Any]]) -> SamplingParams:
    """An Ollama request's `options` object (parsed JSON) -> SamplingParams."""
    o = dict(options or {})
    if int(o.get("mirostat") or 0) != 0:
        raise ProtocolError("mirostat sampling is not implemented in this build")
    if o.get("tfs_z") is not None and float(o["tfs_z"]) != 1.0:
        raise ProtocolError("tail-free sampling (tfs_z) is not implemented in this build")
    if o.get("typical_p") is not None and float(o["typical_p"]) != 1.0:
        raise ProtocolError("typical_p sampling is not implemented in this build")
    p = SamplingParams()
    if o.get("temperature") is not None:
        p.temperature = _range("temperature", o["temperature"], 0.0, 2.0)
    if o.get("top_p") is not None:
        p.top_p = _range("top_p", o["top_p"], 0.0, 1.0)
    if o.get("top_k") is not None:
        k = int(o["top_k"])
        p.top_k = k if k > 0 else None
    if o.get("min_p") is not None:
        p.min_p = _range("min_p", o["min_p"], 0.0, 1.0)
    seed = o.get("seed")
    p.seed = int(seed) if seed is not None and int(seed) >= 0 else None
    if o.get("repeat_penalty") is not None:
        p.repeat_penalty = _range("repeat_penalty", o["repeat_penalty"], 0.0, 2.0)
    if o.get("repeat_last_n") is not None:
        w = int(o["repeat_last_n"])
        p.repeat_last_n = USIZE_MAX if w < 0 else w
    if o.get("frequency_penalty") is not None:
        p.frequency_penalty = _range("frequency_penalty", o["frequency_penalty"], -2.0, 2.0)
    if o.get("presence_penalty") is not None:
        p.presence_penalty = _range("presence_penalty", o["presence_penalty"], -2.0, 2.0)
    n = o.get("num_predict")
    p.max_output_tokens = min(int(n), U32_MAX) if n is not None and int(n) > 0 else None
    p.stop_sequences = [s for s in _stop_list(o.get("stop")) if s]
    return p
