"""A batched decode loop over device-resident state.

The reference runs one request per loop (src/runtime/generation.rs:714-770):
push the current token into `generated`, stop at the end-of-sequence token
or after `maximum` pushes, and sample the next token with the request's
`Sampler` against `generated` as the penalty history
(`runtime.decode_step(input, &mut sampler, &generated)`). `DecodeLoop` runs
that loop for a batch of requests at once with everything on the device:
each step is one caller-supplied logits producer call (the model's forward
pass, out of scope here), one `tqfs_sample` over all rows (per-row
parameters, histories, and xoshiro256++ states seeded as `Sampler::new`
seeds them, src/sampling/mod.rs:45-53), and one `tqfs_decode_append` that
pushes each running row's token and stops rows. Nothing is copied to the
host until the caller asks for the tokens.

Differences from the reference loop, by design: rows that have stopped are
still sampled (their tokens are ignored, their generators advance), and a
row stops sampling once it has pushed `maximum` tokens (the reference runs
one more `decode_step` whose token it discards). Neither changes a row's
generated tokens.
"""
from __future__ import annotations

import time
from typing import Callable, List, Optional, Sequence, Union

import numpy as np

from . import _native as N
from .params import SamplingParams, pack
from .sampler import Xoshiro256PlusPlus, params_tensor

Producer = Callable[[int, "object"], "object"]  # (step, last_tokens_dev) -> (rows, V) logits on the device


class DecodeLoop:
    def __init__(self, params: Sequence[SamplingParams], first_tokens: Sequence[int], vocab: int,
                 max_tokens: Union[int, Sequence[int]], eos: Union[None, int, Sequence[Optional[int]]] = None,
                 cap: Optional[int] = None, device: int = 0, handle: Optional[N.Handle] = None):
        import torch
        rows = len(params)
        if len(first_tokens) != rows:
            raise ValueError("one first token per row")
        self.rows, self.vocab = rows, vocab
        self.dev = torch.device("cuda", device)
        self.h = handle or N.default_handle(device)
        mx = [int(max_tokens)] * rows if np.isscalar(max_tokens) else [int(m) for m in max_tokens]
        eo = [eos] * rows if eos is None or np.isscalar(eos) else list(eos)
        eo = [-1 if e is None else int(e) for e in eo]
        self.cap = int(cap or max(max(mx), 1))
        if self.cap < max(mx):
            raise ValueError("cap must hold every row's token budget")
        i32 = dict(dtype=torch.int32, device=self.dev)
        self.params = params_tensor(pack(list(params)), rows, self.dev)
        states = np.zeros((rows, 4), np.uint64)
        for r, p in enumerate(params):  # Sampler::new: a seeded generator, or the wall clock's
            seed = p.seed if p.seed is not None else time.time_ns()
            states[r] = Xoshiro256PlusPlus.from_seed(int(seed)).state
        self.rng = torch.from_numpy(states.view(np.int64)).to(self.dev)
        self.hist = torch.empty(rows * self.cap, **i32)
        self.hist_off = torch.empty(rows + 1, dtype=torch.int64, device=self.dev)
        self.len = torch.empty(rows, **i32)
        self.done = torch.empty(rows, dtype=torch.uint8, device=self.dev)
        self.eos = torch.tensor(eo, **i32)
        self.max_tokens = torch.tensor(mx, **i32)
        self.tokens = torch.empty(rows, **i32)
        self.status = torch.empty(rows, **i32)
        self.steps = 0
        first = torch.tensor([int(t) for t in first_tokens], **i32)
        self.h.check(N.lib().tqfs_decode_begin(rows, self.cap, first.data_ptr(), self.hist.data_ptr(),
                                               self.hist_off.data_ptr(), self.len.data_ptr(), self.eos.data_ptr(),
                                               self.max_tokens.data_ptr(), self.done.data_ptr(), self._stream()))

    def _stream(self) -> int:
        import torch
        return torch.cuda.current_stream(self.dev).cuda_stream

    def last_tokens(self):
        """Each row's most recently pushed token (device, int64)."""
        import torch
        idx = (self.len.long() - 1).clamp(min=0) + self.cap * torch.arange(self.rows, device=self.dev)
        return self.hist[idx].long()

    def step(self, logits) -> None:
        """One decode step over device logits (rows, ld) f32/bf16: sample every
        row, push the tokens of rows still running."""
        import torch
        dtype = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}[logits.dtype]
        rows, ld = logits.shape
        if rows != self.rows:
            raise ValueError("logits must have one row per request")
        L, s = N.lib(), self._stream()
        self.h.check(L.tqfs_sample(self.h.ptr, logits.data_ptr(), dtype, rows, self.vocab, ld, self.hist.data_ptr(),
                                   self.hist_off.data_ptr(), self.params.data_ptr(), None, self.rng.data_ptr(),
                                   self.tokens.data_ptr(), None, None, self.status.data_ptr(), s))
        self.h.check(L.tqfs_decode_append(rows, self.cap, self.tokens.data_ptr(), self.hist.data_ptr(),
                                          self.hist_off.data_ptr(), self.len.data_ptr(), self.eos.data_ptr(),
                                          self.max_tokens.data_ptr(), self.done.data_ptr(), s))
        self.steps += 1

    def finished(self) -> bool:
        return bool(self.done.all().item())

    def run(self, producer: Producer, max_steps: Optional[int] = None, check_every: int = 8) -> int:
        """Steps until every row has stopped (checked on the host every
        `check_every` steps) or max_steps; returns the steps taken."""
        limit = max_steps if max_steps is not None else self.cap
        taken = 0
        while taken < limit:
            if taken % check_every == 0 and self.finished():
                break
            self.step(producer(self.steps, self.last_tokens()))
            taken += 1
        return taken

    def generated(self) -> List[List[int]]:
        """Every row's `generated` tokens (copies to the host)."""
        h = self.hist.view(self.rows, self.cap).cpu().numpy()
        n = self.len.cpu().numpy()
        return [h[r, : n[r]].astype(np.int64).tolist() for r in range(self.rows)]
