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
        dtype, ld = self._layout(logits)
        rows = logits.shape[0]
        L, s = N.lib(), self._stream()
        self.h.check(L.tqfs_sample(self.h.ptr, logits.data_ptr(), dtype, rows, self.vocab, ld, self.hist.data_ptr(),
                                   self.hist_off.data_ptr(), self.params.data_ptr(), None, self.rng.data_ptr(),
                                   self.tokens.data_ptr(), None, None, self.status.data_ptr(), s))
        self.h.check(L.tqfs_decode_append(rows, self.cap, self.tokens.data_ptr(), self.hist.data_ptr(),
                                          self.hist_off.data_ptr(), self.len.data_ptr(), self.eos.data_ptr(),
                                          self.max_tokens.data_ptr(), self.done.data_ptr(), s))
        self.steps += 1

    def _layout(self, logits):
        """(dtype code, row stride) of a (rows, >= vocab) logits view."""
        import torch
        dtype = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}.get(logits.dtype)
        if dtype is None:
            raise N.TqfsError(N.ERR_UNSUPPORTED_DTYPE, str(logits.dtype))
        if logits.dim() != 2 or logits.shape[0] != self.rows or logits.shape[1] < self.vocab or logits.stride(1) != 1:
            raise ValueError("logits must be (rows, >= vocab) with unit column stride, one row per request")
        return dtype, logits.stride(0)

    def finished(self) -> bool:
        return bool(self.done.all().item())

    def failed(self) -> List[int]:
        """Rows the sampler failed (stopped with done = 2)."""
        return [int(r) for r in (self.done == 2).nonzero().flatten().tolist()]

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


Model = Callable[["object", "object"], "object"]  # (tokens (rows, n) int64, positions (rows, n) int64) -> (rows, n, ld)


def _penalties_neutral(p: SamplingParams) -> bool:
    return p.repeat_penalty == 1.0 and p.frequency_penalty == 0.0 and p.presence_penalty == 0.0


class MtpDecodeLoop(DecodeLoop):
    """Speculative decoding with MTP drafts over the device-resident loop of
    DecodeLoop, driven by an MtpController (src/runtime/mtp.rs:112-168).

    A speculative step runs the draft head `draft_len` times (each call
    scores one position and its token is sampled with the row's own
    parameters and generator), the target model once over the boundary
    token and the drafts, `tqfs_mtp_verify` on the two sets of rows, and
    `tqfs_mtp_commit`, which pushes the accepted drafts and the verify token
    under the decode loop's stop rules. A plain step is DecodeLoop's: the
    target over the boundary token, `tqfs_sample`, `tqfs_decode_append`.

    Model contract. `target(tokens, positions)` and `draft(tokens, positions)`
    take (rows, n) int64 tokens and their absolute positions (token i of
    row r's `generated` has position i) and return (rows, n, >= vocab)
    logits, f32 or bf16. Entry j scores the token after position
    positions[:, j]. The target appends its n inputs to its KV cache; after
    every step `rollback(kv_len)` (optional) gets the entries each row keeps,
    len - 1 (every generated token but the newest, which is the next step's
    input): the rejected drafts' entries are the ones a cache discards.

    Randomness. Drafts draw from the row's generator as tqfs_sample does (one
    draw per sampled row); the verify's draft_len + 1 uniforms then come from
    the same generator (tqfs_rng_draw). Rows must have neutral penalties:
    verification has none (tqfs_mtp_verify reports them unsupported).

    Policy. The reference does not say how evidence is gathered while MTP is
    off; here the loop speculates while the controller's window is filling
    and while it is enabled, runs plain steps while it is disabled, and
    every `probe_every`-th step runs the other mode, which keeps both step
    times measured (CUDA events; medians, the first step of each mode
    dropped as warm-up) and the window fed. The controller and the
    statistics are fed every `check_every` steps, from device logs: each
    running row's verification records `draft_len` drafts, its accepted
    count, `accepted + 1` emitted tokens and one target pass (for
    draft_len = 1 this is MtpStatistics::record of one verify_pair outcome),
    and feeds the controller `accepted + 1 - t_speculative / t_plain`, which
    is record_and_decide(accepted + 1) when the two step times are equal.
    `modes` lists every step's mode (True = speculative).
    """

    def __init__(self, params: Sequence[SamplingParams], first_tokens: Sequence[int], vocab: int,
                 max_tokens: Union[int, Sequence[int]], draft_len: int = 1,
                 eos: Union[None, int, Sequence[Optional[int]]] = None, cap: Optional[int] = None,
                 controller=None, window: int = 16, probe_every: int = 16, device: int = 0,
                 handle: Optional[N.Handle] = None):
        import torch
        from .mtp import MtpController, MtpStatistics
        if draft_len < 1:
            raise ValueError("draft_len must be at least 1")
        bad = [i for i, p in enumerate(params) if not _penalties_neutral(p)]
        if bad:
            raise ValueError(f"rows {bad[:8]} carry an active penalty; MTP verification has none")
        super().__init__(params, first_tokens, vocab, max_tokens, eos, cap, device, handle)
        self.L = int(draft_len)
        self.controller = controller if controller is not None else MtpController(window)
        self.stats = MtpStatistics()
        self.probe_every = int(probe_every)
        self.modes: List[bool] = []
        i32 = dict(dtype=torch.int32, device=self.dev)
        self.kv_len = torch.zeros(self.rows, **i32)
        self.dtok = torch.empty((self.L, self.rows), **i32)
        self.drafts = torch.empty((self.rows, self.L), **i32)
        self.uniforms = torch.empty((self.rows, self.L + 1), dtype=torch.float32, device=self.dev)
        self.accepted = torch.empty(self.rows, **i32)
        self.vtoken = torch.empty(self.rows, **i32)
        self.mask = torch.empty((self.rows, self.L), dtype=torch.uint8, device=self.dev)
        self.emitted = torch.empty(self.rows, **i32)
        self._draft_buf = None
        self._pending = []   # (accepted copy, running-before mask) per speculative step since the last check
        self._events = []    # (mode, start, end) per step since the last check
        self._t = {True: [], False: []}

    # -- one step of each kind --------------------------------------------
    def _positions(self, n: int):
        import torch
        return self.kv_len.long()[:, None] + torch.arange(n, device=self.dev)[None, :]

    def _after_step(self, rollback) -> None:
        import torch
        torch.sub(self.len, 1, out=self.kv_len)
        if rollback is not None:
            rollback(self.kv_len)

    def step_plain(self, target: Model, rollback: Optional[Callable] = None) -> None:
        x = target(self.last_tokens()[:, None], self._positions(1))
        self.step(x[:, 0])
        self._after_step(rollback)

    def step_speculative(self, draft: Model, target: Model, rollback: Optional[Callable] = None) -> None:
        import torch
        L, s = N.lib(), self._stream()
        last = self.last_tokens()
        running = self.done == 0
        tok = last
        for i in range(self.L):
            x = draft(tok[:, None], self._positions(i + 1)[:, i:i + 1])[:, 0]
            dtype, ld = self._layout(x)
            if self._draft_buf is None or self._draft_buf.dtype != x.dtype or self._draft_buf.shape[2] != x.shape[1]:
                self._draft_buf = torch.empty((self.rows, self.L, x.shape[1]), dtype=x.dtype, device=self.dev)
            self.h.check(L.tqfs_sample(self.h.ptr, x.data_ptr(), dtype, self.rows, self.vocab, ld,
                                       self.hist.data_ptr(), self.hist_off.data_ptr(), self.params.data_ptr(),
                                       None, self.rng.data_ptr(), self.dtok[i].data_ptr(), None, None,
                                       self.status.data_ptr(), s))
            self._draft_buf[:, i].copy_(x)
            tok = self.dtok[i].long()
        self.drafts.copy_(self.dtok.t())
        inputs = torch.cat([last[:, None], self.drafts.long()], 1)
        t = target(inputs, self._positions(self.L + 1))
        if t.dim() != 3 or t.shape[:2] != (self.rows, self.L + 1) or t.dtype != self._draft_buf.dtype:
            raise ValueError("target must return (rows, draft_len + 1, ld) logits of the draft's dtype")
        t = t.contiguous()
        db = self._draft_buf
        if t.shape[2] != db.shape[2]:
            raise ValueError("target and draft rows must have the same length")
        dtype = N.DTYPE_F32 if t.dtype == torch.float32 else N.DTYPE_BF16
        self.h.check(L.tqfs_rng_draw(self.rows, self.L + 1, self.rng.data_ptr(), self.uniforms.data_ptr(), s))
        self.h.check(L.tqfs_mtp_verify(self.h.ptr, t.data_ptr(), db.data_ptr(), dtype, self.rows, self.L,
                                       self.vocab, t.shape[2], self.drafts.data_ptr(), self.params.data_ptr(),
                                       self.uniforms.data_ptr(), self.accepted.data_ptr(), self.vtoken.data_ptr(),
                                       self.mask.data_ptr(), self.status.data_ptr(), s))
        self.h.check(L.tqfs_mtp_commit(self.rows, self.L, self.cap, self.accepted.data_ptr(),
                                       self.vtoken.data_ptr(), self.drafts.data_ptr(), self.hist.data_ptr(),
                                       self.hist_off.data_ptr(), self.len.data_ptr(), self.eos.data_ptr(),
                                       self.max_tokens.data_ptr(), self.done.data_ptr(), self.emitted.data_ptr(),
                                       s))
        self.steps += 1
        self._pending.append((self.accepted.clone(), running))
        self._after_step(rollback)

    # -- the controller ---------------------------------------------------
    def speculate_next(self) -> bool:
        c = self.controller
        mode = c.enabled() or not c.window_full()
        if self.probe_every > 0 and len(self.modes) % self.probe_every == self.probe_every - 1:
            mode = not mode
        return mode

    def _time_ratio(self) -> float:
        """Median speculative over median plain step time (the last 16 of
        each, the first of each mode dropped as warm-up); 1.0 until both
        are known."""
        ts, tp = self._t[True][1:], self._t[False][1:]
        if not ts or not tp:
            return 1.0
        return float(np.median(ts[-16:]) / np.median(tp[-16:]))

    def check(self) -> None:
        """Reads the device logs since the last check (one synchronisation)
        and feeds the step times, the statistics and the controller."""
        import torch
        if self._events:
            self._events[-1][2].synchronize()
        for mode, a, b in self._events:
            self._t[mode].append(a.elapsed_time(b))
        self._events.clear()
        ratio = self._time_ratio()
        for acc, running in self._pending:
            acc, running = acc.cpu().numpy(), running.cpu().numpy()
            for r in np.nonzero(running)[0]:
                a = int(acc[r])
                if a < 0:  # the row failed verification (its status says why)
                    continue
                for j in range(self.L):  # one MtpStatistics::record per drafted position
                    last = j == self.L - 1
                    self.stats.record(j < a, a + 1 if last else 0, 1 if last else 0)
                self.controller.record_net_benefit(float(a + 1) - ratio)
        self._pending.clear()

    def run(self, draft: Model, target: Model, rollback: Optional[Callable] = None,
            max_steps: Optional[int] = None, check_every: int = 8) -> int:
        """Steps until every row has stopped (checked with the controller
        every `check_every` steps) or max_steps; returns the steps taken."""
        import torch
        limit = max_steps if max_steps is not None else self.cap
        taken = 0
        while taken < limit:
            if taken % check_every == 0:
                self.check()
                if self.finished():
                    break
            mode = self.speculate_next()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            if mode:
                self.step_speculative(draft, target, rollback)
            else:
                self.step_plain(target, rollback)
            b.record()
            self._events.append((mode, a, b))
            self.modes.append(mode)
            taken += 1
        self.check()
        return taken
