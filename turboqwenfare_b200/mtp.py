"""MTP verification: greedy `verify_pair`, statistics and controller, and the
batched device verify.

Host-side mirror of src/runtime/mtp.rs:47-168. `verify_batch` runs
`tqfs_mtp_verify`: the greedy rule of verify_pair for temperature-0
sequences, and speculative sampling over the sampler's post-filter
distributions for sampled ones (the rule is documented in include/tqfs.h).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class VerifyOutcome:
    """`VerifyOutcome::{Accepted, Rejected} { emitted_tokens }` (mtp.rs:92-96)."""

    accepted: bool
    emitted_tokens: int

    @classmethod
    def Accepted(cls, emitted_tokens: int) -> "VerifyOutcome":
        return cls(True, emitted_tokens)

    @classmethod
    def Rejected(cls, emitted_tokens: int) -> "VerifyOutcome":
        return cls(False, emitted_tokens)


def verify_pair(target_prediction_after_boundary: int, draft_token: int) -> VerifyOutcome:
    """mtp.rs:98-104: accept iff the target's greedy prediction equals the draft."""
    if target_prediction_after_boundary == draft_token:
        return VerifyOutcome.Accepted(2)
    return VerifyOutcome.Rejected(1)


@dataclass
class MtpStatistics:
    """mtp.rs:47-83."""

    drafted_tokens: int = 0
    accepted_tokens: int = 0
    target_backbone_passes: int = 0
    emitted_tokens: int = 0

    def acceptance_rate(self) -> float:
        return 0.0 if self.drafted_tokens == 0 else self.accepted_tokens / self.drafted_tokens

    def emitted_tokens_per_target_pass(self) -> float:
        return 0.0 if self.target_backbone_passes == 0 else self.emitted_tokens / self.target_backbone_passes

    def record(self, accepted: bool, emitted: int, target_passes: int) -> None:
        self.drafted_tokens += 1
        if accepted:
            self.accepted_tokens += 1
        self.target_backbone_passes += target_passes
        self.emitted_tokens += emitted


class MtpController:
    """Hysteresis controller (mtp.rs:112-168): enable above +0.10 rolling net
    benefit, disable below -0.05, only once the window is full."""

    def __init__(self, window_capacity: int):
        self.window: list[float] = []
        self.window_capacity = window_capacity
        self._enabled = False
        self.enable_threshold = 0.10
        self.disable_threshold = -0.05

    def enabled(self) -> bool:
        return self._enabled

    def _rolling_net_benefit(self) -> float:
        return 0.0 if not self.window else sum(self.window) / len(self.window)

    def window_full(self) -> bool:
        return len(self.window) == self.window_capacity

    def record_and_decide(self, emitted_tokens: int) -> bool:
        return self.record_net_benefit(float(emitted_tokens) - 1.0)

    def record_net_benefit(self, net_benefit: float) -> bool:
        """The body of record_and_decide (mtp.rs:147-168) for a net benefit
        the caller has already computed; record_and_decide(e) is
        record_net_benefit(e - 1.0). A loop that charges a speculative step's
        extra time against it passes emitted - t_speculative / t_plain."""
        if len(self.window) == self.window_capacity:
            self.window.pop(0)
        self.window.append(net_benefit)
        if len(self.window) < self.window_capacity:
            return self._enabled
        rolling = self._rolling_net_benefit()
        if not self._enabled and rolling > self.enable_threshold:
            self._enabled = True
        elif self._enabled and rolling < self.disable_threshold:
            self._enabled = False
        return self._enabled


@dataclass
class MtpBatchResult:
    """Per sequence: drafts accepted (0..L), the token to append, the status
    (0 ok, 2 unsupported: active penalty); mask: every position's decision."""

    accepted: "object"
    token: "object"
    mask: "object"
    status: "object"


def verify_batch(target, draft, drafts, params, uniforms, vocab=None, handle=None) -> MtpBatchResult:
    """Device MTP verify over CUDA tensors.

    target: (seqs, L+1, ld) float32/bfloat16; draft: (seqs, L, ld) of the same
    dtype; drafts: (seqs, L) int32; params: one tqfs_params per sequence
    (numpy PARAMS_DTYPE array, SamplingParams list or packed uint8 tensor);
    uniforms: (seqs, L+1) float32 on the 2^-24 grid.
    """
    import torch
    from . import _native as N
    from .sampler import params_tensor, _ptr, _stream

    seqs, L1, ld = target.shape
    L = L1 - 1
    dev = target.device
    h = handle or N.default_handle(dev.index or 0)
    dtype = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}.get(target.dtype)
    if dtype is None or draft.dtype != target.dtype:
        raise N.TqfsError(N.ERR_UNSUPPORTED_DTYPE, str(target.dtype))
    if not (isinstance(params, torch.Tensor) and params.dtype == torch.uint8):
        params = params_tensor(params, seqs, dev)
    acc = torch.empty(seqs, dtype=torch.int32, device=dev)
    tok = torch.empty(seqs, dtype=torch.int32, device=dev)
    mask = torch.empty((seqs, max(L, 1)), dtype=torch.uint8, device=dev)
    status = torch.empty(seqs, dtype=torch.int32, device=dev)
    n = ld if vocab is None else vocab
    h.check(N.lib().tqfs_mtp_verify(
        h.ptr, _ptr(target), _ptr(draft), dtype, seqs, L, n, ld, _ptr(drafts), _ptr(params),
        _ptr(uniforms), _ptr(acc), _ptr(tok), _ptr(mask), _ptr(status), _stream(dev)))
    return MtpBatchResult(acc, tok, mask[:, :L], status)
