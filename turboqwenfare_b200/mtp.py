"""MTP verification: greedy `verify_pair`, statistics and controller.

Host-side mirror of src/runtime/mtp.rs:47-168. The batched device verify
(stochastic speculative sampling over post-filter distributions) is exposed
by `mtp_verify` once the library provides it.
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

    def record_and_decide(self, emitted_tokens: int) -> bool:
        net_benefit = float(emitted_tokens) - 1.0
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
