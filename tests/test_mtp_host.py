"""MTP host-side tests restated from src/runtime/mtp.rs:211-266."""
from turboqwenfare_b200.mtp import MtpController, MtpStatistics, VerifyOutcome, verify_pair


def test_verify_pair_matches_nvmai_accept_reject_semantics():
    assert verify_pair(42, 42) == VerifyOutcome.Accepted(2)
    assert verify_pair(42, 7) == VerifyOutcome.Rejected(1)


def test_statistics_track_acceptance_rate_and_emitted_per_pass():
    stats = MtpStatistics()
    stats.record(True, 2, 1)
    stats.record(False, 1, 1)
    stats.record(True, 2, 1)
    assert stats.drafted_tokens == 3
    assert stats.accepted_tokens == 2
    assert abs(stats.acceptance_rate() - 2.0 / 3.0) < 1e-9
    assert stats.emitted_tokens == 5
    assert stats.target_backbone_passes == 3
    assert abs(stats.emitted_tokens_per_target_pass() - 5.0 / 3.0) < 1e-9


def test_controller_enables_only_after_a_sustained_positive_rolling_benefit():
    c = MtpController(4)
    assert not c.enabled()
    c.record_and_decide(2)
    assert not c.enabled()
    for _ in range(4):
        c.record_and_decide(2)
    assert c.enabled()


def test_controller_disables_after_a_sustained_negative_rolling_benefit():
    c = MtpController(4)
    for _ in range(4):
        c.record_and_decide(2)
    assert c.enabled()
    for _ in range(4):
        c.record_and_decide(0)
    assert not c.enabled()


def test_oracle_verify_pair_agrees():
    import oracle as O
    assert O.verify_pair(42, 42) == 2
    assert O.verify_pair(42, 7) == 1


def test_net_benefit_entry_is_record_and_decide_shifted_by_one():
    a, b = MtpController(3), MtpController(3)
    for e in [2, 2, 1, 0, 0, 0, 2, 2, 2, 2]:
        assert a.record_and_decide(e) == b.record_net_benefit(e - 1.0)
        assert a.window == b.window and a.window_full() == b.window_full()


def test_time_charged_net_benefit_keeps_mtp_off():
    """A verification that emits 2 tokens in 2.5 plain steps' time is a loss."""
    c = MtpController(4)
    for _ in range(8):
        c.record_net_benefit(2.0 - 2.5)
    assert not c.enabled()
