"""The reference sampler's own unit tests (src/sampling/mod.rs:333-693),
restated against an implementation object so the same assertions pin both
the CPU oracle and the GPU product.

An implementation provides:
  new(params) -> sampler with .is_greedy() and .select(values, history, greedy)
  top_logit_candidates(values) -> [(token, logit)] * 4
  xoshiro(seed_or_state) helpers via .rng_from_seed(seed) / .rng_from_state(state)
  penalised_top1(values, history, params) -> token of the top-1 candidate
    after penalties (exact penalty values are checked through it)
"""
from __future__ import annotations

import math

import numpy as np

from turboqwenfare_b200.params import SamplingParams


def greedy_params() -> SamplingParams:
    return SamplingParams()


def stochastic(temperature: float, seed: int) -> SamplingParams:
    return SamplingParams(temperature=temperature, seed=seed)


def logits(impl, count: int, seed: int) -> np.ndarray:
    """mod.rs:351-354: xoshiro next_f32() * 20 - 10."""
    rng = impl.rng_from_seed(seed)
    return np.array([np.float32(np.float32(rng.next_f32()) * np.float32(20.0)) - np.float32(10.0)
                     for _ in range(count)], dtype=np.float32)


def test_greedy_returns_exactly_the_argmax_the_decoder_already_computed(impl, seeds=range(500)):
    for seed in seeds:
        values = logits(impl, 1024, seed)
        expected = impl.top_logit_candidates(values)[0][0]
        s = impl.new(greedy_params())
        assert s.is_greedy()
        assert s.select(values, [], expected) == expected, f"greedy selection diverged on seed {seed}"


def test_default_sampling_params_are_greedy(impl):
    assert SamplingParams().temperature == 0.0
    assert impl.new(SamplingParams()).is_greedy()


def test_temperature_zero_stays_greedy_regardless_of_other_knobs(impl):
    params = SamplingParams(temperature=0.0, top_p=0.5, top_k=3, min_p=0.1, seed=7, repeat_penalty=1.5,
                            frequency_penalty=0.9, presence_penalty=0.9)
    values = logits(impl, 512, 99)
    expected = impl.top_logit_candidates(values)[0][0]
    s = impl.new(params)
    assert s.is_greedy()
    assert s.select(values, [1, 1, 1], expected) == expected


def test_greedy_tie_break_prefers_the_lower_token_index(impl):
    values = np.array([1.0, 5.0, 5.0, 5.0, 2.0], np.float32)
    assert impl.top_logit_candidates(values)[0][0] == 1


def test_a_nan_logit_never_wins_at_realistic_vocabulary_size(impl):
    values = (np.arange(4096, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    values[2000] = np.nan
    expected = impl.top_logit_candidates(values)[0][0]
    s = impl.new(stochastic(1.0, 17))
    for _ in range(200):
        token = s.select(values, [], expected)
        assert not math.isnan(values[token]), f"selected the NaN token {token}"


def test_a_nan_logit_is_never_selected(impl):
    values = np.array([1.0, np.nan, 3.0, np.nan], np.float32)
    assert impl.top_logit_candidates(values)[0][0] == 2
    s = impl.new(stochastic(1.0, 5))
    for _ in range(50):
        token = s.select(values, [], 2)
        assert token in (0, 2), f"selected a NaN token: {token}"


def test_the_same_seed_reproduces_the_same_sequence_and_different_seeds_diverge(impl):
    values = logits(impl, 256, 3)

    def run(seed):
        s = impl.new(stochastic(1.0, seed))
        return [s.select(values, [], 0) for _ in range(40)]

    assert run(42) == run(42), "a seeded run must be reproducible"
    assert run(42) != run(43), "different seeds must produce different runs"


def test_draw_frequencies_track_the_softmax_distribution(impl, draws=200_000):
    values = np.array([3.0, 2.0, 1.0, 0.0], np.float32)
    ex = np.exp(values.astype(np.float64))
    expected = ex / ex.sum()
    counts = np.zeros(4, np.int64)
    s = impl.new(stochastic(1.0, 20260819))
    toks = impl.select_many(s, values, [], 0, draws)
    for t in toks:
        counts[t] += 1
    for token in range(4):
        observed = counts[token] / draws
        assert abs(observed - expected[token]) < 0.01, (token, observed, expected[token])


def test_temperature_controls_how_concentrated_the_draw_is(impl):
    values = np.array([3.0, 2.0, 1.0, 0.0], np.float32)

    def argmax_share(temperature):
        s = impl.new(stochastic(temperature, 11))
        toks = impl.select_many(s, values, [], 0, 20_000)
        return sum(1 for t in toks if t == 0) / 20_000.0

    cold, hot = argmax_share(0.1), argmax_share(5.0)
    assert cold > 0.99, cold
    assert hot < 0.45, hot
    assert cold > hot


def test_top_k_restricts_selection_to_the_k_highest_logits(impl):
    values = np.array([0.0, 10.0, 9.5, 1.0, 0.5], np.float32)
    s = impl.new(SamplingParams(temperature=2.0, top_k=2, seed=1))
    for token in impl.select_many(s, values, [], 1, 2_000):
        assert token in (1, 2), f"top_k=2 leaked token {token}"


def test_top_p_keeps_the_smallest_prefix_reaching_the_threshold(impl):
    values = np.array([3.0, 2.0, 1.0, 0.0], np.float32)
    s = impl.new(SamplingParams(temperature=1.0, top_p=0.8, seed=2))
    for token in impl.select_many(s, values, [], 0, 5_000):
        assert token < 2, f"top_p=0.8 leaked token {token}"


def test_min_p_drops_candidates_far_below_the_most_likely_one(impl):
    values = np.array([5.0, 2.0, 1.0, 0.0], np.float32)
    s = impl.new(SamplingParams(temperature=1.0, min_p=0.5, seed=3))
    for token in impl.select_many(s, values, [], 0, 2_000):
        assert token == 0


def test_repetition_penalty_lowers_repeated_tokens_of_either_sign(impl):
    params = SamplingParams(temperature=1.0, repeat_penalty=2.0)
    got = impl.penalised_values(np.array([4.0, -4.0, 4.0], np.float32), [0, 1], params)
    assert got[0] == 2.0, "positive logit must be divided"
    assert got[1] == -8.0, "negative logit must be multiplied"
    assert got[2] == 4.0, "unrepeated token must be untouched"


def test_the_repetition_window_ignores_tokens_older_than_repeat_last_n(impl):
    params = SamplingParams(temperature=1.0, repeat_penalty=2.0, repeat_last_n=2)
    values = np.zeros(10, np.float32)
    values[9] = 4.0
    got = impl.penalised_values(values, [9, 1, 2], params)
    assert got[9] == 4.0


def test_frequency_penalty_scales_with_count_while_presence_is_binary(impl):
    frequency = SamplingParams(temperature=1.0, frequency_penalty=1.0)
    got = impl.penalised_values(np.array([10.0], np.float32), [0, 0, 0], frequency)
    assert got[0] == 7.0, "three repeats, penalty 1.0 each"
    presence = SamplingParams(temperature=1.0, presence_penalty=1.0)
    got = impl.penalised_values(np.array([10.0], np.float32), [0, 0, 0], presence)
    assert got[0] == 9.0, "presence applies once regardless of count"


def test_xoshiro256pp_matches_its_reference_definition(impl):
    rng = impl.rng_from_state([1, 1, 1, 1])
    assert rng.next_u64() == 16_777_217
    assert rng.next_u64() != 16_777_217, "state must advance"


def test_next_f32_stays_in_the_unit_interval(impl):
    rng = impl.rng_from_seed(12345)
    for _ in range(100_000):
        v = rng.next_f32()
        assert 0.0 <= v < 1.0, v


def test_seeding_from_zero_still_produces_a_well_mixed_stream(impl):
    rng = impl.rng_from_seed(0)
    first = [rng.next_u64() for _ in range(8)]
    assert all(v != 0 for v in first)
    assert len(set(first)) == 8


ALL = [v for k, v in sorted(globals().items()) if k.startswith("test_") and callable(v)]
