"""Implementation adapters for tests/reference_suite.py.

OracleImpl drives the CPU oracle (test infrastructure); ProductImpl drives
the GPU library through its public API (turboqwenfare_b200.Sampler et al.).
"""
from __future__ import annotations

import numpy as np

from turboqwenfare_b200.params import SamplingParams


class _OracleRng:
    def __init__(self, state):
        self.state = np.array(state, dtype=np.uint64)

    def next_u64(self):
        import oracle as O
        return O.xoshiro_next_u64(self.state)

    def next_f32(self):
        import oracle as O
        return O.xoshiro_next_f32(self.state)


class _OracleSampler:
    def __init__(self, params: SamplingParams):
        import oracle as O
        import time
        self.params = params.record()
        self.greedy = float(params.temperature) == 0.0
        seed = params.seed if params.seed is not None else time.time_ns()
        self.state = O.xoshiro_from_seed(seed)

    def is_greedy(self):
        return self.greedy

    def select(self, values, history, greedy_token):
        import oracle as O
        if self.greedy:
            return greedy_token
        return O.sample(values, history, self.params, rng_state=self.state).token


class OracleImpl:
    name = "oracle"

    def new(self, params):
        return _OracleSampler(params)

    def top_logit_candidates(self, values):
        import oracle as O
        return O.top_logit_candidates(values)

    def rng_from_seed(self, seed):
        import oracle as O
        return _OracleRng(O.xoshiro_from_seed(seed))

    def rng_from_state(self, state):
        return _OracleRng(state)

    def select_many(self, sampler, values, history, greedy, n):
        return [sampler.select(values, history, greedy) for _ in range(n)]

    def penalised_values(self, values, history, params):
        import oracle as O
        return O.apply_penalties(values, history, params.record())


class ProductImpl:
    name = "gpu"

    def __init__(self):
        import turboqwenfare_b200 as T
        self.T = T

    def new(self, params):
        return self.T.Sampler.new(params)

    def top_logit_candidates(self, values):
        return [(c.token, c.logit) for c in self.T.top_logit_candidates(values)]

    def rng_from_seed(self, seed):
        return self.T.Xoshiro256PlusPlus.from_seed(seed)

    def rng_from_state(self, state):
        return self.T.Xoshiro256PlusPlus(state)

    def select_many(self, sampler, values, history, greedy, n):
        return [sampler.select(values, history, greedy) for _ in range(n)]

    def penalised_values(self, values, history, params):
        return self.T.apply_penalties(values, history, params)
