"""The reference sampler's own unit tests (src/sampling/mod.rs:333-693) run
against the GPU product through its public API: Sampler.new/select,
top_logit_candidates, Xoshiro256PlusPlus and apply_penalties."""
import pytest

import reference_suite as S
from impls import ProductImpl

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def impl(cuda_device):
    return ProductImpl()


@pytest.mark.parametrize("case", S.ALL, ids=[f.__name__ for f in S.ALL])
def test_reference_case_on_gpu(impl, case):
    case(impl)


def test_gpu_sampler_stream_matches_oracle_draw_for_draw(impl):
    """Same seed, same logits: the GPU Sampler and the oracle pick the same
    token at every step (full-vocabulary rows, the general kernel)."""
    import numpy as np
    import oracle as O
    from turboqwenfare_b200.params import SamplingParams
    values = S.logits(impl, 3000, 21)
    params = SamplingParams(temperature=0.9, top_p=0.93, min_p=0.01, seed=77)
    s = impl.new(params)
    st = O.xoshiro_from_seed(77)
    rec = params.record()
    for _ in range(300):
        assert s.select(values, [], 0) == O.sample(values, [], rec, rng_state=st).token
