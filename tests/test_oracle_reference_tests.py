"""Pins the CPU oracle against the reference sampler's own known-answer tests
(src/sampling/mod.rs:360-692) and the MTP host-side tests
(src/runtime/mtp.rs:211-266). No GPU needed."""
import pytest

import reference_suite as S
from impls import OracleImpl

IMPL = OracleImpl()


@pytest.mark.parametrize("case", S.ALL, ids=[f.__name__ for f in S.ALL])
def test_reference_case_on_oracle(case):
    case(IMPL)


def test_oracle_pinned_choices_are_reported():
    """Top-k ties are resolved to the lowest ids and flagged."""
    import numpy as np
    import oracle as O
    from turboqwenfare_b200.workloads import params_rows
    p = params_rows(1, 1.0, top_k=2)[0]
    r = O.sample(np.array([1.0, 3.0, 3.0, 3.0], np.float32), [], p, u=0.99, dense=True)
    assert r.debug.topk_tie == 1
    assert list(np.nonzero(r.probs)[0]) == [1, 2]


def test_uniform_draw_consumption_matches_reference():
    """A degenerate total (all-NaN logits) returns the first candidate and
    consumes no uniform (src/sampling/mod.rs:235-237)."""
    import numpy as np
    import oracle as O
    from turboqwenfare_b200.workloads import params_rows
    st = O.xoshiro_from_seed(9)
    before = st.copy()
    p = params_rows(1, 1.0)[0]
    r = O.sample(np.full(5, np.nan, np.float32), [], p, rng_state=st)
    assert r.token == 0 and r.debug.consumed == 0
    assert (st == before).all()
