"""The decode loop's history layout (turboqwenfare_b200/decode.py,
tqfs_decode_append) hands tqfs_sample each row's tokens preceded by -1
padding (the previous row's unused slot). The reference never lets an id
outside [0, vocab) match (src/sampling/mod.rs:135-138), so padding in front
of a history must leave apply_penalties unchanged for every window length.
Checked on the CPU oracle, which restates apply_penalties."""
import numpy as np
import pytest

from turboqwenfare_b200.params import USIZE_MAX, SamplingParams

PAD = np.uint32(0xFFFFFFFF)  # -1 as the reference's u32 token


@pytest.mark.parametrize("window", [0, 1, 3, 64, 500, USIZE_MAX])
def test_padding_in_front_of_a_history_changes_no_penalty(window):
    import oracle as O
    rng = np.random.default_rng(window % 1000)
    V = 3000
    values = (rng.standard_normal(V) * 3).astype(np.float32)
    for trial in range(6):
        hist = rng.integers(0, 40 if trial % 2 else V, size=int(rng.integers(0, 300))).astype(np.uint32)
        p = SamplingParams(temperature=0.8, repeat_penalty=1.3, frequency_penalty=0.4, presence_penalty=-0.7,
                           repeat_last_n=window).record()
        want = O.apply_penalties(values, hist, p)
        for pad in (0, 1, 7, 1000):
            got = O.apply_penalties(values, np.concatenate([np.full(pad, PAD, np.uint32), hist]), p)
            np.testing.assert_array_equal(got, want)
