"""Protocol-normalised parameters through the device path against the
oracle: `top_k` 0 (None: the general kernel), Ollama `repeat_last_n` -1 (the
whole history as the penalty window) and the reference's range edges
(penalties at +/-2, min_p, top_p 0 and 1) must sample exactly as the
reference sampler does on the same SamplingParams."""
import numpy as np
import pytest

from parity import compare, gpu_sample
from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.params import pack
from turboqwenfare_b200.protocol import ollama_sampling, openai_sampling

pytestmark = pytest.mark.gpu

REQUESTS = [
    ("ollama", {"temperature": 0.8, "top_k": 0, "top_p": 0.9, "repeat_last_n": -1, "repeat_penalty": 1.1}),
    ("ollama", {"temperature": 0.7, "top_k": 40, "repeat_last_n": -1, "repeat_penalty": 1.2,
                "frequency_penalty": 0.5, "presence_penalty": 0.3, "min_p": 0.05}),
    ("ollama", {"temperature": 1.3, "top_k": 128, "repeat_last_n": 0, "repeat_penalty": 2.0}),
    ("ollama", {"temperature": 2.0, "top_k": 20, "top_p": 0.0, "repeat_last_n": 4096,
                "repeat_penalty": 0.0, "frequency_penalty": -2.0}),
    ("openai", {"temperature": 1.0, "top_k": 0, "min_p": 0.1}),
    ("openai", {}),
    ("openai", {"temperature": 0.5, "top_p": 0.8, "top_k": 20, "frequency_penalty": -1.5,
                "presence_penalty": 2.0}),
    ("openai", {"temperature": 0.9, "top_k": 50, "top_p": 1.0, "min_p": 1.0}),
]


def test_normalised_requests_sample_like_the_reference(cuda_device):
    params = [ollama_sampling(o) if kind == "ollama" else openai_sampling(o) for kind, o in REQUESTS]
    rows = 4 * len(params)
    b = W.config("c4", rows=rows, seed=71)
    b.params = pack([params[i % len(params)] for i in range(rows)])
    rng = np.random.default_rng(72)
    lens = rng.integers(2000, 6000, rows)
    off = np.zeros(rows + 1, np.int64)
    off[1:] = np.cumsum(lens)
    hot = rng.choice(b.vocab, 300, replace=False)   # repeated ids, so the penalties bite
    b.hist = rng.choice(hot, int(off[-1])).astype(np.int32)
    b.hist_off = off
    g = gpu_sample(b, want_probs=True)
    assert (g.status == 0).all(), g.status
    rep = compare(b, g)
    print(rep)
    assert rep.identical + rep.boundary_ties == rep.rows
    assert rep.boundary_ties <= 1
