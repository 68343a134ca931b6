"""Protocol normalisation (turboqwenfare_b200.protocol) against the
reference's mappings: src/server/openai/mod.rs:276-329 and
src/server/ollama/mod.rs:211-273. CPU only; the device path over the mapped
parameters is tests/test_gpu_protocol.py."""
import pytest

from turboqwenfare_b200.params import USIZE_MAX, SamplingParams
from turboqwenfare_b200.protocol import ProtocolError, ollama_sampling, openai_sampling


def test_openai_defaults_are_greedy_and_neutral():
    p = openai_sampling({})
    assert p.temperature == 0.0 and p.top_p == 1.0 and p.top_k is None and p.min_p is None
    assert p.seed is None and p.repeat_penalty == 1.0 and p.repeat_last_n == 64
    assert p.record()["top_k"] == 0 and p.record()["flags"] == 0


def test_openai_top_k_zero_is_off_and_fields_map():
    p = openai_sampling({"temperature": 0.7, "top_p": 0.9, "top_k": 0, "min_p": 0.05, "seed": 7,
                         "frequency_penalty": -2.0, "presence_penalty": 2.0, "max_tokens": 33,
                         "max_completion_tokens": 12, "stop": ["", "###"]})
    assert p.top_k is None and p.record()["top_k"] == 0
    assert p.min_p == pytest.approx(0.05) and p.record()["flags"] == 1
    assert p.seed == 7 and p.frequency_penalty == -2.0 and p.presence_penalty == 2.0
    assert p.max_output_tokens == 12          # max_completion_tokens wins over max_tokens
    assert p.stop_sequences == ["###"]        # empty stop strings are dropped
    assert openai_sampling({"top_k": 40}).top_k == 40


@pytest.mark.parametrize("field,value,msg", [
    ("temperature", 2.5, "temperature must be a finite value between 0 and 2"),
    ("temperature", float("nan"), "temperature must be a finite value between 0 and 2"),
    ("top_p", -0.1, "top_p must be a finite value between 0 and 1"),
    ("min_p", 1.5, "min_p must be a finite value between 0 and 1"),
    ("frequency_penalty", 2.01, "frequency_penalty must be a finite value between -2 and 2"),
    ("presence_penalty", float("inf"), "presence_penalty must be a finite value between -2 and 2"),
    ("max_tokens", 0, "max output tokens must be at least 1"),
    ("stop", ["a", "b", "c", "d", "e"], "at most 4 stop sequences are supported"),
    ("stop", [1], "stop entries must be strings"),
    ("stop", 3, "stop must be a string or an array of strings"),
])
def test_openai_rejections_match_the_reference(field, value, msg):
    with pytest.raises(ProtocolError, match=msg.replace("(", r"\(")):
        openai_sampling({field: value})


def test_ollama_minus_one_window_is_whole_context_and_seed_minus_one_is_none():
    p = ollama_sampling({"repeat_last_n": -1, "seed": -1, "top_k": 0, "num_predict": -2})
    assert p.repeat_last_n == USIZE_MAX and p.record()["repeat_last_n"] == USIZE_MAX
    assert p.seed is None and p.top_k is None and p.max_output_tokens is None
    q = ollama_sampling({"repeat_last_n": 0, "seed": 0, "num_predict": 2**40, "temperature": 0.0})
    assert q.repeat_last_n == 0 and q.seed == 0 and q.max_output_tokens == 2**32 - 1


def test_ollama_defaults_keep_sampling_params_default():
    assert ollama_sampling(None).record() == SamplingParams().record()
    p = ollama_sampling({"mirostat": 0, "tfs_z": 1.0, "typical_p": 1.0, "repeat_penalty": 1.1,
                         "stop": "\n"})
    assert p.repeat_penalty == pytest.approx(1.1) and p.stop_sequences == ["\n"]


@pytest.mark.parametrize("opts,msg", [
    ({"mirostat": 2}, "mirostat sampling is not implemented in this build"),
    ({"tfs_z": 0.9}, r"tail-free sampling \(tfs_z\) is not implemented in this build"),
    ({"typical_p": 0.5}, "typical_p sampling is not implemented in this build"),
    ({"repeat_penalty": 2.5}, "repeat_penalty must be a finite value between 0 and 2"),
    ({"temperature": -1.0}, "temperature must be a finite value between 0 and 2"),
])
def test_ollama_rejections_match_the_reference(opts, msg):
    with pytest.raises(ProtocolError, match=msg):
        ollama_sampling(opts)
