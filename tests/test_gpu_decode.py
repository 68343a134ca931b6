"""§8(f3): the batched decode loop (turboqwenfare_b200.DecodeLoop) against a
CPU reference loop that runs src/runtime/generation.rs:714-770 per request
with the oracle as its sampler: push the token into `generated`, stop at the
end-of-sequence token or after `maximum` pushes, sample the next token
against `generated` with the request's seeded xoshiro256++ stream. The
logits come from a synthetic autoregressive producer (a bank of logits rows
permuted by the previous token), computed identically on the device (torch)
and on the host (numpy). Every row's generated tokens must match; a row may
stop being compared only after a counted CDF boundary tie (the sequences
then legitimately diverge)."""
import numpy as np
import pytest

from parity import BOUNDARY_TOL
from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.decode import DecodeLoop
from turboqwenfare_b200.params import USIZE_MAX, SamplingParams

pytestmark = pytest.mark.gpu

V = 24_576
NB = 5


def _bank(seed=3):
    rng = np.random.default_rng(seed)
    return W.zipf_logits(rng, NB, V)


def _shift(step, last, r):
    return (int(last) * 7919 + 131 * r + 17 * step) % V


def _host_logits(bank, step, last, r, eos):
    x = np.roll(bank[r % NB], -_shift(step, last, r)).astype(np.float32)
    if eos[r] >= 0:
        x[eos[r]] = np.float32(x[eos[r]] + np.float32(4.0))
    return x


def _device_producer(bank_dev, eos):
    import torch
    rows = len(eos)
    dev = bank_dev.device
    ar = torch.arange(V, device=dev)
    r = torch.arange(rows, device=dev)
    rows_bank = bank_dev[r % NB]
    eos_col = torch.tensor([max(e, 0) for e in eos], device=dev)[:, None]
    boost = torch.tensor([4.0 if e >= 0 else 0.0 for e in eos], dtype=torch.float32, device=dev)[:, None]

    def produce(step, last):  # static shapes only, so a step can be captured in a graph
        shift = (last * 7919 + 131 * r + 17 * step) % V
        x = torch.gather(rows_bank, 1, (ar[None, :] + shift[:, None]) % V)
        x.scatter_add_(1, eos_col, boost)  # +4 at the row's end-of-sequence id, +0 elsewhere
        return x
    return produce


def _requests():
    P = SamplingParams
    ps = [
        P(temperature=0.0),
        P(temperature=0.7, top_k=20, top_p=0.9, seed=11),
        P(temperature=1.0, top_k=50, seed=12, repeat_penalty=1.3, repeat_last_n=64),
        P(temperature=0.9, top_k=0, top_p=0.8, seed=13, frequency_penalty=0.5, presence_penalty=0.4,
          repeat_last_n=USIZE_MAX),
        P(temperature=1.2, top_k=40, min_p=0.05, seed=14, repeat_penalty=1.1, repeat_last_n=USIZE_MAX),
        P(temperature=0.5, top_k=128, seed=15, presence_penalty=1.5, repeat_last_n=3),
        P(temperature=0.0, repeat_penalty=1.5),
        P(temperature=1.5, top_k=5, seed=16, frequency_penalty=-0.5, repeat_last_n=USIZE_MAX),
    ]
    rows = 3 * len(ps)
    params = [ps[i % len(ps)] for i in range(rows)]
    params = [SamplingParams(**{**p.__dict__, "seed": (p.seed or 0) + 100 * i if p.seed is not None else None})
              for i, p in enumerate(params)]
    first = [(37 * i + 5) % V for i in range(rows)]
    maxt = [6 + (i * 7) % 35 for i in range(rows)]
    eos = [((13 * i + 1) % V) if i % 3 else -1 for i in range(rows)]
    return params, first, maxt, eos


def _reference_loop(bank, params, first, maxt, eos):
    import oracle as O
    out, margins = [], []
    for r, p in enumerate(params):
        gen, mar = [first[r]], []
        state = O.xoshiro_from_seed(p.seed) if p.seed is not None else None
        rec = p.record()
        step = 0
        if not (first[r] == eos[r] or maxt[r] <= 1):
            while len(gen) < maxt[r]:
                x = _host_logits(bank, step, gen[-1], r, eos)
                if p.temperature == 0.0:  # the greedy arm returns top_logit_candidates' first (runtime.rs:442-443)
                    tok, margin = O.top_logit_candidates(x)[0][0], np.inf
                else:
                    res = O.sample(x, np.array(gen, np.int64).astype(np.uint32), rec, rng_state=state)
                    tok, margin = int(res.token), min(res.debug.cdf_margin, res.debug.topp_margin)
                gen.append(int(tok))
                mar.append(margin)
                step += 1
                if tok == eos[r]:
                    break
        out.append(gen)
        margins.append(mar)
    return out, margins


def test_decode_loop_matches_the_reference_loop(cuda_device):
    import torch
    bank = _bank()
    params, first, maxt, eos = _requests()
    loop = DecodeLoop(params, first, V, maxt, eos)
    produce = _device_producer(torch.from_numpy(bank).cuda(), eos)
    steps = loop.run(produce)
    torch.cuda.synchronize()
    assert loop.finished()
    got = loop.generated()
    want, margins = _reference_loop(bank, params, first, maxt, eos)
    ties = 0
    stopped_early = 0
    for r in range(len(params)):
        g, w = got[r], want[r]
        n = min(len(g), len(w))
        k = next((i for i in range(n) if g[i] != w[i]), None)
        if k is None:
            assert len(g) == len(w), (r, g, w)
        else:
            assert margins[r][k - 1] < BOUNDARY_TOL, (r, k, g, w)
            ties += 1
        stopped_early += len(w) < maxt[r]
    assert ties <= 1
    assert stopped_early >= 2  # some rows met their end-of-sequence token
    assert steps <= max(maxt)


def test_decode_loop_replays_from_a_captured_graph(cuda_device):
    """The loop's step (producer, tqfs_sample, tqfs_decode_append) captured
    once and replayed must generate what the eager loop generates."""
    import torch
    bank = _bank(4)
    params, first, maxt, eos = _requests()
    eager = DecodeLoop(params, first, V, maxt, eos)
    produce = _device_producer(torch.from_numpy(bank).cuda(), eos)
    eager.run(produce)
    import turboqwenfare_b200._native as N
    h = N.Handle(0)
    loop = DecodeLoop(params, first, V, maxt, eos, handle=h)
    logits = torch.empty((len(params), V), dtype=torch.float32, device="cuda")
    step_t = torch.zeros((), dtype=torch.int64, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):   # warm-up outside the capture sizes every buffer
        logits.copy_(produce(step_t, loop.last_tokens()))
        loop.step(logits)
        step_t += 1
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="relaxed"):
        logits.copy_(produce(step_t, loop.last_tokens()))
        loop.step(logits)
        step_t += 1
    for _ in range(max(maxt)):
        g.replay()
    torch.cuda.synchronize()
    assert loop.generated() == eager.generated()
    del g
    h.close()
