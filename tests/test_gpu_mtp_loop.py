"""MTP speculative decoding end to end (turboqwenfare_b200.MtpDecodeLoop):
draft head, target pass, tqfs_mtp_verify, commit, KV rollback and the
MtpController (src/runtime/mtp.rs:47-168) against a CPU reference loop that
runs the same steps per request with the oracle (sampler, verify) and a
numpy copy of the synthetic model.

The synthetic target model keeps a KV cache of its input tokens on the
device and appends every input at its own cache length; its logits depend
on a weighted sum over the whole cached prefix, so a cache that kept a
rejected draft's entry would change every later row. The draft head scores
(token, position) only. The reference loop computes the target's logits
from the committed tokens, so parity holds only if the loop rolls the cache
back to len - 1 entries after every step."""
import numpy as np
import pytest

from parity import BOUNDARY_TOL
from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.decode import MtpDecodeLoop
from turboqwenfare_b200.mtp import MtpController, MtpStatistics, verify_pair
from turboqwenfare_b200.params import PARAMS_DTYPE, SamplingParams

pytestmark = pytest.mark.gpu

V = 24_576
NB = 5
CTX_MOD = 4099
CTX_SCALE = np.float32(0.0625)   # a power of two: the product is exact on both sides
EOS_BOOST = np.float32(4.0)


def _banks(seed=5):
    rng = np.random.default_rng(seed)
    return W.zipf_logits(rng, NB, V), W.zipf_logits(rng, NB, V)


def _shift(pos, tok, r):
    return (int(tok) * 7919 + 131 * r + 17 * int(pos)) % V


def _ctx(tokens):
    return sum((i + 1) * int(t) for i, t in enumerate(tokens)) % CTX_MOD


def _host_target(banks, ctx, r, eos):
    """Logits after the last token of ctx (tokens at positions 0..len-1)."""
    b1, b2 = banks
    p = len(ctx) - 1
    x = np.roll(b1[r % NB], -_shift(p, ctx[-1], r))
    y = np.roll(b2[r % NB], -((_ctx(ctx) * 977) % V)) * CTX_SCALE
    x = (x + y).astype(np.float32)
    if eos[r] >= 0:
        x[eos[r]] = np.float32(x[eos[r]] + EOS_BOOST)
    return x


def _host_draft(banks, tok, pos, r, eos):
    x = np.roll(banks[0][r % NB], -_shift(pos, tok, r)).astype(np.float32)
    if eos[r] >= 0:
        x[eos[r]] = np.float32(x[eos[r]] + EOS_BOOST)
    return x


class DeviceModel:
    """Target with a device KV cache of token ids, and a stateless draft head.
    `heavy` adds a fixed-cost matrix product to every target call (a real
    target's cost hardly depends on how many positions one pass scores)."""

    def __init__(self, banks, eos, rows, cap, heavy=0):
        import torch
        self.dev = torch.device("cuda")
        self.b1 = torch.from_numpy(banks[0]).to(self.dev)
        self.b2 = torch.from_numpy(banks[1]).to(self.dev)
        r = torch.arange(rows, device=self.dev)
        self.r = r
        self.rows1, self.rows2 = self.b1[r % NB], self.b2[r % NB]
        self.ar = torch.arange(V, device=self.dev)
        self.kv = torch.zeros((rows, cap + 8), dtype=torch.int64, device=self.dev)
        self.kv_len = torch.zeros(rows, dtype=torch.int64, device=self.dev)
        self.w = torch.arange(1, cap + 9, device=self.dev, dtype=torch.int64)
        self.eos_col = torch.tensor([max(e, 0) for e in eos], device=self.dev)[:, None]
        self.boost = torch.tensor([float(EOS_BOOST) if e >= 0 else 0.0 for e in eos], device=self.dev)[:, None]
        self.heavy = None
        if heavy:
            self.heavy = torch.randn((heavy, heavy), device=self.dev, dtype=torch.bfloat16)
        self.target_calls = 0
        self.draft_calls = 0

    def _bigram(self, tokens, positions):
        rows, n = tokens.shape
        shift = (tokens * 7919 + 131 * self.r[:, None] + 17 * positions) % V          # (rows, n)
        idx = (self.ar[None, None, :] + shift[:, :, None]) % V
        return torch_gather(self.rows1, idx)

    def _boost(self, x):
        n = x.shape[1]
        x.scatter_add_(2, self.eos_col[:, None, :].expand(-1, n, 1), self.boost[:, None, :].expand(-1, n, 1))
        return x

    def target(self, tokens, positions):
        import torch
        self.target_calls += 1
        n = tokens.shape[1]
        idx = self.kv_len[:, None] + torch.arange(n, device=self.dev)[None, :]
        self.kv.scatter_(1, idx, tokens)
        self.kv_len += n
        cs = torch.cumsum(self.kv * self.w[None, :], 1)
        g = torch.gather(cs, 1, idx) % CTX_MOD
        x = self._bigram(tokens, positions)
        y = torch_gather(self.rows2, (self.ar[None, None, :] + ((g * 977) % V)[:, :, None]) % V) * float(CTX_SCALE)
        x = x + y
        if self.heavy is not None:
            self.heavy @ self.heavy
        return self._boost(x)

    def draft(self, tokens, positions):
        self.draft_calls += 1
        return self._boost(self._bigram(tokens, positions))

    def rollback(self, kv_len):
        self.kv_len.copy_(kv_len.long())


def torch_gather(rows_bank, idx):
    """out[r, j, v] = rows_bank[r, idx[r, j, v]]."""
    import torch
    rows, n, v = idx.shape
    return torch.gather(rows_bank[:, None, :].expand(rows, n, rows_bank.shape[1]), 2, idx)


def _requests(rows=16):
    P = SamplingParams
    ps = [
        P(temperature=0.0),
        P(temperature=0.7, top_k=20, top_p=0.9, seed=11),
        P(temperature=1.0, top_k=50, seed=12),
        P(temperature=0.9, top_k=0, top_p=0.8, seed=13),
        P(temperature=1.2, top_k=40, min_p=0.05, seed=14),
        P(temperature=0.5, top_k=128, seed=15),
        P(temperature=0.8, top_p=0.9, seed=16),
        P(temperature=1.5, top_k=5, seed=17),
    ]
    params = [ps[i % len(ps)] for i in range(rows)]
    params = [SamplingParams(**{**p.__dict__, "seed": p.seed + 100 * i if p.seed is not None else None})
              for i, p in enumerate(params)]
    first = [(37 * i + 5) % V for i in range(rows)]
    maxt = [10 + (i * 7) % 31 for i in range(rows)]
    eos = [((13 * i + 1) % V) if i % 3 else -1 for i in range(rows)]
    return params, first, maxt, eos


def _reference_loop(banks, params, first, maxt, eos, modes, L):
    """Per request: the loop's modes replayed with the oracle. Returns each
    row's generated tokens, per pushed token whether a sampling tie could
    have produced it, and each row's verification outcomes."""
    import oracle as O
    gens, ties, outcomes = [], [], []
    for r, p in enumerate(params):
        rec = p.record()
        greedy = p.temperature == 0.0
        state = None if greedy else O.xoshiro_from_seed(p.seed)
        gen, tie, out = [first[r]], [False], []
        done = first[r] == eos[r] or maxt[r] <= 1

        def draw(x, u=None):
            if greedy:
                return O.top_logit_candidates(x)[0][0], False
            res = O.sample(x, None, rec, u=u, rng_state=None if u is not None else state)
            return int(res.token), min(res.debug.cdf_margin, res.debug.topp_margin) < BOUNDARY_TOL

        def push(ts, flag):
            nonlocal done
            for t in ts:
                gen.append(int(t))
                tie.append(flag)
                if t == eos[r] or len(gen) >= maxt[r]:
                    done = True
                    return

        for mode in modes:
            if done:
                break
            if not mode:
                t, flag = draw(_host_target(banks, gen, r, eos))
                push([t], flag)
                continue
            d, D, flag = [], [], False
            t = gen[-1]
            for i in range(L):
                xd = _host_draft(banks, t, len(gen) - 1 + i, r, eos)
                t, f = draw(xd)
                d.append(t)
                D.append(xd)
                flag |= f
            T = np.stack([_host_target(banks, gen + d[:j], r, eos) for j in range(L + 1)])
            u = np.zeros(L + 1, np.float32) if greedy else \
                np.array([O.xoshiro_next_f32(state) for _ in range(L + 1)], np.float32)
            acc, tok, _ = O.mtp_verify(T[None], np.stack(D)[None], np.array([d], np.int64),
                                       np.array([rec], dtype=PARAMS_DTYPE), u[None])
            acc, tok = int(acc[0]), int(tok[0])
            if acc == L and not greedy:  # the bonus token is the sampler's draw from row L
                _, f = draw(T[L], u=float(u[L]))
                flag |= f
            out.append((acc, d, T))
            push(d[:acc] + [tok], flag)
        gens.append(gen)
        ties.append(tie)
        outcomes.append(out)
    return gens, ties, outcomes


def _compare(got, want, ties):
    tied = 0
    for r in range(len(want)):
        g, w = got[r], want[r]
        n = min(len(g), len(w))
        k = next((i for i in range(n) if g[i] != w[i]), None)
        if k is None:
            assert len(g) == len(w), (r, g, w)
        else:
            assert ties[r][k], (r, k, g, w)
            tied += 1
    return tied


@pytest.mark.parametrize("L,probe", [(1, 4), (3, 3)])
def test_mtp_loop_matches_the_reference_loop_and_rolls_the_cache_back(cuda_device, L, probe):
    import torch
    banks = _banks()
    params, first, maxt, eos = _requests()
    rows = len(params)
    model = DeviceModel(banks, eos, rows, max(maxt))
    loop = MtpDecodeLoop(params, first, V, maxt, draft_len=L, eos=eos, window=8, probe_every=probe)
    steps = loop.run(model.draft, model.target, model.rollback)
    torch.cuda.synchronize()
    assert loop.finished() and not loop.failed()
    assert True in loop.modes and False in loop.modes     # both kinds of step ran
    got = loop.generated()
    want, ties, outcomes = _reference_loop(banks, params, first, maxt, eos, loop.modes, L)
    assert _compare(got, want, ties) <= 1
    assert steps <= max(maxt)
    # the cache holds exactly the committed tokens but the newest
    kv, kvl = model.kv.cpu().numpy(), model.kv_len.cpu().numpy()
    for r in range(rows):
        assert kvl[r] == len(got[r]) - 1
        assert kv[r, :kvl[r]].tolist() == got[r][:-1]
    accepted = sum(a for o in outcomes for a, _, _ in o)
    assert accepted > 0 and loop.stats.accepted_tokens > 0


def test_mtp_statistics_follow_verify_pair(cuda_device):
    """draft_len 1 and greedy rows: each verification is one verify_pair of
    the target's argmax and the draft, recorded as MtpStatistics::record
    (mtp.rs:72-79, 98-104)."""
    import oracle as O
    import torch
    b1, b2 = _banks(6)
    banks = (b1, b2 * np.float32(16.0))   # a context term as large as the draft's: some drafts miss
    _, first, maxt, eos = _requests(12)
    params = [SamplingParams(temperature=0.0) for _ in first]
    model = DeviceModel(banks, eos, len(params), max(maxt))
    loop = MtpDecodeLoop(params, first, V, maxt, draft_len=1, eos=eos, window=4, probe_every=3)
    loop.run(model.draft, model.target, model.rollback)
    torch.cuda.synchronize()
    want, ties, outcomes = _reference_loop(banks, params, first, maxt, eos, loop.modes, 1)
    assert _compare(loop.generated(), want, ties) == 0
    ref = MtpStatistics()
    for out in outcomes:
        for acc, d, T in out:
            v = verify_pair(O.top_logit_candidates(T[0])[0][0], d[0])
            assert v.accepted == (acc == 1)
            ref.record(v.accepted, v.emitted_tokens, 1)
    assert loop.stats == ref
    assert 0.0 < ref.acceptance_rate() < 1.0


def test_controller_keeps_mtp_off_for_useless_drafts(cuda_device):
    """Drafts that the target never confirms (greedy rows whose draft head
    scores another row's bank) and a cheap target: every verification emits
    one token in more time than a plain step, the rolling net benefit is
    negative, the controller stays off, and only probes speculate."""
    import torch
    banks = _banks(7)
    _, first, maxt, eos = _requests(8)
    params = [SamplingParams(temperature=0.0) for _ in first]
    model = DeviceModel(banks, [-1] * len(params), len(params), 40)
    model.rows1_draft = model.b1[(model.r + 1) % NB]

    def bad_draft(tokens, positions):
        saved = model.rows1
        model.rows1 = model.rows1_draft
        try:
            return model.draft(tokens, positions)
        finally:
            model.rows1 = saved

    maxt = [40] * len(params)
    ctl = MtpController(4)
    loop = MtpDecodeLoop(params, first, V, maxt, draft_len=1, eos=None, controller=ctl, probe_every=8)
    loop.run(bad_draft, model.target, model.rollback, check_every=1)
    torch.cuda.synchronize()
    assert not ctl.enabled()
    assert loop.stats.acceptance_rate() < 0.2
    late = loop.modes[2:]
    assert sum(late) <= len(late) // 8 + 1, loop.modes


def test_controller_enables_mtp_for_good_drafts(cuda_device):
    """Drafts equal to the target's own next-token rows for greedy rows and
    a target whose cost hardly depends on the positions it scores: most
    verifications accept, the rolling net benefit is positive, the
    controller turns MTP on and the loop stays speculative."""
    import torch
    banks = _banks(8)
    banks = (banks[0], np.zeros_like(banks[1]))   # no context term: the draft is the target
    _, first, maxt, eos = _requests(8)
    params = [SamplingParams(temperature=0.0) for _ in first]
    maxt = [60] * len(params)
    model = DeviceModel(banks, [-1] * len(params), len(params), max(maxt), heavy=8192)
    ctl = MtpController(4)
    loop = MtpDecodeLoop(params, first, V, maxt, draft_len=1, eos=None, controller=ctl, probe_every=8)
    loop.run(model.draft, model.target, model.rollback, check_every=1)
    torch.cuda.synchronize()
    assert ctl.enabled()
    assert loop.stats.acceptance_rate() == 1.0
    assert loop.stats.emitted_tokens_per_target_pass() == 2.0
    assert loop.steps < 40


def test_mtp_loop_rejects_penalised_rows(cuda_device):
    with pytest.raises(ValueError):
        MtpDecodeLoop([SamplingParams(temperature=0.7, seed=1, repeat_penalty=1.2)], [1], V, 4)
