"""GPU parity of the general kernel (rows with top_k None / >= vocab / > 256)
against the oracle. These rows depend on the reference's sequential f32 sums
over the whole vocabulary; the kernel reproduces them, so tokens must match
exactly (counted CDF boundary ties aside) even for spread distributions where
the reference's own rounding decides the draw."""
import numpy as np
import pytest

from parity import compare, gpu_sample
from test_gpu_stream import _batch, _subset
from turboqwenfare_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _assert_ok(g):
    assert (g.status == 0).all(), g.status


def test_c2_full_vocabulary_rows(cuda_device):
    b = W.config("c2", rows=48, seed=6)
    keep = np.nonzero((b.params["top_k"] == 0) & (b.params["temperature"] > 0))[0]
    sub = _subset(b, keep)
    g = gpu_sample(sub, want_probs=True)
    _assert_ok(g)
    rep = compare(sub, g)
    print(rep)
    assert rep.identical + rep.boundary_ties == rep.rows
    assert rep.boundary_ties <= max(1, rep.rows // 10)


def test_spread_row_many_uniforms_matches_reference_rounding(cuda_device):
    """One spread row (T = 1, no top_p): the reference's sequential sums drop
    the tail; every uniform must still give the oracle's token."""
    rng = np.random.default_rng(12)
    V = 151_936
    row = (3.0 * rng.standard_normal(V)).astype(np.float32)
    n = 64
    x = np.repeat(row[None, :], n, axis=0)
    p = W.params_rows(n, 1.0)
    u = ((np.arange(n) + 0.5) / n).astype(np.float32)
    b = _batch(x, p, uniforms=u)
    g = gpu_sample(b)
    _assert_ok(g)
    rep = compare(b, g, check_probs=False)
    assert rep.identical + rep.boundary_ties == rep.rows
    assert rep.boundary_ties == 0


@pytest.mark.parametrize("vocab", [1, 2, 4, 33, 1000, 10_241])
def test_general_rows_small_vocab(cuda_device, vocab):
    rng = np.random.default_rng(vocab + 5)
    rows = 12
    x = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    ps = []
    for r in range(rows):
        k = [0, vocab, vocab + 5, 300, vocab - 1, 0][r % 6]
        T = [0.3, 1.0, 1.9, 0.7][r % 4]
        top_p = [1.0, 0.9, 0.5, 0.0][(r // 2) % 4]
        mp = [None, 0.05, 0.5][(r // 3) % 3]
        ps.append(W.params_rows(1, T, top_p=top_p, top_k=max(k, 0), min_p=mp)[0])
    b = _batch(x, np.array(ps), seed=vocab)
    g = gpu_sample(b, want_probs=True)
    _assert_ok(g)
    rep = compare(b, g)
    assert rep.identical + rep.boundary_ties == rep.rows


def test_general_special_values_and_penalties(cuda_device):
    rng = np.random.default_rng(3)
    V = 5000
    x = rng.standard_normal((6, V)).astype(np.float32)
    x[0, 7] = np.nan
    x[1, :] = np.nan
    x[2, :] = -np.inf
    x[2, 3] = 1.0
    x[3, 11] = np.inf
    x[4, :] = 2.0
    hl = [list(rng.integers(0, V, 100)), [], [3, 3, 3], [11], list(range(50)), list(rng.integers(0, 10, 500))]
    p = W.params_rows(6, 1.0, top_p=0.9)
    p["top_k"] = [0, 0, 0, 400, 0, 4999]
    p["repeat_penalty"] = [1.3, 1.0, 2.0, 1.1, 1.5, 0.9]
    p["frequency_penalty"] = [0.1, 0.0, 0.0, 0.2, 0.0, -0.5]
    p["repeat_last_n"] = [64, 64, 64, 64, 2**64 - 1, 300]
    b = _batch(x, p, hist_lists=hl)
    g = gpu_sample(b, want_probs=True)
    _assert_ok(g)
    rep = compare(b, g)
    assert rep.identical + rep.boundary_ties == rep.rows


def test_large_top_k_rows(cuda_device):
    b = W.config("c1", rows=6, seed=9)
    b.params["top_k"] = [257, 1000, 50_000, 151_935, 151_936, 10**6]
    g = gpu_sample(b, want_probs=True)
    _assert_ok(g)
    rep = compare(b, g)
    assert rep.identical + rep.boundary_ties == rep.rows


def test_prefix_sorted_rows_all_branches(cuda_device):
    """Full-vocabulary rows cut by top_p and/or min_p: the kernel sorts only a
    prefix of the (p desc, id asc) order (collected by min_p's floor, or by
    top_p's exponent bins) or falls back to the whole sort when that prefix
    is too large; every branch must give the oracle's tokens and kept
    probabilities."""
    rng = np.random.default_rng(77)
    V = 151_936
    cases = [  # (T, top_p, min_p)
        (0.5, 0.9, None),     # top_p alone, small prefix
        (1.5, 0.9, None),     # top_p alone, prefix above the shared-memory cap
        (1.0, 0.6, None),
        (1.0, 1.0, 0.05),     # min_p alone
        (1.5, 1.0, 0.001),    # min_p alone, floor prefix above the cap
        (0.8, 0.3, 0.1),      # top_p cuts before min_p
        (1.2, 0.95, 0.2),     # min_p cuts before top_p
        (1.0, 0.0, None),     # top_p 0 keeps one entry
        (1.0, 0.9, 1.5),      # min_p above 1 keeps one entry
        (0.2, 0.5, 0.05),     # peaked row
        (1.0, 0.999, None),
        (3.0, 0.5, None),     # very flat row
    ]
    n = len(cases)
    x = (3.0 * rng.standard_normal((n, V))).astype(np.float32)
    for r in range(n):
        x[r, rng.choice(V, size=2, replace=False)] += 8.0
    ps = [W.params_rows(1, T, top_p=tp, top_k=0, min_p=mp)[0] for T, tp, mp in cases]
    for dtype in ("f32", "bf16"):
        xb = x if dtype == "f32" else W.to_bf16_bits(x)
        b = _batch(xb, np.array(ps), seed=4, dtype=dtype)
        g = gpu_sample(b, want_probs=True)
        _assert_ok(g)
        rep = compare(b, g)
        print(dtype, rep)
        assert rep.identical + rep.boundary_ties == rep.rows


def test_mixed_batches_on_one_handle(cuda_device):
    """After a call with full-vocabulary rows, the handle's next call has its
    stream kernel count the general rows and leave one SM per general row to
    the general kernel. The same mixed batch twice on a fresh handle (the
    second call splits the SMs), then a batch with no general rows (counted,
    none found, no split), then the mixed batch again: every call's tokens
    equal the oracle's."""
    import torch

    import turboqwenfare_b200._native as N
    from parity import GpuResult, to_device_logits
    from turboqwenfare_b200 import sample_batch

    h = N.Handle(0)
    mixed = W.config("c2", rows=96, seed=11)
    assert ((mixed.params["top_k"] == 0) & (mixed.params["temperature"] > 0)).any()
    topk_only = W.config("c1", rows=64, seed=12)

    def run(b):
        lg = to_device_logits(b.logits, b.dtype)
        hist = torch.from_numpy(b.hist).cuda()
        off = torch.from_numpy(b.hist_off).cuda()
        u = torch.from_numpy(b.uniforms).cuda()
        res = sample_batch(lg, b.params, hist, off, uniforms=u, vocab=b.vocab, handle=h)
        torch.cuda.synchronize()
        g = GpuResult(res.tokens.cpu().numpy(), res.status.cpu().numpy())
        _assert_ok(g)
        rep = compare(b, g)
        print(rep)
        assert rep.identical + rep.boundary_ties == rep.rows
        assert rep.boundary_ties <= max(1, rep.rows // 10)

    for b in (mixed, mixed, topk_only, mixed):
        run(b)
