"""GPU-vs-oracle comparison helpers for the `gpu` tests.

A token mismatch is accepted only as a floating-point CDF boundary tie: the
oracle's own decision margin (distance of u*total to the CDF bound of the
drawn entry, or of the top_p cumulative to top_p) is below BOUNDARY_TOL
relative. Such rows are counted and reported; any other mismatch fails.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

BOUNDARY_TOL = 1e-5   # relative CDF margin below which a mismatch is a tie
PROB_RTOL = 1e-5      # post-filter probabilities
PROB_ATOL = 1e-12


def to_device_logits(logits: np.ndarray, dtype: str, ld: int | None = None):
    import torch
    rows, vocab = logits.shape
    ld = ld or vocab
    if ld != vocab:
        pad = np.zeros((rows, ld), logits.dtype)
        pad[:, :vocab] = logits
        logits = pad
    if dtype == "f32":
        return torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    return torch.from_numpy(np.ascontiguousarray(logits).view(np.int16)).cuda().view(torch.bfloat16)


@dataclass
class GpuResult:
    tokens: np.ndarray
    status: np.ndarray
    probs: np.ndarray | None = None
    top4_tokens: np.ndarray | None = None
    top4_logits: np.ndarray | None = None
    rng_state: np.ndarray | None = None


def gpu_sample(batch, use_uniforms=True, rng_state=None, want_probs=False, want_top4=False,
               ld=None) -> GpuResult:
    import torch
    from turboqwenfare_b200 import sample_batch
    lg = to_device_logits(batch.logits, batch.dtype, ld)
    hist = torch.from_numpy(batch.hist if batch.hist.size else np.zeros(1, np.int32)).cuda()
    off = torch.from_numpy(batch.hist_off).cuda()
    u = torch.from_numpy(batch.uniforms).cuda() if use_uniforms else None
    st = None
    if not use_uniforms:
        st = torch.from_numpy(np.ascontiguousarray(rng_state).view(np.int64)).cuda()
    res = sample_batch(lg, batch.params, hist, off, uniforms=u, rng_state=st, vocab=batch.vocab,
                       want_top4=want_top4, want_probs=want_probs)
    torch.cuda.synchronize()
    out = GpuResult(res.tokens.cpu().numpy(), res.status.cpu().numpy())
    if want_probs:
        out.probs = res.probs.cpu().numpy()[:, : batch.vocab]
    if want_top4:
        t4 = res.top4.cpu().numpy()
        out.top4_tokens = t4[..., 0].view(np.uint32)
        out.top4_logits = t4[..., 1].copy().view(np.float32)
    if st is not None:
        out.rng_state = st.cpu().numpy().view(np.uint64)
    return out


@dataclass
class Report:
    rows: int = 0
    identical: int = 0
    boundary_ties: int = 0
    prob_rows_checked: int = 0
    details: list = field(default_factory=list)

    def __str__(self):
        return (f"rows={self.rows} identical={self.identical} boundary_ties={self.boundary_ties} "
                f"prob_rows={self.prob_rows_checked}")


def row_history(batch, r):
    return batch.hist[batch.hist_off[r]: batch.hist_off[r + 1]].astype(np.int64).astype(np.uint32)


def compare(batch, gpu: GpuResult, check_probs=True, rows=None) -> Report:
    import oracle as O
    rep = Report()
    lf = batch.logits_f32()
    want = O.sample_batch(batch.logits, batch.params, batch.hist, batch.hist_off, batch.uniforms,
                          vocab=batch.vocab)
    for r in (range(batch.rows) if rows is None else rows):
        rep.rows += 1
        greedy = float(batch.params[r]["temperature"]) == 0.0
        if gpu.tokens[r] == want[r]:
            rep.identical += 1
        if greedy:
            assert gpu.tokens[r] == want[r], f"row {r}: greedy token {gpu.tokens[r]} != {want[r]}"
            continue
        need_detail = gpu.tokens[r] != want[r] or (check_probs and gpu.probs is not None)
        if not need_detail:
            continue
        res = O.sample(lf[r], row_history(batch, r), batch.params[r], u=float(batch.uniforms[r]),
                       dense=check_probs and gpu.probs is not None)
        assert res.token == want[r]
        if gpu.tokens[r] != want[r]:
            tie = res.debug.cdf_margin < BOUNDARY_TOL or res.debug.topp_margin < BOUNDARY_TOL
            assert tie, (f"row {r}: token {gpu.tokens[r]} != oracle {want[r]} with margins "
                         f"cdf={res.debug.cdf_margin:.3g} top_p={res.debug.topp_margin:.3g}")
            rep.boundary_ties += 1
            rep.details.append((r, int(gpu.tokens[r]), int(want[r])))
            continue
        if check_probs and gpu.probs is not None:
            g, o = gpu.probs[r], res.probs
            assert np.array_equal(np.nonzero(g)[0], np.nonzero(o)[0]), f"row {r}: kept sets differ"
            np.testing.assert_allclose(g, o, rtol=PROB_RTOL, atol=PROB_ATOL, err_msg=f"row {r}")
            rep.prob_rows_checked += 1
    return rep
