"""The LM head on the tensor cores (tqfs_lm_head_logits): logits = hidden .
weight^T with bf16 operands and f32 accumulation, against an fp64 product
of the same bf16 values. The tensor cores sum in their own order, so the
bound is relative to the sum of |products| (the f32 rounding of a K-term
sum), written in the test."""
import numpy as np
import pytest

import turboqwenfare_b200._native as N

pytestmark = pytest.mark.gpu


def _run(rows, hidden, vocab, seed, ld=None):
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(rows, hidden, generator=g) * 0.5).to(torch.bfloat16).cuda()
    w = (torch.randn(vocab, hidden, generator=g) * 0.05).to(torch.bfloat16).cuda()
    ld = ld or ((vocab + 3) // 4 * 4)
    out = torch.full((rows, ld), float("nan"), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = N.lib().tqfs_lm_head_logits(x.data_ptr(), w.data_ptr(), rows, hidden, vocab, hidden, hidden,
                                     out.data_ptr(), ld, err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == N.OK, st
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = x.double() @ w.double().T
    mag = x.double().abs() @ w.double().abs().T
    return out[:, :vocab].double(), ref, mag, out


@pytest.mark.parametrize("rows,hidden,vocab", [(128, 2048, 4096), (1, 64, 256), (37, 128, 1000),
                                               (256, 2048, 151_936), (300, 1024, 8192)])
def test_lm_head_logits_match_fp64(cuda_device, rows, hidden, vocab):
    got, ref, mag, out = _run(rows, hidden, vocab, seed=rows + vocab)
    tol = hidden * 2.0 ** -24 * mag + 1e-6   # f32 accumulation of `hidden` products, any order
    bad = (got - ref).abs() > tol
    assert not bad.any(), (bad.sum().item(), (got - ref).abs().max().item())
    if out.shape[1] > vocab:  # padding columns are not written
        assert out[:, vocab:].isnan().all()


def _fused_case(rows, hidden, vocab, seed, hlen=1024, with_hist=True):
    """Hidden states, LM head, c1-style parameters (with some greedy rows and
    rows the fused path does not serve), histories and uniforms."""
    import torch
    from turboqwenfare_b200 import workloads as W
    rng = np.random.default_rng(seed)
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(rows, hidden, generator=g) * 0.5).to(torch.bfloat16).cuda()
    w = (torch.randn(vocab, hidden, generator=g) * 0.05).to(torch.bfloat16).cuda()
    p = W.params_rows(rows, 0.6, top_p=0.95, top_k=20, repeat_penalty=1.1, repeat_last_n=1024,
                      presence_penalty=0.5, frequency_penalty=0.3)
    p["temperature"][::9] = 0.0               # greedy rows
    p["top_k"][5::11] = 32                    # the largest served top_k
    p["top_k"][7::13] = 1
    p["top_k"][3::17] = 50                    # not served: tqfs_sample's stream path owns it
    p["top_p"][2::5] = 1.0
    lens = [hlen] * rows if with_hist else [0] * rows
    # histories biased toward ids near the head of the logits, so penalties bite
    hist = np.concatenate([rng.integers(0, vocab, n).astype(np.int32) for n in lens]) if with_hist else \
        np.zeros(0, np.int32)
    off = np.zeros(rows + 1, np.int64)
    off[1:] = np.cumsum(lens)
    u = W.philox_uniforms(seed + 7, rows)
    return x, w, p, hist, off, u


@pytest.mark.parametrize("rows,hidden,vocab,with_hist", [(64, 2048, 151_936, True), (256, 2048, 151_936, True),
                                                         (37, 1024, 20_000, False), (130, 512, 50_000, True)])
def test_fused_lm_head_sampling_matches_the_oracle_on_its_logits(cuda_device, rows, hidden, vocab, with_hist):
    """The fused path's tokens equal the oracle's on the logits the same
    GEMM produces (tqfs_lm_head_logits): same MMAs, so the same f32 values;
    everything after them is exact."""
    import torch
    from parity import GpuResult, compare
    from turboqwenfare_b200 import workloads as W
    x, w, p, hist, off, u = _fused_case(rows, hidden, vocab, seed=rows + hidden, with_hist=with_hist)
    s = torch.cuda.current_stream().cuda_stream
    logits = torch.empty((rows, vocab + (-vocab) % 4), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert N.lib().tqfs_lm_head_logits(x.data_ptr(), w.data_ptr(), rows, hidden, vocab, hidden, hidden,
                                       logits.data_ptr(), logits.shape[1], err.data_ptr(), s) == N.OK
    h = N.default_handle(0)
    par = torch.from_numpy(p.view(np.uint8).copy()).cuda()
    hd = torch.from_numpy(hist if hist.size else np.zeros(1, np.int32)).cuda()
    od = torch.from_numpy(off).cuda()
    ud = torch.from_numpy(u).cuda()
    tok = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    st = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    h.check(N.lib().tqfs_lm_head_sample(h.ptr, x.data_ptr(), w.data_ptr(), rows, hidden, vocab, hidden, hidden,
                                        hd.data_ptr(), od.data_ptr() if with_hist else None, par.data_ptr(),
                                        ud.data_ptr(), None, tok.data_ptr(), st.data_ptr(), s))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    tok, st = tok.cpu().numpy(), st.cpu().numpy()
    served = (p["temperature"] == 0) | ((p["top_k"] >= 1) & (p["top_k"] <= 32))
    assert (st[~served] == N.ROW_ERR_UNSUPPORTED).all() and (tok[~served] == -1).all()
    assert (st[served] == N.ROW_OK).all(), st
    lg = logits[:, :vocab].cpu().numpy()
    b = W.Batch("lmhead", lg, p, hist, off if with_hist else np.zeros(rows + 1, np.int64), u, "f32")
    rows_served = np.nonzero(served)[0]
    rep = compare(b, GpuResult(tok, st), check_probs=False, rows=rows_served)
    print(rep)
    assert rep.identical + rep.boundary_ties == rep.rows
    assert rep.boundary_ties <= max(1, rep.rows // 20)


def test_fused_lm_head_rejects_bad_operands(cuda_device):
    import torch
    h = N.default_handle(0)
    x = torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")
    par = torch.zeros(40 * 4, dtype=torch.uint8, device="cuda")
    tok = torch.zeros(4, dtype=torch.int32, device="cuda")
    u = torch.zeros(4, dtype=torch.float32, device="cuda")
    # hidden not a multiple of 64
    assert N.lib().tqfs_lm_head_sample(h.ptr, x.data_ptr(), x.data_ptr(), 4, 100, 4, 100, 100, None, None,
                                       par.data_ptr(), u.data_ptr(), None, tok.data_ptr(), None,
                                       torch.cuda.current_stream().cuda_stream) == N.ERR_INVALID_ARG
