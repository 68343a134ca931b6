"""Device MTP verify (tqfs_mtp_verify) against the oracle's orc_mtp_verify.

Decisions, accepted counts and tokens must be identical. The only allowed
difference is a decision whose oracle margin |u*q_draft - q_target| is below
1e-5 relative at a position both sides reach (the kernels' exponential is
correctly rounded; glibc's expf differs from it by one ulp in about 9 of
100,000 arguments), counted and asserted to be rare.
"""
import numpy as np
import pytest

from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.params import HAS_MIN_P

pytestmark = pytest.mark.gpu

MARGIN = 1e-5


def _run_device(b, dtype="f32"):
    import torch
    from turboqwenfare_b200.mtp import verify_batch
    if dtype == "f32":
        t = torch.from_numpy(b.target).cuda()
        d = torch.from_numpy(b.draft).cuda()
    else:
        t = torch.from_numpy(W.to_bf16_bits(b.target).view(np.int16)).cuda().view(torch.bfloat16)
        d = torch.from_numpy(W.to_bf16_bits(b.draft).view(np.int16)).cuda().view(torch.bfloat16)
    r = verify_batch(t, d, torch.from_numpy(b.drafts).cuda(), b.params, torch.from_numpy(b.uniforms).cuda())
    torch.cuda.synchronize()
    return (r.accepted.cpu().numpy(), r.token.cpu().numpy(), r.mask.cpu().numpy(), r.status.cpu().numpy())


def _widened(b, dtype):
    if dtype == "f32":
        return b.target, b.draft
    bf = lambda x: (W.to_bf16_bits(x).astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    return bf(b.target), bf(b.draft)


def _compare(b, dtype="f32"):
    import oracle as O
    acc, tok, mask, status = _run_device(b, dtype)
    tgt, dft = _widened(b, dtype)
    oacc, otok, omask = O.mtp_verify(tgt, dft, b.drafts.astype(np.uint32), b.params, b.uniforms)
    assert (status == 0).all()
    boundary = 0
    for s in range(b.seqs):
        if acc[s] == oacc[s] and tok[s] == otok[s] and (mask[s] == omask[s]).all():
            continue
        # a mismatch is tolerated only at a decision on the knife's edge
        p = b.params[s]
        edge = False
        for j in range(b.draft_len):
            if mask[s, j] != omask[s, j]:
                x = int(b.drafts[s, j])
                qt = O.filtered_distribution(tgt[s, j], p)[x]
                qd = O.filtered_distribution(dft[s, j], p)[x]
                lhs = np.float32(b.uniforms[s, j]) * np.float32(qd)
                edge = abs(float(lhs) - float(qt)) <= MARGIN * max(float(qt), 1e-30)
                break
        assert edge, f"seq {s}: device ({acc[s]}, {tok[s]}, {mask[s]}) vs oracle ({oacc[s]}, {otok[s]}, {omask[s]})"
        boundary += 1
    assert boundary <= max(1, b.seqs // 32)
    return acc, oacc


def _params(n, temps, top_k=0, top_p=0.9, min_p=None):
    p = W.params_rows(n, 0.8, top_p=top_p, top_k=top_k)
    p["temperature"] = np.asarray(temps, np.float32)
    if min_p is not None:
        p["min_p"] = min_p
        p["flags"] = HAS_MIN_P
    return p


def test_small_vocab_mixed_rows(cuda_device):
    b = W.mtp_config(seqs=12, draft_len=3, vocab=3000, seed=5)
    b.params = _params(12, [0.8, 0.0, 1.2, 0.8, 0.5, 0.0, 1.0, 0.8, 0.3, 1.5, 0.8, 0.0], top_k=0)
    b.params["top_k"][[2, 6]] = [20, 100]
    b.params["min_p"][[3, 7]] = [0.05, 0.1]
    b.params["flags"][[3, 7]] = HAS_MIN_P
    b.params["top_p"][[4, 9]] = [1.0, 0.5]
    acc, oacc = _compare(b)
    assert len(set(acc.tolist())) > 1  # both acceptances and rejections occur


def test_greedy_sequences_follow_verify_pair(cuda_device):
    b = W.mtp_config(seqs=6, draft_len=3, vocab=2048, seed=9)
    b.params["temperature"] = 0.0
    b.drafts[:3] = np.argmax(b.target[:3, :3], axis=-1)  # all accepted: bonus from row L
    acc, tok, mask, status = _run_device(b)
    assert (acc[:3] == 3).all() and (tok[:3] == np.argmax(b.target[:3, 3], axis=-1)).all()
    _compare(b)


def test_bf16_rows(cuda_device):
    b = W.mtp_config(seqs=8, draft_len=2, vocab=4096, seed=13)
    _compare(b, "bf16")


def test_active_penalties_are_refused_per_sequence(cuda_device):
    b = W.mtp_config(seqs=3, draft_len=2, vocab=1000, seed=2)
    b.params["repeat_penalty"][1] = 1.1
    acc, tok, mask, status = _run_device(b)
    assert status[1] == 2 and acc[1] == -1 and tok[1] == -1
    assert status[0] == 0 and status[2] == 0


def test_configuration_3_full_vocabulary(cuda_device):
    """32 sequences x (3 drafts + bonus), V = 151,936, T = 0.8, top_p = 0.9."""
    b = W.mtp_config(seqs=32, draft_len=3, seed=2026)
    _compare(b)
