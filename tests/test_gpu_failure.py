"""Failure detection on the device without a GPU fault.

Every copy wait of the stream kernel is bounded. The test hook
`tqfs_debug_stall_row` arms one row's bulk copies on their barriers without
issuing them, so the waits for that row run out (a flag nothing sets, as the
bounded-wait design intends); nothing is in flight, so no write can land
after the kernel returns. The call must complete, the stalled row must
report TQFS_ROW_ERR_TIMEOUT with token -1, every other row must either be
correct or report the timeout, and the next call on the same handle must be
fully correct (no failure mark or bound left behind)."""
import numpy as np
import pytest

import turboqwenfare_b200._native as N
from parity import compare, gpu_sample
from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.sampler import sample_batch
from turboqwenfare_b200.sharding import shard_export, shard_merge, vocab_shards

pytestmark = pytest.mark.gpu

WAIT_NS = 200_000  # 0.2 ms per bounded wait in these calls


def _device(b):
    import torch
    lg = torch.from_numpy(b.logits).cuda() if b.dtype == "f32" else \
        torch.from_numpy(b.logits.view(np.int16)).cuda().view(torch.bfloat16)
    return (lg, torch.from_numpy(b.hist).cuda(), torch.from_numpy(b.hist_off).cuda(),
            torch.from_numpy(b.uniforms).cuda())


@pytest.mark.parametrize("name,rows,stalled", [("c1", 16, 5), ("c1x256", 256, 200)])
def test_stalled_row_reports_timeout_and_the_next_call_is_clean(cuda_device, name, rows, stalled):
    import oracle as O
    import torch
    b = W.config(name, rows=rows, seed=41)
    b.params["temperature"][::7] = 0.0   # greedy rows share the path
    lg, hist, off, uni = _device(b)
    h = N.default_handle(0)
    want = O.sample_batch(b.logits, b.params, b.hist, b.hist_off, b.uniforms)

    h.check(N.lib().tqfs_debug_stall_row(h.ptr, stalled, WAIT_NS))
    r = sample_batch(lg, b.params, hist, off, uniforms=uni, vocab=b.vocab, handle=h)
    torch.cuda.synchronize()
    tok, st = r.tokens.cpu().numpy(), r.status.cpu().numpy()
    assert st[stalled] == N.ROW_ERR_TIMEOUT and tok[stalled] == -1
    ok = st == N.ROW_OK
    assert ((st == N.ROW_OK) | (st == N.ROW_ERR_TIMEOUT)).all(), st
    assert (tok[~ok] == -1).all()
    assert ok.sum() >= rows // 2, f"only {ok.sum()} of {rows} rows survived one stalled row"
    assert (tok[ok] == want[ok]).all()

    g = gpu_sample(b)          # the same handle, no hook: every row exact again
    assert (g.status == 0).all(), g.status
    rep = compare(b, g, check_probs=False)
    assert rep.identical + rep.boundary_ties == rep.rows


def test_stalled_shard_marks_the_merged_row(cuda_device):
    import torch
    b = W.config("c4", rows=32, seed=43)
    lg, hist, off, uni = _device(b)
    h = N.default_handle(0)
    recs = []
    for i, (o, n) in enumerate(vocab_shards(b.vocab, 2)):
        if i == 1:
            h.check(N.lib().tqfs_debug_stall_row(h.ptr, 9, WAIT_NS))
        recs.append(shard_export(lg[:, o:o + n], b.params, o, b.vocab, history=hist, history_offsets=off))
    tok, st = shard_merge(torch.stack(recs), b.params, b.vocab, uniforms=uni, history_offsets=off)
    torch.cuda.synchronize()
    tok, st = tok.cpu().numpy(), st.cpu().numpy()
    assert st[9] == N.ROW_ERR_TIMEOUT and tok[9] == -1
    assert ((st == N.ROW_OK) | (st == N.ROW_ERR_TIMEOUT)).all()


def test_stall_hook_rejects_bad_arguments(cuda_device):
    h = N.default_handle(0)
    assert N.lib().tqfs_debug_stall_row(h.ptr, -1, WAIT_NS) == N.ERR_INVALID_ARG
    assert N.lib().tqfs_debug_stall_row(h.ptr, 0, 0) == N.ERR_INVALID_ARG


def test_nccl_rank_that_never_joins_times_out(cuda_device):
    """Host-side failure: a 2-rank communicator whose second rank never joins.
    Rank 0's init must give up within its deadline with TQFS_ERR_TIMEOUT
    (the communicator is aborted) instead of hanging."""
    import ctypes
    import time
    h = N.Handle(0)
    uid = (ctypes.c_uint8 * 128)()
    st = N.lib().tqfs_nccl_unique_id(ctypes.addressof(uid))
    if st != N.OK:
        pytest.skip("NCCL not available")
    comm = ctypes.c_void_p()
    t0 = time.monotonic()
    st = N.lib().tqfs_nccl_comm_init_timeout(h.ptr, 2, 0, ctypes.addressof(uid), 2000, ctypes.byref(comm))
    dt = time.monotonic() - t0
    assert st == N.ERR_TIMEOUT, (st, N.lib().tqfs_last_error(h.ptr))
    assert not comm.value
    assert dt < 30.0, dt
    assert b"aborted" in N.lib().tqfs_last_error(h.ptr)
    h.close()
