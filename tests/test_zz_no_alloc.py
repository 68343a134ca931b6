"""tqfs_sample_static: the sampler for callers that cannot allocate GPU memory
(hosts whose GPU memory is reserved by their own pool, and decode loops that
must not synchronise on cudaMalloc/cudaFree). It runs the stream kernel on a
fixed static scratch array; its tokens must equal tqfs_sample's on the same
inputs, call after call, since every call reuses the same array.

Named to be collected last; it passes alone in a fresh process and after the
other tests."""
import ctypes

import numpy as np
import pytest

import turboqwenfare_b200._native as N
from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.sampler import params_tensor

pytestmark = pytest.mark.gpu


def _device_batch(b):
    import torch
    dev = torch.device("cuda", 0)
    if b.dtype == "f32":
        lg = torch.from_numpy(b.logits).to(dev)
    else:
        lg = torch.from_numpy(b.logits.view(np.int16)).to(dev).view(torch.bfloat16)
    hist = torch.from_numpy(b.hist if b.hist.size else np.zeros(1, np.int32)).to(dev)
    off = torch.from_numpy(b.hist_off).to(dev)
    par = params_tensor(b.params, b.rows, dev)
    uni = torch.from_numpy(b.uniforms).to(dev)
    return lg, hist, off, par, uni


def _run_both(b):
    import torch
    lg, hist, off, par, uni = _device_batch(b)
    dt = N.DTYPE_F32 if b.dtype == "f32" else N.DTYPE_BF16
    rows, v = b.rows, b.vocab
    tok_a = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    st_a = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    tok_b = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    st_b = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    h = N.default_handle(0)
    h.check(N.lib().tqfs_sample(h.ptr, lg.data_ptr(), dt, rows, v, v, hist.data_ptr(), off.data_ptr(),
                                par.data_ptr(), uni.data_ptr(), None, tok_a.data_ptr(), None, None,
                                st_a.data_ptr(), stream))
    rc = N.lib().tqfs_sample_static(lg.data_ptr(), dt, rows, v, v, hist.data_ptr(), off.data_ptr(),
                                    par.data_ptr(), uni.data_ptr(), None, tok_b.data_ptr(), st_b.data_ptr(),
                                    stream)
    assert rc == N.OK, rc
    torch.cuda.synchronize()
    return tok_a.cpu().numpy(), st_a.cpu().numpy(), tok_b.cpu().numpy(), st_b.cpu().numpy()


def test_static_scratch_matches_the_allocating_entry_point_on_consecutive_calls(cuda_device):
    first = W.config("c1", rows=24, seed=31)
    first.params["temperature"][::5] = 0.0          # greedy rows too
    second = W.config("c4", rows=40, seed=32)        # different shape, dtype and rows
    for b in (first, second, first):
        tok_a, st_a, tok_b, st_b = _run_both(b)
        assert (st_a == 0).all() and (st_b == 0).all(), (st_a, st_b)
        np.testing.assert_array_equal(tok_b, tok_a)


def test_rows_outside_the_stream_kernel_report_unsupported(cuda_device):
    b = W.config("c1", rows=6, seed=33, vocab=20_000)
    b.params["top_k"][1] = 0        # full-vocabulary row: not this kernel's
    b.params["top_k"][4] = 1000     # top_k above 128: not this kernel's
    import torch
    lg, hist, off, par, uni = _device_batch(b)
    tok = torch.empty(6, dtype=torch.int32, device="cuda")
    st = torch.empty(6, dtype=torch.int32, device="cuda")
    rc = N.lib().tqfs_sample_static(lg.data_ptr(), N.DTYPE_F32, 6, b.vocab, b.vocab, hist.data_ptr(),
                                    off.data_ptr(), par.data_ptr(), uni.data_ptr(), None, tok.data_ptr(),
                                    st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == N.OK
    torch.cuda.synchronize()
    s = st.cpu().numpy()
    t = tok.cpu().numpy()
    assert s[1] == N.ROW_ERR_UNSUPPORTED and s[4] == N.ROW_ERR_UNSUPPORTED and t[1] == -1 and t[4] == -1
    assert (s[[0, 2, 3, 5]] == 0).all()


def test_batches_beyond_the_fixed_scratch_are_rejected_without_a_launch(cuda_device):
    import torch
    x = torch.zeros(1, dtype=torch.float32, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    # 2,000 rows at vocab 151,936 need about 72 MiB of scratch > 48 MiB.
    rc = N.lib().tqfs_sample_static(x.data_ptr(), N.DTYPE_F32, 2000, 151_936, 151_936, None, None,
                                    x.data_ptr(), x.data_ptr(), None, out.data_ptr(), out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == N.ERR_UNSUPPORTED
