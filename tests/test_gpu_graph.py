"""tqfs_sample captured once in a CUDA graph and replayed on new inputs.

A decode loop that captures its step replays the same kernel arguments every
step, so every piece of per-call state must be reset on the device in stream
order. The stream kernel shares each row's best k-th bound between the row's
units through one word per row; the finalize kernel clears that word after
reading it. Replays whose logits sit far below the previous replay's (a stale
bound from the earlier replay would drop the true top-k) must still match
the oracle on their own inputs."""
import numpy as np
import pytest

from parity import compare, GpuResult
from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.sampler import params_tensor, sample_batch

pytestmark = pytest.mark.gpu


def test_replayed_graph_matches_oracle_on_each_input(cuda_device):
    import torch
    import turboqwenfare_b200._native as N
    first = W.config("c1", rows=64, seed=51)
    shifts = [0.0, -40.0, 25.0, -80.0]
    batches = []
    for i, sh in enumerate(shifts):
        b = W.config("c1", rows=64, seed=60 + i)
        b.logits = (b.logits + np.float32(sh)).astype(np.float32)
        batches.append(b)
    dev = torch.device("cuda", 0)
    h = N.Handle(0)   # its own handle: scratch sized by the warm-up, never grown while captured
    lg = torch.from_numpy(first.logits).to(dev)
    hist = torch.from_numpy(first.hist).to(dev)
    off = torch.from_numpy(first.hist_off).to(dev)
    par = params_tensor(first.params, first.rows, dev)
    uni = torch.from_numpy(first.uniforms).to(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        sample_batch(lg, par, hist, off, uniforms=uni, vocab=first.vocab, handle=h)   # warm-up
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="relaxed"):
        res = sample_batch(lg, par, hist, off, uniforms=uni, vocab=first.vocab, handle=h)
    for b in batches:
        lg.copy_(torch.from_numpy(b.logits))
        hist.copy_(torch.from_numpy(b.hist))
        uni.copy_(torch.from_numpy(b.uniforms))
        graph.replay()
        torch.cuda.synchronize()
        g = GpuResult(res.tokens.cpu().numpy(), res.status.cpu().numpy())
        assert (g.status == 0).all(), g.status
        rep = compare(b, g, check_probs=False)
        assert rep.identical + rep.boundary_ties == rep.rows, rep
    del graph
    h.close()
