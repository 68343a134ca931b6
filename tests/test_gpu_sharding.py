"""Vocabulary-sharded sampling on the device.

One GPU emulates N ranks (export each vocabulary slice, stack the records as
the all-gather would, merge): tokens must equal tqfs_sample on the whole
rows, bit for bit, since both run the same exact top-k and draw. With two or
more GPUs the NCCL path runs for real, one process per GPU.
"""
import os
import socket

import numpy as np
import pytest

from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.sharding import shard_export, shard_merge, vocab_shards

pytestmark = pytest.mark.gpu


def _device_batch(b):
    import torch
    if b.dtype == "f32":
        lg = torch.from_numpy(b.logits).cuda()
    else:
        lg = torch.from_numpy(b.logits.view(np.int16)).cuda().view(torch.bfloat16)
    hist = torch.from_numpy(b.hist).cuda()
    off = torch.from_numpy(b.hist_off).cuda()
    uni = torch.from_numpy(b.uniforms).cuda()
    return lg, hist, off, uni


def _emulated(b, nranks):
    import torch
    lg, hist, off, uni = _device_batch(b)
    recs = []
    for o, n in vocab_shards(b.vocab, nranks):
        recs.append(shard_export(lg[:, o:o + n], b.params, o, b.vocab, history=hist, history_offsets=off))
    tokens, status = shard_merge(torch.stack(recs), b.params, b.vocab, uniforms=uni, history_offsets=off)
    torch.cuda.synchronize()
    return tokens.cpu().numpy(), status.cpu().numpy()


def _whole(b):
    from turboqwenfare_b200.sampler import sample_batch
    lg, hist, off, uni = _device_batch(b)
    r = sample_batch(lg, b.params, history=hist, history_offsets=off, uniforms=uni, vocab=b.vocab)
    return r.tokens.cpu().numpy(), r.status.cpu().numpy()


def _oracle_parity(b, tok, st):
    from parity import GpuResult, compare
    rep = compare(b, GpuResult(tok, st), check_probs=False)
    assert rep.identical + rep.boundary_ties == rep.rows, rep
    assert rep.boundary_ties <= max(1, rep.rows // 100), rep
    return rep


@pytest.mark.parametrize("nranks,rows", [(2, 128), (8, 128), (8, 1024)])
def test_configuration_4_emulated_shards_match_oracle(cuda_device, nranks, rows):
    """Configuration 4 split by vocabulary (records merged as the all-gather
    would deliver them): tokens equal the oracle's on the whole rows, and the
    unsharded call's."""
    b = W.config("c4", rows=rows, seed=11)
    tok, st = _emulated(b, nranks)
    assert (st == 0).all()
    print(nranks, rows, _oracle_parity(b, tok, st))
    wtok, wst = _whole(b)
    assert (wst == 0).all() and (tok == wtok).all()


def test_f32_rows_greedy_and_unsupported(cuda_device):
    b = W.config("c1", rows=16, seed=3, vocab=50_000)
    b.params["temperature"][[1, 5]] = 0.0          # greedy: shards' top-4
    b.params["top_k"][7] = 0                        # whole vocabulary: not shardable
    b.params["top_k"][9] = 128                      # the largest shardable k
    tok, st = _emulated(b, 3)
    wtok, wst = _whole(b)
    ok = np.ones(16, bool)
    ok[7] = False
    assert st[7] == 2 and tok[7] == -1
    assert (st[ok] == 0).all() and (tok[ok] == wtok[ok]).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from turboqwenfare_b200.sharding import NcclComm, sample_vocab_sharded
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    comm = None
    try:
        b = W.config("c4", rows=64, seed=5)
        lg, hist, off, uni = _device_batch(b)
        comm = NcclComm(rank, world, rank)
        o, n = vocab_shards(b.vocab, world)[rank]
        tok, st = sample_vocab_sharded(comm, lg[:, o:o + n].contiguous(), b.params, o, b.vocab, uniforms=uni,
                                       history=hist, history_offsets=off)
        torch.cuda.synchronize()
        q.put((rank, tok.cpu().numpy(), st.cpu().numpy()))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_nccl_two_gpus(cuda_device):
    import multiprocessing as mp
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (t, s)) for r, t, s in (q.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    b = W.config("c4", rows=64, seed=5)
    wtok, _ = _whole(b)
    for r in range(world):
        assert (res[r][1] == 0).all() and (res[r][0] == wtok).all()
    _oracle_parity(b, res[0][0], res[0][1])
