"""Partitioning helpers and the vocabulary-sharding scheme, on CPU.

The scheme's claim: per-shard exact top-k (after penalties, global ids),
all-gathered, contain the row's top-k, so sampling from their union gives the
unsharded sampler's token. Checked here with the oracle on two gloo ranks.
"""
import os
import socket

import numpy as np
import pytest

from turboqwenfare_b200 import workloads as W
from turboqwenfare_b200.sharding import row_shard, vocab_shards


@pytest.mark.parametrize("vocab,n", [(151_936, 8), (1000, 3), (5, 8), (7, 1)])
def test_vocab_shards_cover_the_vocabulary(vocab, n):
    s = vocab_shards(vocab, n)
    assert len(s) == n and s[0][0] == 0
    for (o0, n0), (o1, _) in zip(s, s[1:]):
        assert o1 == o0 + n0
    assert s[-1][0] + s[-1][1] == vocab
    assert max(x[1] for x in s) - min(x[1] for x in s) <= 1


def test_configuration_4_slices_are_18992_ids():
    assert all(n == 18_992 for _, n in vocab_shards(151_936, 8))


def test_row_shards_partition_the_rows():
    rows = [row_shard(1024, 8, r) for r in range(8)]
    assert sum(n for _, n in rows) == 1024 and rows[3] == (384, 128)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_candidates(b, rank, world):
    """This rank's exact top-k keys per row: (global id, penalised value)."""
    import oracle as O
    off, n = vocab_shards(b.vocab, world)[rank]
    logits = (b.logits.astype(np.uint32) << 16).view(np.float32)  # bf16 widened exactly
    out = []
    for r in range(b.rows):
        h = b.hist[b.hist_off[r]:b.hist_off[r + 1]].astype(np.int64) - off
        v = O.apply_penalties(logits[r, off:off + n], h.astype(np.int32), b.params[r])
        k = int(b.params["top_k"][r])
        order = np.lexsort((np.arange(n), -v))[:k]  # value desc, id asc (no NaN here)
        out.append([(int(i) + off, float(v[i])) for i in order])
    return out


def _worker(rank, world, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        b = W.config("c4", rows=6, vocab=4000, seed=7)
        mine = _shard_candidates(b, rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        if rank == 0:
            q.put(gathered)
    finally:
        dist.destroy_process_group()


def test_union_of_shard_top_k_reproduces_the_unsharded_draw():
    import multiprocessing as mp
    import oracle as O
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = W.config("c4", rows=6, vocab=4000, seed=7)
    logits = (b.logits.astype(np.uint32) << 16).view(np.float32)
    neutral = b.params.copy()
    neutral["repeat_penalty"] = 1.0
    neutral["frequency_penalty"] = 0.0
    neutral["presence_penalty"] = 0.0
    for r in range(b.rows):
        merged = np.full(b.vocab, -np.inf, np.float32)
        for shard in gathered:
            for tok, val in shard[r]:
                merged[tok] = val
        h = b.hist[b.hist_off[r]:b.hist_off[r + 1]]
        whole = O.sample(logits[r], h, b.params[r], u=b.uniforms[r]).token
        union = O.sample(merged, np.zeros(0, np.int32), neutral[r], u=b.uniforms[r]).token
        assert whole == union, (r, whole, union)
