"""Multi-GPU partitioning of the sampling batch.

Row sharding (configurations 1-3 and the row variants of 4): each rank owns a
contiguous block of rows and samples them on its own GPU; no collective.

Vocabulary sharding (configuration 4): rank r owns ids [offset_r, offset_r +
len_r) of every row. `sample_vocab_sharded` runs tqfs_sample_vocab_sharded:
each rank exports its exact per-row top-k (global ids), one NCCL all-gather
collects the records over NVLink, and every rank merges them and draws, so all
ranks return the same tokens (include/tqfs.h documents the contract).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

from . import _native as N


def vocab_shards(vocab: int, nranks: int) -> List[Tuple[int, int]]:
    """Contiguous (offset, length) slices covering [0, vocab); the first
    vocab % nranks slices are one id longer."""
    if nranks <= 0:
        raise ValueError("nranks must be positive")
    base, extra = divmod(vocab, nranks)
    out, off = [], 0
    for r in range(nranks):
        n = base + (1 if r < extra else 0)
        out.append((off, n))
        off += n
    return out


def row_shard(rows: int, nranks: int, rank: int) -> Tuple[int, int]:
    """(first row, row count) of `rank` for row sharding."""
    return vocab_shards(rows, nranks)[rank]


def record_words() -> int:
    return int(N.lib().tqfs_shard_record_words())


def shard_export(logits, params, vocab_offset: int, vocab_total: int, history=None,
                 history_offsets=None, handle=None, records=None):
    """This rank's per-row records from its logits slice: a (rows, len) view
    whose row stride is its first stride (a column slice of the full rows)."""
    import torch
    from .sampler import params_tensor, _ptr, _stream

    rows, vocab_local = logits.shape
    ld = logits.stride(0)
    dev = logits.device
    h = handle or N.default_handle(dev.index or 0)
    dtype = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}[logits.dtype]
    if not (isinstance(params, torch.Tensor) and params.dtype == torch.uint8):
        params = params_tensor(params, rows, dev)
    if records is None:
        records = torch.empty((rows, record_words()), dtype=torch.int64, device=dev)
    h.check(N.lib().tqfs_shard_export(h.ptr, _ptr(logits), dtype, rows, vocab_local, ld, vocab_offset, vocab_total,
                                      _ptr(history), _ptr(history_offsets), _ptr(params), _ptr(records),
                                      _stream(dev)))
    return records


def shard_merge(records, params, vocab_total: int, uniforms=None, rng_state=None, history_offsets=None,
                handle=None):
    """Tokens and statuses from all ranks' records, (nranks, rows, words)."""
    import torch
    from .sampler import params_tensor, _ptr, _stream

    nranks, rows, _ = records.shape
    dev = records.device
    h = handle or N.default_handle(dev.index or 0)
    if not (isinstance(params, torch.Tensor) and params.dtype == torch.uint8):
        params = params_tensor(params, rows, dev)
    tokens = torch.empty(rows, dtype=torch.int32, device=dev)
    status = torch.empty(rows, dtype=torch.int32, device=dev)
    h.check(N.lib().tqfs_shard_merge(h.ptr, _ptr(records.contiguous()), nranks, rows, vocab_total,
                                     _ptr(history_offsets), _ptr(params), _ptr(uniforms), _ptr(rng_state),
                                     _ptr(tokens), _ptr(status), _stream(dev)))
    return tokens, status


class NcclComm:
    """A library-owned NCCL communicator over the ranks of a torch.distributed
    group; the unique id travels over that group (any backend)."""

    def __init__(self, rank: int, nranks: int, device: int, group=None, handle: Optional[N.Handle] = None,
                 timeout_ms: int = 120_000):
        import ctypes
        import torch
        import torch.distributed as dist

        self.handle = handle or N.default_handle(device)
        uid = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            buf = (ctypes.c_uint8 * 128)()
            st = N.lib().tqfs_nccl_unique_id(ctypes.addressof(buf))
            if st != 0:
                raise N.TqfsError(st, "ncclGetUniqueId")
            uid.copy_(torch.tensor(list(buf), dtype=torch.uint8))
        if dist.get_backend(group) == "nccl":
            uid_dev = uid.to(f"cuda:{device}")
            dist.broadcast(uid_dev, 0, group=group)
            uid = uid_dev.cpu()
        else:
            dist.broadcast(uid, 0, group=group)
        idbuf = (ctypes.c_uint8 * 128)(*uid.tolist())
        comm = ctypes.c_void_p()
        self.handle.check(N.lib().tqfs_nccl_comm_init_timeout(self.handle.ptr, nranks, rank, ctypes.addressof(idbuf),
                                                              int(timeout_ms), ctypes.byref(comm)))
        self.ptr = comm.value
        self.rank, self.nranks = rank, nranks

    def wait(self, stream=None, timeout_ms: int = 10_000) -> None:
        """Host watchdog over this communicator's collectives on `stream` (the
        current stream by default): raises TqfsError (TIMEOUT) and aborts the
        communicator when they do not complete within timeout_ms."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream()
        self.handle.check(N.lib().tqfs_nccl_wait(self.handle.ptr, self.ptr, s.cuda_stream, int(timeout_ms)))

    def close(self) -> None:
        if self.ptr:
            N.lib().tqfs_nccl_comm_destroy(self.ptr)
            self.ptr = None


def sample_vocab_sharded(comm: NcclComm, logits, params, vocab_offset: int, vocab_total: int,
                         uniforms=None, rng_state=None, history=None, history_offsets=None):
    """One vocabulary-sharded sampling step on this rank; every rank gets the
    same (tokens, status)."""
    import torch
    from .sampler import params_tensor, _ptr, _stream

    rows, vocab_local = logits.shape
    ld = logits.stride(0)
    dev = logits.device
    h = comm.handle
    dtype = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}[logits.dtype]
    if not (isinstance(params, torch.Tensor) and params.dtype == torch.uint8):
        params = params_tensor(params, rows, dev)
    tokens = torch.empty(rows, dtype=torch.int32, device=dev)
    status = torch.empty(rows, dtype=torch.int32, device=dev)
    h.check(N.lib().tqfs_sample_vocab_sharded(
        h.ptr, comm.ptr, comm.nranks, _ptr(logits), dtype, rows, vocab_local, ld, vocab_offset, vocab_total,
        _ptr(history), _ptr(history_offsets), _ptr(params), _ptr(uniforms), _ptr(rng_state),
        _ptr(tokens), _ptr(status), _stream(dev)))
    return tokens, status
