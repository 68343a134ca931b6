#!/usr/bin/env python3
"""Benchmark of the B200 token-sampling path (libtqfsample).

Metric: sampled rows/sec at V = 151,936 (whole job over all ranks), with the
dominant kernel's achieved HBM bandwidth against the measured copy peak.

Workload (default "c1x256"): the C1 parameter set (T 0.6, top_k 20,
top_p 0.95, repeat/presence/frequency penalties 1.1/0.5/0.3 over 1,024-token
histories, fp32 logits, Philox uniforms) at the batch the north-star target
is stated for: 256 rows per GPU. A step is one tqfs_sample launch over one
batch resident in HBM. Inputs rotate over enough buffers to exceed 2x L2.
Multi-GPU runs shard rows (each rank owns its own 256-row block; no
collective on the data path): weak scaling.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c1x256|c1|c0|c2|c3|c4]
  python bench.py --impl reference ...   # the reference CPU sampler (oracle port)
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c1x256")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--vocab-shard", action="store_true",
                    help="configuration 4's vocabulary split over the ranks (NCCL all-gather of "
                         "per-shard top-k) instead of row sharding")
    return ap.parse_args()


def measured_hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = f"/tmp/tqfs_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    import torch
    if n_gpus <= 1 or "RANK" not in os.environ:
        return 0, 1, 0
    import torch.distributed as dist
    from datetime import timedelta
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def workload(name: str, rank: int, seed: int):
    from turboqwenfare_b200 import workloads as W
    return W.config(name, seed=seed + 7919 * rank)


def cpu_baseline(batch, budget_s: float = 12.0):
    """The oracle (a C++ port of the reference sampler) on the host cores, on a
    bounded sample of the workload: batches of the workload's first rows, one
    row per thread at a time, repeated until about budget_s of wall time."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = len(os.sched_getaffinity(0))
    n = min(batch.rows, 4 * threads)
    idx = np.arange(n)
    done, t0 = 0, time.perf_counter()
    while True:
        O.sample_batch(batch.logits[idx], batch.params[idx], batch.hist[: batch.hist_off[n]],
                       batch.hist_off[: n + 1], batch.uniforms[idx], threads=threads)
        done += n
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{done} rows of the {batch.name} workload ({n} per batch call) in {dt:.1f}s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    batch = workload(args.workload, 0, args.seed)
    base = cpu_baseline(batch, budget_s=max(5.0, 0.5 * (args.steps + args.warmup)))
    line = {
        "impl": "reference", "metric": "sampled rows/sec at V=151,936", "value": base["value"],
        "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * batch.rows / base["value"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": batch.dtype if batch.dtype != "f32" else "f32",
        "data": "synthetic", "config": config_dict(batch, args, None),
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(batch, args, nbuf):
    p = batch.params[0]
    d = {"workload": batch.name, "rows_per_gpu": batch.rows, "vocab": batch.vocab, "logits_dtype": batch.dtype,
         "temperature": float(p["temperature"]), "top_k": int(p["top_k"]), "top_p": round(float(p["top_p"]), 4),
         "history_tokens_per_row": int(batch.hist_off[1] - batch.hist_off[0]),
         "global_batch": batch.rows * args.gpus, "parallelism": f"rows sharded over {args.gpus} GPU(s)",
         "seed": args.seed}
    if nbuf:
        d["l2"] = f"{nbuf} rotating input buffers of {batch.logits.nbytes / 1e6:.1f} MB (> 2x L2)"
    return d


def run_ours(args):
    import torch
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import turboqwenfare_b200._native as N
    from turboqwenfare_b200.sampler import params_tensor

    batch = workload(args.workload, rank, args.seed)
    esz = 4 if batch.dtype == "f32" else 2
    nbuf = max(1, math.ceil(2 * L2_BYTES / batch.logits.nbytes) + 1)
    if batch.dtype == "f32":
        base = torch.from_numpy(batch.logits)
    else:
        base = torch.from_numpy(batch.logits.view(np.int16)).view(torch.bfloat16)
    bufs = []
    for i in range(nbuf):  # distinct contents per buffer (rolled ids)
        bufs.append(torch.roll(base, shifts=i * 977, dims=1).to(dev).contiguous() if i else base.to(dev))
    hist = torch.from_numpy(batch.hist).to(dev)
    off = torch.from_numpy(batch.hist_off).to(dev)
    params = params_tensor(batch.params, batch.rows, dev)
    uni = torch.from_numpy(batch.uniforms).to(dev)
    tokens = torch.empty(batch.rows, dtype=torch.int32, device=dev)
    h = N.Handle(local)
    L = N.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    dt = N.DTYPE_F32 if batch.dtype == "f32" else N.DTYPE_BF16

    def step(i):
        b = bufs[i % nbuf]
        st = L.tqfs_sample(h.ptr, b.data_ptr(), dt, batch.rows, batch.vocab, batch.vocab, hist.data_ptr(),
                           off.data_ptr(), params.data_ptr(), uni.data_ptr(), None, tokens.data_ptr(), None, None,
                           None, sp)
        if st != 0:
            h.check(st)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()

    # ---- value: K steps, events on the launching stream, max over ranks ----
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    ms = max_over_ranks(ms, world)
    ms_per_step = ms / args.steps
    value = batch.rows * world * args.steps / (ms / 1000.0)

    # ---- dominant kernel: per-launch duration from the library's events ----
    L.tqfs_set_timing(h.ptr, 1)
    for i in range(args.steps):
        step(i)
    kms = (ctypes.c_float * 5)()
    launches = (ctypes.c_int64 * 5)()
    L.tqfs_get_timing(h.ptr, 5, kms, launches)
    L.tqfs_set_timing(h.ptr, 0)
    kernel_ms = kms[0] / max(1, launches[0])
    window_ms = kms[2] / max(1, launches[2])
    general_ms = kms[1] / max(1, launches[1])
    finalize_ms = kms[4] / max(1, launches[4])
    alg_bytes = batch.algorithmic_bytes()
    peak, peak_kind = measured_hbm_peak()
    achieved = alg_bytes / (kernel_ms / 1000.0) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_kind,
            "kernel": "stream_kernel", "kernel_us": round(kernel_ms * 1000, 2),
            "algorithmic_bytes_per_launch": alg_bytes,
            "other_kernels_us": {"window_kernel": round(window_ms * 1000, 2),
                                 "finalize_kernel": round(finalize_ms * 1000, 2),
                                 "general_kernel": round(general_ms * 1000, 2)},
            "traffic": None}
    tpath = os.path.join(ROOT, "profiles", "stream_kernel_traffic.json")
    if os.path.exists(tpath):
        try:
            tr = json.load(open(tpath))
            if tr.get("workload") == batch.name:
                roof["traffic"] = tr["bytes_per_launch"]
        except Exception:
            pass

    # ---- e2e through the host-buffer C ABI (H2D + sample + D2H per step) ----
    pinned = torch.empty(batch.logits.shape, dtype=torch.float32 if batch.dtype == "f32" else torch.int16,
                         pin_memory=True)
    pinned.copy_(torch.from_numpy(batch.logits if batch.dtype == "f32" else batch.logits.view(np.int16)))
    hist_h = torch.from_numpy(batch.hist).pin_memory()
    off_h = torch.from_numpy(batch.hist_off).pin_memory()
    par_h = torch.from_numpy(batch.params.view(np.uint8).copy()).pin_memory()
    uni_h = torch.from_numpy(batch.uniforms).pin_memory()
    tok_h = torch.empty(batch.rows, dtype=torch.int32, pin_memory=True)

    def e2e_step():
        st = L.tqfs_sample_host(h.ptr, pinned.data_ptr(), dt, batch.rows, batch.vocab, batch.vocab,
                                hist_h.data_ptr(), off_h.data_ptr(), par_h.data_ptr(), uni_h.data_ptr(), None,
                                tok_h.data_ptr(), sp)
        if st != 0:
            h.check(st)

    for _ in range(3):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = {"value": batch.rows * world * args.e2e_steps / e2e_s, "unit": "rows/s",
           "h2d_bytes_per_step": int(batch.logits.nbytes + batch.hist.nbytes + batch.hist_off.nbytes
                                     + batch.params.nbytes + batch.uniforms.nbytes),
           "d2h_bytes_per_step": int(tok_h.numel() * 4), "api": "tqfs_sample_host"}

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(batch)

    # launches of our kernels inside the timed region: the window pre-pass
    # (rows with a history), the stream, finalize and general kernels
    per_step_launches = 3 + (1 if batch.hist_off is not None else 0)
    line = {
        "metric": "sampled rows/sec at V=151,936", "value": round(value, 1), "unit": "rows/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if batch.dtype == "f32" else "bf16", "data": "synthetic",
        "config": config_dict(batch, args, nbuf), "roofline": roof, "cpu_baseline": base, "e2e": e2e,
        "gpu_launches": args.steps * per_step_launches, "clocks": clk,
        "hbm_gbs_whole_step": round(alg_bytes / (ms_per_step / 1000.0) / 1e9, 1),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    h.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_vocab_sharded(args):
    """Configuration 4: every rank holds all rows' ids [offset, offset + V/N);
    one step = export, NCCL all-gather, merge and draw on every rank. Total
    work is fixed as N grows (strong scaling)."""
    import torch
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from turboqwenfare_b200 import workloads as W
    from turboqwenfare_b200.sampler import params_tensor
    from turboqwenfare_b200.sharding import NcclComm, sample_vocab_sharded, vocab_shards
    batch = W.config("c4", seed=args.seed)  # the same rows on every rank
    off0, n = vocab_shards(batch.vocab, world)[rank]
    full = torch.from_numpy(batch.logits.view(np.int16)).view(torch.bfloat16)
    nbuf = max(1, math.ceil(2 * L2_BYTES / (batch.rows * n * 2)) + 1)
    bufs = [torch.roll(full, shifts=i * 977, dims=1)[:, off0:off0 + n].contiguous().to(dev) for i in range(nbuf)]
    hist = torch.from_numpy(batch.hist).to(dev)
    hoff = torch.from_numpy(batch.hist_off).to(dev)
    params = params_tensor(batch.params, batch.rows, dev)
    uni = torch.from_numpy(batch.uniforms).to(dev)
    if world > 1:
        comm = NcclComm(rank, world, local)
    else:
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % _free_port(), rank=0, world_size=1)
        comm = NcclComm(0, 1, local)

    def step(i):
        sample_vocab_sharded(comm, bufs[i % nbuf], params, off0, batch.vocab, uniforms=uni, history=hist,
                             history_offsets=hoff)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    clk = clocks.stop()
    ms_per_step = ms / args.steps
    alg = batch.rows * batch.vocab * 2 + 4 * int(batch.hist_off[-1]) * world
    line = {
        "metric": "sampled rows/sec at V=151,936", "value": round(batch.rows * args.steps / (ms / 1000.0), 1),
        "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "c4", "rows": batch.rows, "vocab": batch.vocab, "vocab_per_gpu": n,
                   "parallelism": f"vocabulary split over {world} GPU(s), NCCL all-gather of per-shard top-50",
                   "l2": f"{nbuf} rotating input buffers", "seed": args.seed},
        "hbm_gbs_whole_step": round(alg / world / (ms_per_step / 1000.0) / 1e9, 1),
        "gpu_launches": args.steps * 4, "clocks": clk,  # window, stream, finalize (export), merge
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    comm.close()
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()


def run_mtp(args):
    """Configuration 3: MTP verify of 32 sequences x (3 drafts + bonus) per
    call (tqfs_mtp_verify). The metric counts the target rows a call verifies
    (seqs x (L + 1)); rows shard across ranks with no collective."""
    import ctypes
    import torch
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import turboqwenfare_b200._native as N
    from turboqwenfare_b200 import workloads as W
    from turboqwenfare_b200.sampler import params_tensor
    m = W.mtp_config(seed=args.seed + 7919 * rank)
    S, L, V = m.seqs, m.draft_len, m.target.shape[-1]
    rows = S * (L + 1)
    tgt = torch.from_numpy(m.target).to(dev)
    dft = torch.from_numpy(m.draft).to(dev)
    drafts = torch.from_numpy(m.drafts).to(dev)
    params = params_tensor(m.params, S, dev)
    uni = torch.from_numpy(m.uniforms).to(dev)
    acc = torch.empty(S, dtype=torch.int32, device=dev)
    tok = torch.empty(S, dtype=torch.int32, device=dev)
    mask = torch.empty((S, L), dtype=torch.uint8, device=dev)
    st = torch.empty(S, dtype=torch.int32, device=dev)
    h = N.Handle(local)
    Lb = N.lib()
    sp = torch.cuda.current_stream(dev).cuda_stream

    def call(t_ptr, d_ptr):
        r = Lb.tqfs_mtp_verify(h.ptr, t_ptr, d_ptr, N.DTYPE_F32, S, L, V, V, drafts.data_ptr(),
                               params.data_ptr(), uni.data_ptr(), acc.data_ptr(), tok.data_ptr(),
                               mask.data_ptr(), st.data_ptr(), sp)
        if r != 0:
            h.check(r)

    for _ in range(max(args.warmup, 3)):
        call(tgt.data_ptr(), dft.data_ptr())
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call(tgt.data_ptr(), dft.data_ptr())
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    clk = clocks.stop()
    ms_per_step = ms / args.steps
    # e2e: the rows copied from pinned host memory each call, the results back
    th = torch.from_numpy(m.target).pin_memory()
    dh = torch.from_numpy(m.draft).pin_memory()
    out_h = torch.empty(S, dtype=torch.int32, pin_memory=True)
    torch.cuda.synchronize()
    e2 = max(3, args.e2e_steps)
    t0 = time.perf_counter()
    for _ in range(e2):
        tgt.copy_(th, non_blocking=True)
        dft.copy_(dh, non_blocking=True)
        call(tgt.data_ptr(), dft.data_ptr())
        out_h.copy_(tok, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / e2
    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        done, t1 = 0, time.perf_counter()
        while time.perf_counter() - t1 < 10.0:
            O.mtp_verify(m.target, m.draft, m.drafts.astype(np.uint32), m.params, m.uniforms)
            done += rows
        dt = time.perf_counter() - t1
        base = {"value": done / dt, "unit": "rows/s", "cores": 1, "kind": "port",
                "sample": f"{done // rows} oracle verify calls of configuration 3 in {dt:.1f}s"}
    line = {
        "metric": "verified target rows/sec at V=151,936", "value": round(rows * world * args.steps / (ms / 1000.0), 1),
        "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "c3", "seqs_per_gpu": S, "draft_len": L, "vocab": V, "temperature": 0.8,
                   "top_p": 0.9, "l2": "inputs resident (78 MB), no flush"},
        "cpu_baseline": base,
        "e2e": {"value": round(rows * world / e2e_s, 1), "unit": "rows/s",
                "h2d_bytes_per_step": int(m.target.nbytes + m.draft.nbytes), "d2h_bytes_per_step": 4 * S},
        "gpu_launches": args.steps * 2, "clocks": clk,  # the row kernel and the decide kernel
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()


def _free_port():
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.vocab_shard:
        run_vocab_sharded(args)
    elif args.workload == "c3":
        run_mtp(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
