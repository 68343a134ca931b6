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

The step is timed in passes of exactly K steps, repeated until about 0.4 s of
device time has run; the median pass is reported. The same line carries
configurations 2 and 3 (`other_workloads`), and with N > 1 GPUs the
vocabulary-split configuration 4 (`vocab_shard`: NCCL all-gather of per-shard
top-50 records, with the collective's share of the step).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c1x256|c1|c0|c2|c4]
  python bench.py --vocab-shard ...      # configuration 4 split by vocabulary as the headline
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


def cpu_baseline(batch, budget_s: float = 12.0, gpu_tokens=None, parity_rows: int = 32):
    """The CPU baseline leg: the oracle (a C++ port of the reference sampler)
    on the host cores, on a bounded sample of the workload: batches of the
    workload's first rows, one row per thread at a time, repeated until about
    budget_s of wall time. As the checker, the same leg compares the GPU's
    tokens for the workload's first `parity_rows` rows with the oracle's
    (a mismatch counts as a boundary tie only when the oracle's own CDF or
    top_p margin is below 1e-5 relative)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = len(os.sched_getaffinity(0))
    n = min(batch.rows, 4 * threads)
    idx = np.arange(n)
    done, t0 = 0, time.perf_counter()
    want = None
    while True:
        want = O.sample_batch(batch.logits[idx], batch.params[idx], batch.hist[: batch.hist_off[n]],
                              batch.hist_off[: n + 1], batch.uniforms[idx], threads=threads)
        done += n
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    base = {"value": done / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{done} rows of the {batch.name} workload ({n} per batch call) in {dt:.1f}s"}
    parity = None
    if gpu_tokens is not None:
        parity = oracle_parity(O, batch, gpu_tokens, want, min(parity_rows, n))
    return base, parity


def oracle_parity(O, batch, gpu_tokens, want, rows):
    lf = batch.logits_f32()
    ident = ties = bad = 0
    for r in range(rows):
        if gpu_tokens[r] == want[r]:
            ident += 1
            continue
        hist = batch.hist[batch.hist_off[r]: batch.hist_off[r + 1]].astype(np.int64).astype(np.uint32)
        res = O.sample(lf[r], hist, batch.params[r], u=float(batch.uniforms[r]))
        if res.debug.cdf_margin < 1e-5 or res.debug.topp_margin < 1e-5:
            ties += 1
        else:
            bad += 1
    return {"rows": rows, "identical": ident, "boundary_ties": ties, "mismatches": bad,
            "checker": "oracle (C++ restatement of src/sampling/mod.rs)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    batch = workload(args.workload, 0, args.seed)
    base, _ = cpu_baseline(batch, budget_s=max(5.0, 0.5 * (args.steps + args.warmup)))
    line = {
        "impl": "reference", "metric": "sampled rows/sec at V=151,936", "value": base["value"],
        "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * batch.rows / base["value"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": batch.dtype,
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


def timed_passes(step, steps, stream, world, min_s=0.4, max_passes=400):
    """Times `steps` steps per pass with CUDA events on the launching stream,
    repeating passes until about min_s of device time has run, after one
    barrier + synchronize; the passes' times are maxed over ranks pass by
    pass. Returns (median pass ms, pass stats)."""
    import torch
    barrier(world)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    for i in range(steps):
        step(i)
    ev[1].record(stream)
    torch.cuda.synchronize()
    first = ev[0].elapsed_time(ev[1])
    passes = int(max(1, min(max_passes, math.ceil(min_s * 1000.0 / max(first, 1e-3)))))
    passes = int(max_over_ranks(float(passes), world))   # every rank runs the same passes
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(passes + 1)]
    barrier(world)
    torch.cuda.synchronize()
    evs[0].record(stream)
    for p in range(passes):
        for i in range(steps):
            step(p * steps + i)
        evs[p + 1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = [evs[p].elapsed_time(evs[p + 1]) for p in range(passes)]
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor(ms, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.cpu().tolist()
    med = statistics.median(ms)
    return med, {"passes": passes, "steps_per_pass": steps, "pass_ms_median": round(med, 5),
                 "pass_ms_min": round(min(ms), 5), "pass_ms_max": round(max(ms), 5),
                 "timed_device_ms_total": round(sum(ms), 3)}


def device_logits(batch, dev, nbuf=1):
    """nbuf device copies of the batch's logits with distinct contents (ids
    rolled), enough of them to exceed 2x L2 when nbuf is chosen so."""
    import torch
    if batch.dtype == "f32":
        base = torch.from_numpy(batch.logits)
    else:
        base = torch.from_numpy(batch.logits.view(np.int16)).view(torch.bfloat16)
    return [torch.roll(base, shifts=i * 977, dims=1).to(dev).contiguous() if i else base.to(dev)
            for i in range(nbuf)]


class SampleStep:
    """One tqfs_sample call per step over rotating device buffers."""

    def __init__(self, batch, dev, h, stream, nbuf=1):
        import torch
        import turboqwenfare_b200._native as N
        from turboqwenfare_b200.sampler import params_tensor
        self.batch, self.h, self.L = batch, h, N.lib()
        self.bufs = device_logits(batch, dev, nbuf)
        self.hist = torch.from_numpy(batch.hist if batch.hist.size else np.zeros(1, np.int32)).to(dev)
        self.off = torch.from_numpy(batch.hist_off).to(dev)
        self.params = params_tensor(batch.params, batch.rows, dev)
        self.uni = torch.from_numpy(batch.uniforms).to(dev)
        self.tokens = torch.empty(batch.rows, dtype=torch.int32, device=dev)
        self.sp = stream.cuda_stream
        self.dt = N.DTYPE_F32 if batch.dtype == "f32" else N.DTYPE_BF16

    def __call__(self, i):
        b = self.bufs[i % len(self.bufs)]
        bt = self.batch
        st = self.L.tqfs_sample(self.h.ptr, b.data_ptr(), self.dt, bt.rows, bt.vocab, bt.vocab,
                                self.hist.data_ptr(), self.off.data_ptr(), self.params.data_ptr(),
                                self.uni.data_ptr(), None, self.tokens.data_ptr(), None, None, None, self.sp)
        if st != 0:
            self.h.check(st)


def kernel_times(h, step, steps):
    """Per-launch device time of each library kernel (the library's own CUDA
    events around every launch; kernels run back to back in this mode)."""
    import turboqwenfare_b200._native as N
    L = N.lib()
    L.tqfs_set_timing(h.ptr, 1)
    for i in range(steps):
        step(i)
    kms = (ctypes.c_float * 5)()
    launches = (ctypes.c_int64 * 5)()
    L.tqfs_get_timing(h.ptr, 5, kms, launches)
    L.tqfs_set_timing(h.ptr, 0)
    names = ["stream_kernel", "general_kernel", "window_kernel", "mtp_kernels", "unused"]
    return {names[i]: (kms[i] / launches[i] if launches[i] else 0.0) for i in range(5)}


def run_other_workloads(args, rank, world, local, h, stream, peak):
    """Configurations 2 and 3 on this rank (weak scaling: each rank its own
    rows), timed like the headline; their lines' figures go into the
    headline's JSON under `other_workloads`."""
    import torch
    import turboqwenfare_b200._native as N
    from turboqwenfare_b200 import workloads as W
    from turboqwenfare_b200.sampler import params_tensor
    dev = torch.device("cuda", local)
    out = {}
    c2 = W.config("c2", seed=args.seed + 7919 * rank)
    st2 = SampleStep(c2, dev, h, stream, nbuf=max(1, math.ceil(2 * L2_BYTES / c2.logits.nbytes) + 1))
    for i in range(3):
        st2(i)
    ms, stats = timed_passes(st2, 20, stream, world, min_s=0.2)
    alg = c2.algorithmic_bytes()
    kt = kernel_times(h, st2, 10)
    out["c2"] = {"rows_per_gpu": c2.rows, "dtype": "bf16", "ms_per_step": round(ms / 20, 5),
                 "value": round(c2.rows * world * 20 / (ms / 1000.0), 1), "unit": "rows/s",
                 "whole_step_hbm_frac": round(alg / (ms / 20 / 1000.0) / 1e9 / peak, 4),
                 "algorithmic_bytes": alg, "kernel_us": {k: round(v * 1000, 2) for k, v in kt.items() if v},
                 "general_rows": int(((c2.params["top_k"] == 0) & (c2.params["temperature"] > 0)).sum()),
                 "timing": stats}
    del st2
    m = W.mtp_config(seed=args.seed + 7919 * rank)
    S, Ld, V = m.seqs, m.draft_len, m.target.shape[-1]
    tgt = torch.from_numpy(m.target).to(dev)
    dft = torch.from_numpy(m.draft).to(dev)
    drafts = torch.from_numpy(m.drafts).to(dev)
    params = params_tensor(m.params, S, dev)
    uni = torch.from_numpy(m.uniforms).to(dev)
    acc = torch.empty(S, dtype=torch.int32, device=dev)
    tok = torch.empty(S, dtype=torch.int32, device=dev)
    L = N.lib()

    def mtp_step(i):
        r = L.tqfs_mtp_verify(h.ptr, tgt.data_ptr(), dft.data_ptr(), N.DTYPE_F32, S, Ld, V, V, drafts.data_ptr(),
                              params.data_ptr(), uni.data_ptr(), acc.data_ptr(), tok.data_ptr(), None, None,
                              stream.cuda_stream)
        if r != 0:
            h.check(r)

    for i in range(3):
        mtp_step(i)
    ms, stats = timed_passes(mtp_step, 10, stream, world, min_s=0.2)
    alg = m.algorithmic_bytes()
    out["c3"] = {"seqs_per_gpu": S, "draft_len": Ld, "ms_per_call": round(ms / 10, 5),
                 "value": round(S * (Ld + 1) * world * 10 / (ms / 1000.0), 1), "unit": "verified target rows/s",
                 "whole_call_hbm_frac": round(alg / (ms / 10 / 1000.0) / 1e9 / peak, 4),
                 "algorithmic_bytes": alg, "l2": "inputs resident (136 MB, about L2 size), no flush",
                 "timing": stats}
    del tgt, dft
    out["lm_head"] = run_lm_head(args, rank, world, dev, h, stream)
    return out


def run_lm_head(args, rank, world, dev, h, stream):
    """The producer step on the tensor cores: logits = hidden . W^T for the
    headline's 256 rows, hidden 2048 (the Qwen3.6 geometry of the reference,
    src/model/qwen36/geometry.rs), V = 151,936, bf16 operands (random), f32
    logits; alone (tqfs_lm_head_logits), feeding the sampler (then
    tqfs_sample on c1x256's parameters and histories), and fused
    (tqfs_lm_head_sample). The weights (622 MB) exceed L2, so every step
    streams them from HBM."""
    import torch
    import turboqwenfare_b200._native as N
    from turboqwenfare_b200 import workloads as W
    from turboqwenfare_b200.sampler import params_tensor
    rows, hidden, vocab = 256, 2048, 151_936
    g = torch.Generator(device="cpu").manual_seed(args.seed + 31 * rank)
    x = (torch.randn(rows, hidden, generator=g) * 0.5).to(torch.bfloat16).to(dev)
    w = (torch.randn(vocab, hidden, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    b = W.config("c1x256", seed=args.seed + 7919 * rank)
    hist = torch.from_numpy(b.hist).to(dev)
    off = torch.from_numpy(b.hist_off).to(dev)
    par = params_tensor(b.params, rows, dev)
    uni = torch.from_numpy(b.uniforms).to(dev)
    logits = torch.empty((rows, vocab), dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    tok = torch.empty(rows, dtype=torch.int32, device=dev)
    sts = torch.empty(rows, dtype=torch.int32, device=dev)
    L, s = N.lib(), stream.cuda_stream

    def gemm(i):
        h.check(L.tqfs_lm_head_logits(x.data_ptr(), w.data_ptr(), rows, hidden, vocab, hidden, hidden,
                                      logits.data_ptr(), vocab, err.data_ptr(), s))

    def gemm_sample(i):
        gemm(i)
        h.check(L.tqfs_sample(h.ptr, logits.data_ptr(), N.DTYPE_F32, rows, vocab, vocab, hist.data_ptr(),
                              off.data_ptr(), par.data_ptr(), uni.data_ptr(), None, tok.data_ptr(), None, None,
                              sts.data_ptr(), s))

    def fused(i):
        h.check(L.tqfs_lm_head_sample(h.ptr, x.data_ptr(), w.data_ptr(), rows, hidden, vocab, hidden, hidden,
                                      hist.data_ptr(), off.data_ptr(), par.data_ptr(), uni.data_ptr(), None,
                                      tok.data_ptr(), sts.data_ptr(), s))

    flops = 2.0 * rows * hidden * vocab
    peaks = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")))
    res = {"rows_per_gpu": rows, "hidden": hidden, "vocab": vocab, "operands": "bf16 (random), f32 accumulate",
           "algorithmic_flops": flops, "weight_bytes": vocab * hidden * 2}
    for name, f in (("gemm", gemm), ("gemm_then_sample", gemm_sample), ("fused", fused)):
        for i in range(3):
            f(i)
        ms, stats = timed_passes(f, 10, stream, world, min_s=0.2)
        us = ms / 10 * 1000.0
        res[name] = {"us_per_step": round(us, 1), "rows_per_s": round(rows * world / (us / 1e6), 1), "timing": stats}
    tf = flops / (res["gemm"]["us_per_step"] / 1e6) / 1e12
    res["gemm"]["tflops"] = round(tf, 1)
    res["gemm"]["tensor_frac"] = round(tf / peaks["bf16_tflops"], 4)
    res["gemm"]["weight_gbs"] = round(vocab * hidden * 2 / (res["gemm"]["us_per_step"] / 1e6) / 1e9, 1)
    res["gemm"]["peak_source"] = "measured bf16_tflops (burst)"
    res["err"] = int(err.item())
    del w, logits
    return res


def run_ours(args):
    import torch
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import turboqwenfare_b200._native as N

    batch = workload(args.workload, rank, args.seed)
    nbuf = max(1, math.ceil(2 * L2_BYTES / batch.logits.nbytes) + 1)
    h = N.Handle(local)
    L = N.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    step = SampleStep(batch, dev, h, stream, nbuf)
    dt = step.dt
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()

    # ---- value: passes of exactly K steps, events on the launching stream,
    # each pass maxed over ranks; the median pass is reported --------------
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    pass_ms, timing = timed_passes(step, args.steps, stream, world)
    clk = clocks.stop()
    ms_per_step = pass_ms / args.steps
    value = batch.rows * world * args.steps / (pass_ms / 1000.0)

    # ---- dominant kernel: per-launch duration from the library's events ----
    kt = kernel_times(h, step, args.steps)
    kernel_ms = kt["stream_kernel"]
    alg_bytes = batch.algorithmic_bytes()
    peak, peak_kind = measured_hbm_peak()
    achieved = alg_bytes / (kernel_ms / 1000.0) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_kind,
            "kernel": "stream_kernel", "kernel_us": round(kernel_ms * 1000, 2),
            "algorithmic_bytes_per_launch": alg_bytes,
            "other_kernels_us": {k: round(v * 1000, 2) for k, v in kt.items()
                                 if k != "stream_kernel" and v},
            "traffic": None}
    tpath = os.path.join(ROOT, "profiles", "stream_kernel_traffic.json")
    if os.path.exists(tpath):
        try:
            tr = json.load(open(tpath))
            if tr.get("workload") == batch.name:
                roof["traffic"] = tr["bytes_per_launch"]
        except Exception:
            pass

    # the tokens of the first buffer (the batch's own logits), for the checker
    step(0)
    torch.cuda.synchronize()
    tokens0 = step.tokens.cpu().numpy().copy()

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
    h2d = int(batch.logits.nbytes + batch.hist.nbytes + batch.hist_off.nbytes + batch.params.nbytes
              + batch.uniforms.nbytes)
    e2e = {"value": batch.rows * world * args.e2e_steps / e2e_s, "unit": "rows/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": int(tok_h.numel() * 4), "api": "tqfs_sample_host",
           "h2d_gbs_per_gpu": round(h2d * args.e2e_steps / e2e_s / 1e9, 1)}
    del pinned

    others = run_other_workloads(args, rank, world, local, h, stream, peak)
    vshard = run_vocab_split(args, rank, world, local) if world > 1 else None

    base = parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base, parity = cpu_baseline(batch, gpu_tokens=tokens0)

    # launches of our kernels inside the timed passes: the window pre-pass
    # (rows with a history), the stream kernel (which finalises its rows) and
    # the general kernel
    per_step_launches = 2 + (1 if batch.hist_off is not None else 0)
    line = {
        "metric": "sampled rows/sec at V=151,936", "value": round(value, 1), "unit": "rows/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": batch.dtype, "data": "synthetic",
        "config": config_dict(batch, args, nbuf), "roofline": roof, "cpu_baseline": base, "e2e": e2e,
        "gpu_launches": args.steps * timing["passes"] * per_step_launches, "clocks": clk, "timing": timing,
        "hbm_gbs_whole_step": round(alg_bytes / (ms_per_step / 1000.0) / 1e9, 1),
        "whole_step_hbm_frac": round(alg_bytes / (ms_per_step / 1000.0) / 1e9 / peak, 4),
        "parity": parity, "other_workloads": others,
    }
    if vshard is not None:
        line["vocab_shard"] = vshard
    if rank == 0:
        print(json.dumps(line), flush=True)
    h.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_vocab_split(args, rank, world, local, steps=20):
    """Configuration 4 split by vocabulary over the job's ranks: every rank
    holds ids [offset, offset + V/N) of the same 1,024 bf16 rows; one step =
    per-shard export, one NCCL all-gather of the records, merge and draw on
    every rank (tqfs_sample_vocab_sharded). Strong scaling. Also timed in
    parts (export, all-gather of the records through torch.distributed's
    NCCL, merge) for the collective's share, and checked: rank 0's tokens
    against the unsharded call on its own GPU."""
    import torch
    import torch.distributed as dist
    from turboqwenfare_b200 import workloads as W
    from turboqwenfare_b200.sampler import params_tensor, sample_batch
    from turboqwenfare_b200.sharding import (NcclComm, record_words, sample_vocab_sharded, shard_export,
                                             shard_merge, vocab_shards)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    batch = W.config("c4", seed=args.seed)          # the same rows on every rank
    off0, n = vocab_shards(batch.vocab, world)[rank]
    full = torch.from_numpy(batch.logits.view(np.int16)).view(torch.bfloat16)
    nbuf = max(1, math.ceil(2 * L2_BYTES / (batch.rows * n * 2)) + 1)
    bufs = [torch.roll(full, shifts=i * 977, dims=1)[:, off0:off0 + n].contiguous().to(dev) for i in range(nbuf)]
    hist = torch.from_numpy(batch.hist).to(dev)
    hoff = torch.from_numpy(batch.hist_off).to(dev)
    params = params_tensor(batch.params, batch.rows, dev)
    uni = torch.from_numpy(batch.uniforms).to(dev)
    comm = NcclComm(rank, world, local)
    out = {}

    def step(i):
        out["r"] = sample_vocab_sharded(comm, bufs[i % nbuf], params, off0, batch.vocab, uniforms=uni,
                                        history=hist, history_offsets=hoff)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    ms, stats = timed_passes(step, steps, stream, world, min_s=0.2)
    # parts: export, all-gather, merge, each with its own events
    words = record_words()
    recs = torch.empty((batch.rows, words), dtype=torch.int64, device=dev)
    gathered = torch.empty((world, batch.rows, words), dtype=torch.int64, device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    part = [0.0, 0.0, 0.0]
    barrier(world)
    for i in range(steps):
        ev[0].record(stream)
        shard_export(bufs[i % nbuf], params, off0, batch.vocab, history=hist, history_offsets=hoff, records=recs)
        ev[1].record(stream)
        if world > 1:
            dist.all_gather_into_tensor(gathered, recs)
        else:
            gathered[0].copy_(recs)
        ev[2].record(stream)
        shard_merge(gathered, params, batch.vocab, uniforms=uni, history_offsets=hoff)
        ev[3].record(stream)
        torch.cuda.synchronize()
        for j in range(3):
            part[j] += ev[j].elapsed_time(ev[j + 1])
    part = [max_over_ranks(x / steps, world) for x in part]
    # check: rank 0's sharded tokens (the batch's own logits) == the whole-row call
    step(0)
    torch.cuda.synchronize()
    tok, st = (t.cpu().numpy() for t in out["r"])
    agree = None
    if rank == 0:
        whole = sample_batch(full.to(dev), params, hist, hoff, uniforms=uni, vocab=batch.vocab)
        torch.cuda.synchronize()
        agree = bool((tok == whole.tokens.cpu().numpy()).all() and (st == 0).all())
    comm.close()
    ms_step = ms / steps
    return {"workload": "c4", "rows": batch.rows, "vocab_per_gpu": n, "n_gpus": world,
            "ms_per_step": round(ms_step, 5), "value": round(batch.rows * steps / (ms / 1000.0), 1),
            "unit": "rows/s", "scaling": "strong",
            "parts_ms": {"export": round(part[0], 5), "all_gather": round(part[1], 5), "merge": round(part[2], 5)},
            "all_gather_share": round(part[1] / max(1e-9, sum(part)), 4),
            "all_gather_bytes_per_rank": int(batch.rows * words * 8),
            "tokens_equal_unsharded": agree, "timing": stats}


def run_vocab_sharded(args):
    """`--vocab-shard`: configuration 4 split by vocabulary as the headline
    line (strong scaling)."""
    import torch
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    if world == 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % _free_port(), rank=0, world_size=1)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    r = run_vocab_split(args, rank, world, local, steps=args.steps)
    clk = clocks.stop()
    line = {
        "metric": "sampled rows/sec at V=151,936", "value": r["value"], "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "c4", "rows": r["rows"], "vocab_per_gpu": r["vocab_per_gpu"],
                   "parallelism": f"vocabulary split over {world} GPU(s), NCCL all-gather of per-shard top-50",
                   "seed": args.seed},
        "gpu_launches": args.steps * r["timing"]["passes"] * 4, "clocks": clk, "vocab_shard": r,
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
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
