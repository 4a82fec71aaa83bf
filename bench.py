"""Benchmark: Tsetlin Machine training (and inference) samples/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5] [--impl ours|reference]

Default workload: configuration 5 (65,536 shared clauses, 16,384 boolean
features, 100 classes, 4096 TA states = 13 bit planes, T=20000, s=20,
mini-batch 1024) on seeded synthetic planted-rule data; it is the largest
configuration and the one the multi-GPU scaling is quoted on.  A step is one
mini-batch: clause evaluation of the batch, class sums (summed over ranks when
N > 1: clauses are sharded), and the Type I/II feedback.  The timed steps are
the batches W..W+K-1 of a fresh model (the early-training regime, where every
(sample, class) pair is still active).  N > 1 runs under torchrun, one rank
per GPU, NCCL.

The JSON line also carries:
  e2e        the same K batches through MultiClassTM.fit from the same model
             state, pinned host inputs copied in every step, class sums read back;
  roofline   the feedback kernel (the dominant one) against the measured INT
             ceiling, from device counters of its work (ytm_train_update_counted);
  infer      inference samples/s on the trained model (configuration 5:
             2^20 samples, chunked as the reference's _score_batch does);
  target_c1  configuration 1 (20,000 clauses, batch 1) on one GPU, device and
             e2e, with the reference's own CPU path (pytm, baseline/_ref)
             timed on this host beside it;
  cpu_baseline  the CPU restatement (oracle/, OpenMP) on a bounded sample of
             the default workload.

--impl reference times the CPU restatement of the reference algorithm
(oracle/, OpenMP over all host cores) on the same workload, rank 0 only: the
reference has no CPU implementation of the cutm algorithm (its pytm package
covers configuration 1 only and is timed inside target_c1).

--profile all|converged|case  launch a chosen set of kernels inside a
cudaProfilerStart/Stop range for ncu (no JSON line); see profile_run().
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train & infer samples/s (1/2/4/8 B200) + % of HBM/INT-pipe roofline vs CPU"
L2_BYTES = 126 * 1024 * 1024
# DRAM bytes (read + write) of one feedback launch in the regime bench.py
# times it in, from one ncu capture of a reduced-clause model of the same
# workload, scaled by clauses (the feedback's traffic is per clause); None
# where no capture was made.
# configuration 5: 223 MB read + 179 MB written by one k_update launch over
# 4096 clauses (profiles/k_update_c5.md)
TRAFFIC_PER_CLAUSE = {"c5": (223e6 + 179e6) / 4096}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and clock-event (throttle) reasons,
    every 20 ms, from before the timed region until after it."""

    Q = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, dev):
        import torch
        self.bus = None
        try:
            self.bus = torch.cuda.get_device_properties(dev).pci_bus_id
        except Exception:
            pass
        self.index = dev.index if hasattr(dev, "index") else int(dev)
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.5)  # let the sampler start before the timed region
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def _mine(self, rows):
        """Rows of this process's GPU: matched on the PCI bus id, else the
        device index among the GPUs nvidia-smi lists."""
        if self.bus is not None:
            def bus_of(x):  # nvidia-smi "00000000:1B:00.0" -> 0x1B
                try:
                    return int(x.split(":")[1], 16)
                except (IndexError, ValueError):
                    return None
            want = self.bus if isinstance(self.bus, int) else bus_of(str(self.bus))
            m = [r[1:] for r in rows if bus_of(r[0]) == want]
            if m:
                return m
        ids = sorted({r[0] for r in rows})
        if self.index < len(ids):
            return [r[1:] for r in rows if r[0] == ids[self.index]]
        return []

    def summary(self):
        rows = self._mine([r for r in self.rows if len(r) >= 9])
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({n for r in rows for n, v in zip(self.NAMES, r[4:8]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sm), "source": "nvidia-smi -lms 20"}


def count_launches(fn):
    """Kernels of this library (names k_*) that fn launches, from the CUDA
    activity trace of one untimed call."""
    import re

    import torch
    from torch.autograd import DeviceType
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    pat = re.compile(r"(^|[\s:])k_\w+")
    return sum(1 for e in prof.events() if e.device_type == DeviceType.CUDA and pat.search(e.name))


def _probe_lib():
    import ctypes as ct
    from ytm_b200 import build
    path = build.build_probe()
    lib = ct.CDLL(path)
    for name in ("bench_probe_lop3", "bench_probe_philox7"):
        f = getattr(lib, name)
        f.argtypes = [ct.c_int32, ct.c_int32, ct.c_void_p, ct.POINTER(ct.c_uint64), ct.c_void_p]
        f.restype = ct.c_int
    return lib


def probe_peak(dev, name):
    """Measured throughput (operations/s) of this GPU for one probe of
    bench_probe.cu: LOP3 operations (the word-test instruction) or
    Philox4x32-7 calls (the literal-mask draw); best of three long runs."""
    import ctypes as ct

    import torch
    lib = _probe_lib()
    fn = getattr(lib, name)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    ops = ct.c_uint64(0)
    stream = ct.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    blocks = torch.cuda.get_device_properties(dev).multi_processor_count * 8
    best = 0.0
    long_iters = 4096 if name == "bench_probe_lop3" else 256
    for it in (16, long_iters, long_iters, long_iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        rc = fn(blocks, it, ct.c_void_p(out.data_ptr()), ct.byref(ops), stream)
        b.record()
        torch.cuda.synchronize(dev)
        if rc != 0:
            raise RuntimeError(f"{name} failed: CUDA error {rc}")
        best = max(best, ops.value / (a.elapsed_time(b) / 1000.0))
    return best


def workload(name, n):
    from ytm_b200 import synthetic
    return synthetic.make(name, n)


def oracle_kw(kw):
    """Model kwargs -> oracle kwargs (rule variants as flags)."""
    kw = dict(kw)
    pytm = kw.pop("rules", "cutm") == "pytm"
    return dict(kw, one_negative=pytm, count_empty=pytm)


def _cfgjson(kw):
    return {k: (list(v) if isinstance(v, tuple) else v) for k, v in kw.items()}


def config_of(name, world):
    """The `config` object of both arms' JSON lines (identical for a workload)."""
    from ytm_b200 import synthetic
    kw = synthetic.MODELS[name]
    B = synthetic.BATCH[name]
    S = B if B > 1 else 256
    return {"workload": name, "global_batch": B, "samples_per_step": S, "parallelism": f"clause-shard{world}",
            "l2": "flushed between timed steps (2x L2 write)",
            "regime": "batches W..W+K-1 of a fresh model (early training)", **_cfgjson(kw)}


def cpu_sample(name, kw, B, budget_s=20.0, threads=None):
    """Oracle (CPU restatement, OpenMP) training throughput on a bounded sample
    of the workload.  Models whose state would not fit a modest host budget
    (configuration 5: 8.6 GB of u32 states) run a leading clause shard and
    the rate is scaled by shard/total clauses (the work is linear in
    clauses).  Returns (samples/s, samples, seconds, threads, note)."""
    from oracle import oracle as O
    if threads:
        O.set_threads(threads)
    o = O.Oracle(seed=42, **oracle_kw(kw))
    nc = min(o.C, max(64, (256 << 20) // (o.L * 4)))
    b = B if nc == o.C else min(B, 16)
    X, y = workload(name, max(4 * b, 64))
    lits = o.encode(X)
    Y = O.encode_Y_multiclass(y, kw["n_classes"], kw["T"])
    ta = np.ascontiguousarray(o.init_state()[:nc]) if nc < o.C else o.init_state()
    w = np.ascontiguousarray(o.init_weights(0, nc))
    pw = np.zeros((nc, o.P), np.int32)
    done, t, i = 0, 0, 0
    t0 = time.perf_counter()
    while True:
        s = (i * b) % (len(lits) - b + 1)
        cs, sel, ninc = o.train_eval(0, ta, w, lits[s:s + b], b, t, patch_w=pw)
        o.train_update(0, ta, w, cs, Y[s:s + b], lits[s:s + b], b, t, sel, ninc)
        t += b
        done += b
        i += 1
        el = time.perf_counter() - t0
        if el > budget_s or done >= (4 * B if B > 1 else 256):
            break
    rate = done / el * nc / o.C
    note = "" if nc == o.C else f" on clauses 0..{nc - 1} of {o.C}, rate scaled by {nc}/{o.C}"
    return rate, done, el, O.get_threads(), note


def pytm_baseline(budget_s=8.0):
    """The reference's own CPU path: pytm.base.BaseTM.fit (src/pytm/base.py,
    installed unmodified in baseline/_ref) on configuration-1 data, at
    n_clause 2000 and 20000, each on a bounded number of samples.  pytm is a
    numpy loop over samples (bool matmuls, no BLAS): one core."""
    import contextlib
    import io
    refdir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(refdir, "pytm")):
        return {"unavailable": "baseline/_ref has no pytm (run oracle/install_reference.py)"}
    sys.path.insert(0, refdir)
    try:
        from pytm.base import BaseTM
    finally:
        sys.path.remove(refdir)
    X, y = workload("c1", 1200)
    Xb = X.astype(bool)
    yi = y.astype(np.int64)
    out = {"kind": "reference", "source": "pytm.base.BaseTM.fit (src/pytm/base.py:145-156), baseline/_ref",
           "cores": 1, "cpu": _cpu_model(), "numpy": np.__version__, "host_threads": os.cpu_count()}
    for n_clause in (2000, 20000):
        tm = BaseTM(n_clause=n_clause, T=50, s=10.0, q=1.0, n_class=10, dim=(28, 28, 1), seed=1)
        done, el, i = 0, 0.0, 0
        with contextlib.redirect_stderr(io.StringIO()):  # pytm's tqdm bar
            tm.fit(Xb[:2], yi[:2])  # warm-up
            t0 = time.perf_counter()
            while el < budget_s and done < 1000:
                n = 50 if n_clause == 2000 else 5
                tm.fit(Xb[i:i + n], yi[i:i + n])
                done += n
                i = (i + n) % 1000
                el = time.perf_counter() - t0
        out[f"n_clause_{n_clause}"] = {"value": done / el, "unit": "samples/s", "samples": done,
                                       "seconds": round(el, 2)}
    out["best"] = max(out["n_clause_2000"]["value"], out["n_clause_20000"]["value"])
    return out


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args):
    """Reference arm: the CPU restatement of the reference algorithm (oracle/,
    OpenMP over all host threads) on the same workload, rank 0 only.  A step
    is one batch of the workload (256 single-sample batches for batch-1
    workloads); models too large for host memory run a leading clause shard
    with the rate scaled by shard/total clauses."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    from ytm_b200 import synthetic
    kw = synthetic.MODELS[args.workload]
    B = synthetic.BATCH[args.workload]
    O.build()
    O.set_threads(os.cpu_count())
    o = O.Oracle(seed=42, **oracle_kw(kw))
    nc = min(o.C, max(64, (256 << 20) // (o.L * 4)))
    b = B if nc == o.C else min(B, 16)
    S = b if b > 1 else 256
    X, y = workload(args.workload, max(2 * S, 64))
    lits = o.encode(X)
    Y = O.encode_Y_multiclass(y, kw["n_classes"], kw["T"])
    ta = np.ascontiguousarray(o.init_state()[:nc])
    w = np.ascontiguousarray(o.init_weights(0, nc))
    pw = np.zeros((nc, o.P), np.int32)
    t = 0

    def step():
        nonlocal t
        for _ in range(S // b):
            s = t % (len(lits) - b + 1)
            cs, sel, ninc = o.train_eval(0, ta, w, lits[s:s + b], b, t, patch_w=pw)
            o.train_update(0, ta, w, cs, Y[s:s + b], lits[s:s + b], b, t, sel, ninc)
            t += b

    for _ in range(args.warmup):
        step()
    t_start = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t_start
    v = args.steps * S / el * nc / o.C
    note = "" if nc == o.C else f", clauses 0..{nc - 1} of {o.C} (rate scaled by {nc}/{o.C})"
    out = {"metric": METRIC, "impl": "reference", "value": v, "unit": "samples/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el / args.steps,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u32",
           "data": "synthetic", "config": config_of(args.workload, args.gpus),
           "cpu_baseline": {"value": v, "unit": "samples/s", "cores": O.get_threads(), "kind": "port",
                            "sample": f"{args.steps} steps of {S} samples (batch {b}) of {args.workload}{note}; "
                                      "oracle/ytm_oracle.c (CPU restatement of kernel.cu), OpenMP"},
           "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------ helpers of our arm

class Snapshot:
    """Device copy of a model's trainable state and sample counter, so that
    several measurements start from the same state."""

    def __init__(self, tm):
        e = tm.engine
        self.tm = tm
        self.t = tm.sample_counter
        self.bufs = [(x, x.clone()) for x in (e.state, e.weights, e.patch_w, e.bias)]

    def restore(self):
        for dst, src in self.bufs:
            dst.copy_(src)
        self.tm.sample_counter = self.t
        self.tm._model_version += 1


def max_over_ranks(v, world, dev):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def match_counts():
    """(tiles, chunks) of the dense clause match on the current device since
    the previous call (ytm_match_counters reads and clears them)."""
    import ctypes as ct

    import torch
    from ytm_b200 import _lib
    out = (ct.c_uint64 * 2)()
    _lib.check(_lib.load().ytm_match_counters(out, ct.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "ytm_match_counters")
    return int(out[0]), int(out[1])


def planted_infer(tm, lits_i, ni, dev, world, flush, lop3, barrier, rule_seed=1005, n_features=16384):
    """Configuration-5 inference on a model whose clauses are the planted
    rules (clause g includes the 8 literals of rule g mod 1000, the table of
    synthetic.rules_torch): the clauses fire on the samples of their rule, so
    nearly every 64 x 64 match tile holds a matching pair and runs all its
    chunks, the converged-model counterpart of the early-training figure.
    Replaces the model's states (the last leg of the run)."""
    import torch
    eng = tm.engine
    C, W, NB = eng.C, eng.W, eng.NB
    rng = np.random.default_rng(rule_seed)
    feat = rng.integers(0, n_features, (100, 10, 8))
    pol = rng.random((100, 10, 8)) < 0.5
    rule = (tm.clause_lo + np.arange(C)) % 1000
    cls, r = rule // 10, rule % 10
    lit = np.where(pol[cls, r], feat[cls, r], n_features + feat[cls, r])  # [C, 8] literal indices
    top = np.zeros(C * W, np.uint32)
    np.bitwise_or.at(top, (np.arange(C)[:, None] * W + lit // 32).reshape(-1),
                     (np.uint32(1) << (lit % 32).astype(np.uint32)).reshape(-1))
    # the include mask is the top bit plane; the other planes are cleared
    eng.state.zero_()
    eng.state.view(NB, C * W)[NB - 1].copy_(torch.from_numpy(top.view(np.int32)))
    tm._model_version += 1
    tm._score_device(lits_i[:min(ni, 262144)])  # warm-up (include masks, caches)
    match_counts()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush.zero_()
    e0.record()
    cs = tm._score_device(lits_i)
    e1.record()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    tiles, chunks = match_counts()
    nz = int((cs != 0).any(dim=1).sum().item())  # samples with a fired clause
    if world > 1:
        import torch.distributed as dist
        tc = torch.tensor([tiles, chunks], dtype=torch.float64, device=dev)
        dist.all_reduce(tc)
        tiles, chunks = int(tc[0].item()), int(tc[1].item())
    executed = chunks * 64 * 64 * 32
    return {"value": ni / (ms / 1000.0), "unit": "samples/s", "samples": ni,
            "model": "clause g includes the 8 literals of planted rule g mod 1000 (rules_torch table)",
            "samples_with_nonzero_class_sums": nz,
            "match_tiles": tiles, "match_chunks": chunks, "chunks_per_tile": chunks / tiles if tiles else None,
            "int_pipe_frac": executed / (ms / 1000.0) / (lop3 * world)}


def device_lits(name, tm, n, dev, seed=777):
    """The engine input of n synthetic samples (literals [n, 1, W], or packed
    bit images for convolutional models), generated and encoded in chunks
    (configuration 5's 2^20 samples would be 64 GB as host u32)."""
    import torch
    from ytm_b200 import synthetic
    shape = (n, tm.engine.cfg.image_words) if tm.number_of_patches > 1 else \
        (n, tm.number_of_patches, tm.number_of_literal_chunks)
    out = torch.empty(shape, dtype=torch.int32, device=dev)
    chunk = 32768
    for i in range(0, n, chunk):
        m = min(chunk, n - i)
        if name == "c5":
            X = synthetic.rules_torch(m, seed + i, dev)
        else:
            X = torch.from_numpy(synthetic.make(name, m, seed=seed + i)[0].view(np.int32)).to(dev)
        out[i:i + m] = tm._input_device(X)
        del X
    return out


def run_target_c1(args, dev, flush, clk_rows=None):
    """Configuration 1 (vanilla, 2000 clauses per class x 10, 784 features,
    batch 1) on this GPU: a step is 256 samples through the fused batch-1
    path (the one MultiClassTM.fit takes), device-timed from a fixed
    warmed-up state; e2e the same samples through MultiClassTM.fit with pinned
    host inputs and the class sums read back per step; beside it the
    reference's pytm on this host."""
    import torch
    from ytm_b200 import synthetic
    from ytm_b200.cutm import MultiClassTM
    kw = synthetic.MODELS["c1"]
    S, K, W = 256, max(args.steps, 10), 3
    X, y = workload("c1", S * (K + W))
    tm = MultiClassTM(seed=42, device=dev, **kw)
    eng = tm.engine
    lits = tm._encode_device(X)
    Yd = torch.from_numpy(tm.encode_Y(y)).to(dev)
    for i in range(W):
        eng.train_fit_b1(lits[i * S:(i + 1) * S], Yd[i * S:(i + 1) * S], tm.sample_counter, None)
        tm.sample_counter += S
    torch.cuda.synchronize()
    snap = Snapshot(tm)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for j in range(K):
        i = W + j
        flush.zero_()
        ev[j][0].record()
        eng.train_fit_b1(lits[i * S:(i + 1) * S], Yd[i * S:(i + 1) * S], tm.sample_counter, None)
        ev[j][1].record()
        tm.sample_counter += S
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    value = K * S / (ms / 1000.0)
    launches = count_launches(lambda: eng.train_fit_b1(lits[:S], Yd[:S], 0, None))
    # e2e from the same state, after one untimed call of the same API path
    # (its host-side set-up happens once, as in any repeated fit)
    Xh = torch.from_numpy(X.view(np.int32)).pin_memory()
    tm.fit(Xh[:S], y[:S], batch_size=1)
    tm.last_class_sums.cpu()
    snap.restore()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for j in range(K):
        i = W + j
        tm.fit(Xh[i * S:(i + 1) * S], y[i * S:(i + 1) * S], batch_size=1)
        tm.last_class_sums.cpu()
    b.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b)
    out = {"workload": "c1", "config": {"global_batch": 1, "samples_per_step": S, **_cfgjson(kw)},
           "value": value, "unit": "samples/s", "steps": K, "warmup_steps": W,
           "us_per_sample": 1e6 / value, "gpu_launches_per_step": launches,
           "e2e": {"value": K * S / (e2e_ms / 1000.0), "unit": "samples/s",
                   "h2d_bytes_per_step": int(S * 784 * 4 + S * kw["n_classes"] * 4),
                   "d2h_bytes_per_step": int(kw["n_classes"] * 4)}}
    if not args.no_cpu:
        pb = pytm_baseline()
        out["cpu_baseline"] = pb
        if "best" in pb:
            out["vs_pytm_best"] = out["e2e"]["value"] / pb["best"]
            out["vs_pytm_20000"] = out["e2e"]["value"] / pb["n_clause_20000"]["value"]
            out["target"] = ">= 50x the best pytm training samples/s (e2e)"
    del tm, eng, lits
    return out


def counted_feedback(tm, lits, Yd, B, base, nb, dev):
    """Run nb batches of the per-call path from the current state with the
    feedback's device counters on; returns the summed counters and the batch
    count."""
    import torch
    eng = tm.engine
    ctr = torch.zeros(6, dtype=torch.int64, device=dev)
    for r in range(nb):
        j = (base + r) * B
        t = tm.sample_counter
        cs = eng.train_eval(lits[j:j + B], t, None, add_bias=tm.rank == 0)
        cs = tm._allreduce(cs)
        eng.train_update(cs, Yd[j:j + B], lits[j:j + B], t, None, counters=ctr)
        tm.sample_counter += B
    torch.cuda.synchronize()
    return [int(v) for v in ctr.cpu().tolist()]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c5", choices=["c1", "c2", "c3", "c4", "c5", "p1"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline legs")
    ap.add_argument("--no-target", action="store_true", help="skip the configuration-1 target object")
    ap.add_argument("--infer-samples", type=int, default=None)
    ap.add_argument("--profile", choices=["all", "converged", "case"], default=None)
    ap.add_argument("--profile-batches", type=int, default=2)
    ap.add_argument("--profile-clauses", type=int, default=None)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return profile_run(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    from ytm_b200 import synthetic
    from ytm_b200.cutm import MultiClassTM

    name = args.workload
    kw = synthetic.MODELS[name]
    B = synthetic.BATCH[name]
    S = B if B > 1 else 256  # samples per step (batch-1 workloads: 256 single-sample batches)
    n_train = S * (max(args.steps, 3) + args.warmup)  # the feedback timing replays 3 batches
    X, y = workload(name, n_train)
    tm = MultiClassTM(seed=42, device=dev, **kw)
    eng = tm.engine
    lits = tm._input_device(X)  # what MultiClassTM.fit feeds the engine (conv models: packed bit images)
    Yd = torch.from_numpy(tm.encode_Y(y)).to(dev)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    fused = B == 1 and world == 1 and tm._fused_b1_ok()

    def step(i):
        if fused:  # the path MultiClassTM.fit takes at batch 1: one fused launch per sample
            eng.train_fit_b1(lits[i * S:(i + 1) * S], Yd[i * S:(i + 1) * S], tm.sample_counter, None)
        else:  # the path MultiClassTM.fit takes at batch > 1: the C batch loop
            par = tm._peer_ar(B * kw["n_classes"])  # None above the peer kernel's size: NCCL
            eng.train_fit_batches(lits[i * S:(i + 1) * S], Yd[i * S:(i + 1) * S], B, tm.sample_counter, None,
                                  rank == 0, None if par is not None else tm._nccl(), par)
        tm.sample_counter += S

    for i in range(args.warmup):
        step(i)
    barrier()
    snap = Snapshot(tm)
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(dev) as clk:
        barrier()
        for j in range(args.steps):
            flush.zero_()  # L2 flush between timed steps (outside the step events)
            starts[j].record()
            step(args.warmup + j)
            ends[j].record()
        barrier()
    if getattr(tm, "_par", None) is not None:
        tm._check_peer_status(tm._par)
    total_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)), world, dev)
    value = args.steps * S / (total_ms / 1000.0)
    launches = None

    # the dominant kernel (feedback) in the same regime: the first timed
    # batches again from the snapshot, through the per-call path with events
    # around the feedback, then once more with its device counters on
    cfg = eng.cfg
    nb = 3 if not fused else 1
    if fused:
        upd_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)][:3]
        ctrs = None
    else:
        snap.restore()
        barrier()
        upd_ms = []
        for r in range(nb):
            j = (args.warmup + r) * B
            t = tm.sample_counter
            cs = eng.train_eval(lits[j:j + B], t, None, add_bias=rank == 0)
            cs = tm._allreduce(cs)
            flush.zero_()
            a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            eng.train_update(cs, Yd[j:j + B], lits[j:j + B], t, None)
            b_.record()
            tm.sample_counter += B
            barrier()
            upd_ms.append(a.elapsed_time(b_))
        snap.restore()
        barrier()
        ctrs = counted_feedback(tm, lits, Yd, B, args.warmup, nb, dev)
    snap.restore()
    barrier()
    launches = count_launches(lambda: step(args.warmup))
    snap.restore()
    barrier()
    upd_s = statistics.mean(upd_ms) / 1000.0

    lop3 = probe_peak(dev, "bench_probe_lop3")
    philox = probe_peak(dev, "bench_probe_philox7")
    hbm_peak, peak_kind = load_peaks()
    NB, W = cfg.planes, cfg.words
    if ctrs is not None:
        units, calls, words, events, dcalls, tests = (v / nb for v in ctrs)
        # INT work one feedback launch executes, counted on the device: every
        # Philox4x32-7 call (literal masks, Type Ib run counts, the decisions
        # of the active pairs) priced at the measured LOP3 : Philox
        # throughput ratio, a ripple add / bit-sliced subtraction over the
        # planes (2 * planes logic ops) per literal-word operation, and a
        # 16-plane carry chain (16 logic ops) per run-count threshold tested.
        # The per-event view of the same work (every (event, literal word)
        # pair of the reference's one-event-at-a-time algorithm) is carried
        # as units_per_launch.event_word_pairs.
        event_words = events * W
        mask_ops = lop3 / philox
        ops = (calls + dcalls) * mask_ops + units * 2 * NB + tests * 16
        alg_bytes = cfg.clause_count * NB * W * 4 * 2 + B * W * 4 * cfg.patches  # one read + write of the planes
        roofline = {"bound": "int", "achieved": ops / upd_s / 1e9, "peak": lop3 / 1e9, "unit": "G int-ops/s",
                    "frac": ops / upd_s / lop3, "traffic": None, "kernel": "k_update (feedback)",
                    "peak_kind": "measured on this GPU (bench_probe.cu LOP3 probe)",
                    "launch_ms": upd_s * 1000.0, "launches_averaged": nb,
                    "units_per_launch": {"event_word_pairs": event_words, "events": events},
                    "op_model": "executed, from device counters: Philox4x32-7 calls x (LOP3 peak / Philox peak) "
                                "+ 2*planes LOP3 per literal-word operation + 16 LOP3 per run-count threshold",
                    "counters_per_launch": {"literal_word_ops": units, "philox7_calls": calls,
                                            "decision_philox7_calls": dcalls, "run_thresholds": tests,
                                            "state_words_streamed": words},
                    "philox7_peak_calls_per_s": philox, "lop3_peak_per_s": lop3,
                    # the same kernel read by ncu (profiles/k_update_c5.md, 4096-clause capture of
                    # this workload's shape and regime)
                    "ncu": {"source": "profiles/k_update_c5.md"},
                    "hbm": {"algorithmic_bytes": alg_bytes, "achieved_gbs": alg_bytes / upd_s / 1e9,
                            "peak_gbs": hbm_peak, "frac": alg_bytes / upd_s / 1e9 / hbm_peak,
                            "peak_kind": peak_kind,
                            "l2_bytes": words * NB * 4 * 2}}
        tpc = TRAFFIC_PER_CLAUSE.get(name)
        if tpc is not None and world == 1:
            roofline["traffic"] = tpc * cfg.clause_count
    else:
        alg_bytes = S * (cfg.clause_count * NB * W * 4 * 2 + W * 4 * cfg.patches)
        roofline = {"bound": "hbm", "achieved": alg_bytes / upd_s / 1e9, "peak": hbm_peak, "unit": "GB/s",
                    "frac": alg_bytes / upd_s / 1e9 / hbm_peak, "traffic": None,
                    "kernel": "k_fused_b1 (feedback of sample i + evaluation of sample i+1), per 256 launches",
                    "peak_kind": peak_kind, "launch_ms": upd_s * 1000.0}

    # end to end through the public API from the same state: pinned host
    # inputs copied in every step, class sums of the step's last batch read back
    # (after one untimed call of the same path: its host-side set-up happens
    # once, as in any repeated fit; then the snapshot's state again)
    Xh = torch.from_numpy(X.view(np.int32)).pin_memory()
    tm.fit(Xh[:S], y[:S], batch_size=B)
    tm.last_class_sums.cpu()
    snap.restore()
    barrier()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for j in range(args.steps):
        i = args.warmup + j
        tm.fit(Xh[i * S:(i + 1) * S], y[i * S:(i + 1) * S], batch_size=B)
        tm.last_class_sums.cpu()
    b_.record()
    barrier()
    e2e_ms = max_over_ranks(a.elapsed_time(b_), world, dev)
    e2e = {"value": args.steps * S / (e2e_ms / 1000.0), "unit": "samples/s",
           "h2d_bytes_per_step": int(S * X.shape[1] * 4 + S * kw["n_classes"] * 4),
           "d2h_bytes_per_step": int(min(B, S) * kw["n_classes"] * 4)}
    del Xh

    # inference samples/s on the trained state
    ni = args.infer_samples or (1 << 20 if name == "c5" else (65536 if name in ("c1", "c2") else 4096))
    del lits
    lits_i = device_lits(name, tm, ni, dev)
    for _ in range(2):  # warm-up at the chunk size the timed call uses (its workspace is then allocated)
        tm._score_device(lits_i[:min(ni, 262144)])
    match_counts()  # clears the device's match counters
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush.zero_()
    e0.record()
    tm._score_device(lits_i)
    e1.record()
    barrier()
    infer_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    tiles, chunks = match_counts()  # executed by this rank's timed call
    if world > 1:
        import torch.distributed as dist
        tc = torch.tensor([tiles, chunks], dtype=torch.float64, device=dev)
        dist.all_reduce(tc)
        tiles, chunks = int(tc[0].item()), int(tc[1].item())
    executed_tests = chunks * 64 * 64 * 32  # a chunk: 32 words x 64 x 64 (row, clause) pairs, one LOP3 each
    infer_value = ni / (infer_ms / 1000.0)
    word_tests = ni * cfg.clauses * cfg.patches * cfg.words  # all clauses (every rank scores its sample slice)
    sparse = cfg.patches > 1 and cfg.words * 129 * 4 <= 220 * 1024
    planted = None
    if name == "c5" and world == 1:  # one rank: a failed leg cannot leave others waiting at a barrier
        try:
            planted = planted_infer(tm, lits_i, ni, dev, world, flush, lop3, barrier)
        except Exception as e:  # a measurement leg: the main line stands without it
            planted = {"error": f"{type(e).__name__}: {e}"}
    del lits_i

    target = None
    if rank == 0 and world == 1 and not args.no_target and name != "c1":
        target = run_target_c1(args, dev, flush)

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u32", "data": "synthetic",
            "config": config_of(name, world),
            "e2e": e2e,
            "gpu_launches": launches * args.steps,
            "roofline": roofline,
            "infer": {"value": infer_value, "unit": "samples/s", "samples": ni,
                      "chunking": "MultiClassTM._score_device chunks of at most 2^31 bytes of literals + fired bits",
                      "dense_word_tests_per_s": word_tests / (infer_ms / 1000.0),
                      "lop3_peak_per_s": lop3,
                      # executed: the 32-word chunks the match tiles processed (device
                      # counters; a tile stops at the chunk after which every pair has a
                      # violation); dense-equivalent: W word tests per (sample, clause)
                      # pair, which can exceed the ceiling; samples are sharded over the
                      # GPUs, so both against the ceiling of all of them
                      "executed_word_tests_per_s": executed_tests / (infer_ms / 1000.0),
                      "match_tiles": tiles, "match_chunks": chunks,
                      "chunks_per_tile": chunks / tiles if tiles else None,
                      "int_pipe_frac": None if sparse else executed_tests / (infer_ms / 1000.0) / (lop3 * world),
                      "dense_equiv_frac": word_tests / (infer_ms / 1000.0) / (lop3 * world),
                      "kernel": ("k_match_sparse<any> (compacted include words; dense-equivalent rate)" if sparse
                                 else "k_match<0> (64 x 64 tiles, one LOP3 per word test, early exit "
                                      "once every pair of the tile is violated; dense-equivalent rate)"),
                      "planted_rules_model": planted},
            "clocks": clk.summary(),
        }
        if target is not None:
            out["target_c1"] = target
        if not args.no_cpu:
            v, done, el, thr, note = cpu_sample(name, kw, B)
            out["cpu_baseline"] = {"value": v, "unit": "samples/s", "cores": thr, "kind": "port",
                                   "sample": f"{done} samples of {name} in {el:.1f}s{note}, oracle/ytm_oracle.c, "
                                             "OpenMP"}
        print(json.dumps(out), flush=True)
    if world > 1:
        tm.close()
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ profiling ranges

def profile_run(args):
    """Launch kernels inside one cudaProfilerStart/Stop range, for
    `ncu --profile-from-start off` (no JSON line; prints "done").

    all        warm-up outside the range (configuration-2 batches, batch-1
               training of configurations 1 and 3, a thermometer encode); in
               the range one configuration-2 training batch and 65,536-sample
               inference, a transform, an encode, two fused batch-1 samples of
               configurations 1 and 3, a patch-wise transform and a
               thermometer encode.
    converged  configuration 2 trained --profile-batches batches outside the
               range, then one batch (evaluation, thresholds, feedback) in it.
    case       --workload with --profile-clauses clauses per class (default:
               the full model), --profile-batches warm-up batches outside the
               range, then one training batch (batch-1 workloads: 2 samples
               of the fused path) and inference of one batch in it."""
    import torch

    from ytm_b200 import synthetic
    from ytm_b200.cutm import MultiClassTM
    torch.cuda.set_device(0)
    if args.profile == "converged":
        nb = args.profile_batches
        X, y = synthetic.make("c2", 256 * (nb + 1))
        tm = MultiClassTM(seed=42, **synthetic.MODELS["c2"])
        lits, Y, e = tm._encode_device(X), torch.from_numpy(tm.encode_Y(y)).cuda(), tm.engine
        for i in range(nb + 1):
            if i == nb:
                torch.cuda.synchronize()
                torch.cuda.profiler.start()
            sl = slice(i * 256, (i + 1) * 256)
            cs = e.train_eval(lits[sl], i * 256, None, True)
            e.train_update(cs, Y[sl], lits[sl], i * 256, None)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print("done", flush=True)
        return
    if args.profile == "case":
        name = args.workload
        kw = dict(synthetic.MODELS[name])
        if args.profile_clauses:
            kw["number_of_clauses_per_class"] = args.profile_clauses
        B = synthetic.BATCH[name]
        nb = args.profile_batches
        n = (B if B > 1 else 2) * (nb + 1)
        X, y = synthetic.make(name, n)
        tm = MultiClassTM(seed=42, **kw)
        lits, Y, e = tm._input_device(X), torch.from_numpy(tm.encode_Y(y)).cuda(), tm.engine
        step = B if B > 1 else 2
        for i in range(nb + 1):
            sl = slice(i * step, (i + 1) * step)
            if i == nb:
                torch.cuda.synchronize()
                torch.cuda.profiler.start()
            if B == 1 and tm._fused_b1_ok():
                e.train_fit_b1(lits[sl], Y[sl], i * step, None)
            else:
                for j in range(sl.start, sl.stop, B):
                    cs = e.train_eval(lits[j:j + B], j, None, True)
                    e.train_update(cs, Y[j:j + B], lits[j:j + B], j, None)
        e.infer(lits[-step:])
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print("done", flush=True)
        return
    X, y = synthetic.make("c2", 256 * 5)
    tm = MultiClassTM(seed=42, **synthetic.MODELS["c2"])
    lits, Y, e = tm._encode_device(X), torch.from_numpy(tm.encode_Y(y)).cuda(), tm.engine
    for i in range(4):
        sl = slice(i * 256, (i + 1) * 256)
        cs = e.train_eval(lits[sl], i * 256, None, True)
        e.train_update(cs, Y[sl], lits[sl], i * 256, None)
    Xi, _ = synthetic.make("c2", 65536)
    Xi_d = torch.from_numpy(Xi.view(np.int32)).cuda()
    li = tm._encode_device(Xi)
    X1, y1 = synthetic.make("c1", 600)
    t1 = MultiClassTM(seed=1, **synthetic.MODELS["c1"])
    l1, Y1 = t1._encode_device(X1), torch.from_numpy(t1.encode_Y(y1)).cuda()
    t1.engine.train_fit_b1(l1[:500], Y1[:500], 0, None)
    X3, y3 = synthetic.make("c3", 300)
    t3 = MultiClassTM(seed=1, **synthetic.MODELS["c3"])
    l3, Y3 = t3._input_device(X3), torch.from_numpy(t3.encode_Y(y3)).cuda()
    t3.engine.train_fit_b1(l3[:200], Y3[:200], 0, None)
    kw4 = dict(synthetic.MODELS["c4"])
    kw4["number_of_clauses_per_class"] = 64
    t4 = MultiClassTM(seed=1, **kw4)
    img = torch.randint(0, 256, (2048, 32 * 32 * 3), dtype=torch.uint8, device="cuda")
    t4.encode_thermometer(img, 8, on_device=True)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    i = 4
    sl = slice(i * 256, (i + 1) * 256)
    cs = e.train_eval(lits[sl], i * 256, None, True)
    e.train_update(cs, Y[sl], lits[sl], i * 256, None)
    e.infer(li)
    e.transform(li[:4096])
    e.encode(Xi_d)
    t1.engine.train_fit_b1(l1[500:502], Y1[500:502], 500, None)
    t3.engine.train_fit_b1(l3[200:202], Y3[200:202], 200, None)
    t3.engine.transform_patchwise(l3[:16])
    t4.encode_thermometer(img, 8, on_device=True)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("done", flush=True)


if __name__ == "__main__":
    main()
