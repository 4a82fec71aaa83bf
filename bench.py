"""Benchmark: Tsetlin Machine training (and inference) samples/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2] [--impl ours|reference]

Default workload: configuration 2 (coalesced TM, 10k shared clauses, 784
features, 10 classes, T=1000, s=15, mini-batch 256) on seeded synthetic
prototype data.  A step is one mini-batch: clause evaluation of the batch,
class sums (all-reduced over ranks when N > 1: clauses are sharded), and the
Type I/II feedback.  N > 1 runs under torchrun, one rank per GPU, NCCL.

--impl reference times the CPU restatement of the reference algorithm
(oracle/, OpenMP over all host cores) on the same workload, rank 0 only.
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
# DRAM bytes (read + write) per launch of the dominant kernel in the regime
# bench.py times it in (a converged model), from one ncu capture of
# `python -m ytm_b200.profile_kernels --converged 100`; None where no capture
# was made.
TRAFFIC = {"c2": 11.8976e6}


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


def lop3_peak(dev):
    """Measured LOP3 throughput (ops/s) of this GPU: the ceiling of the
    word-test (one LOP3 each) clause evaluation."""
    import ctypes as ct
    import torch
    from ytm_b200 import _lib
    lib = _lib.load()
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    ops = ct.c_uint64(0)
    stream = ct.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    blocks = torch.cuda.get_device_properties(dev).multi_processor_count * 8
    best = 0.0
    for it in (64, 4096, 4096, 4096):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        _lib.check(lib.ytm_probe_lop3(blocks, it, ct.c_void_p(out.data_ptr()), ct.byref(ops), stream))
        b.record()
        torch.cuda.synchronize(dev)
        best = max(best, ops.value / (a.elapsed_time(b) / 1000.0))
    return best


def workload(name, n):
    from ytm_b200 import synthetic
    X, y = synthetic.make(name, n)
    return X, y


def oracle_kw(kw):
    """Model kwargs -> oracle kwargs (rule variants as flags)."""
    kw = dict(kw)
    pytm = kw.pop("rules", "cutm") == "pytm"
    return dict(kw, one_negative=pytm, count_empty=pytm)


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


def run_reference(args):
    """Reference arm: the CPU restatement of the reference algorithm (oracle/,
    OpenMP over all host threads) on the same workload, rank 0 only.  A step
    is one batch of the workload (256 single-sample batches for batch-1
    workloads); models too large for host memory run a leading clause shard
    with the rate scaled by shard/total clauses."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from ytm_b200 import synthetic
    from oracle import oracle as O
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
           "data": "synthetic", "config": {"workload": args.workload, "global_batch": B, **_cfgjson(kw)},
           "cpu_baseline": {"value": v, "unit": "samples/s", "cores": O.get_threads(), "kind": "port",
                            "sample": f"{args.steps} steps of {S} samples (batch {b}) of {args.workload}{note}; "
                                      "oracle/ytm_oracle.c (CPU restatement of kernel.cu), OpenMP"},
           "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def _cfgjson(kw):
    return {k: (list(v) if isinstance(v, tuple) else v) for k, v in kw.items()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5", "p1"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--infer-samples", type=int, default=None)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

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
    n_train = S * (args.steps + args.warmup)
    X, y = workload(name, n_train)
    tm = MultiClassTM(seed=42, device=dev, **kw)
    eng = tm.engine
    lits = tm._encode_device(X)
    Yd = torch.from_numpy(tm.encode_Y(y)).to(dev)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    fused = B == 1 and world == 1 and tm._fused_b1_ok()

    def step(i, ev=None):
        if fused:  # the path MultiClassTM.fit takes at batch 1: one fused launch per sample
            if ev:
                ev[0].record()
            eng.train_fit_b1(lits[i * S:(i + 1) * S], Yd[i * S:(i + 1) * S], tm.sample_counter, None)
            if ev:
                ev[1].record()
            tm.sample_counter += S
            return
        if hasattr(eng, "train_fit_batches") and not ev:  # the path MultiClassTM.fit takes at batch > 1
            par = tm._peer_ar(B * kw["n_classes"])
            eng.train_fit_batches(lits[i * S:(i + 1) * S], Yd[i * S:(i + 1) * S], B, tm.sample_counter, None,
                                  rank == 0, None if par is not None else tm._nccl(), par)
            tm.sample_counter += S
            return
        for j in range(i * S, (i + 1) * S, B):
            lb, yb = lits[j:j + B], Yd[j:j + B]
            t = tm.sample_counter
            cs = eng.train_eval(lb, t, None, add_bias=rank == 0)
            cs = tm._allreduce(cs)
            if ev and j == i * S:
                ev[0].record()
            eng.train_update(cs, yb, lb, t, None)
            if ev and j == i * S:
                ev[1].record()
            tm.sample_counter += B

    for i in range(args.warmup):
        step(i)
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    upd = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(dev) as clk:
        barrier()
        for j in range(args.steps):
            flush.zero_()  # L2 flush between timed steps (outside the step events)
            starts[j].record()
            step(args.warmup + j, upd[j] if fused else None)
            ends[j].record()
        barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if fused:
        upd_ms = [a.elapsed_time(b) for a, b in upd]
    else:
        # the dominant kernel's duration: three more batches through the
        # per-call path with events around the feedback only (after the timed
        # region, so the timed steps stay on the C loop)
        upd = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(3)]
        base = (args.warmup + args.steps) % max(1, n_train // S - 3)
        for r in range(3):
            step(base + r, upd[r])
        barrier()
        upd_ms = [a.elapsed_time(b) for a, b in upd]
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = args.steps * S / (total_ms / 1000.0)

    # roofline of the dominant kernel (feedback): the state's read-modify-write
    cfg = eng.cfg
    if fused:  # per sample: every clause's planes read + written once, literals read once
        alg_bytes = S * (cfg.clause_count * cfg.planes * cfg.words * 4 * 2 + cfg.words * 4 * cfg.patches)
        kernel = "k_fused_b1 (feedback of sample i + evaluation of sample i+1), per 256 launches"
    else:
        # one read and one write of every clause's bit planes per launch (the
        # kernel streams them once per chunk of samples; the roofline counts
        # the minimum), plus the batch's literals
        alg_bytes = cfg.clause_count * cfg.planes * cfg.words * 4 * 2 + B * cfg.words * 4 * cfg.patches
        kernel = "k_update (feedback)"
    # this library's kernels in one step, counted from the CUDA activity trace
    launches = count_launches(lambda: step((args.warmup + args.steps) % max(1, n_train // S)))
    upd_s = statistics.mean(upd_ms) / 1000.0
    peak, peak_kind = load_peaks()
    achieved = alg_bytes / upd_s / 1e9

    # inference samples/s on the trained state
    ni = args.infer_samples or (65536 if name in ("c1", "c2") else 4096)
    Xi, _ = workload(name, ni)
    lits_i = tm._encode_device(Xi)
    for _ in range(2):
        tm._score_device(lits_i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush.zero_()
    e0.record()
    tm._score_device(lits_i)
    e1.record()
    barrier()
    infer_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([infer_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        infer_ms = float(t.item())
    infer_value = ni / (infer_ms / 1000.0)
    word_tests = ni * cfg.clauses * cfg.patches * cfg.words
    # conv models whose patch tile fits shared memory take the sparse match
    # (compacted include words): the dense word-test rate is then only a
    # dense-equivalent figure, not a fraction of the INT pipe
    sparse = cfg.patches > 1 and cfg.words * 129 * 4 <= 220 * 1024

    lop3 = lop3_peak(dev)

    # end to end through the public API: pinned host inputs, H2D, encode, train,
    # D2H of the batch's class sums
    Xh = torch.from_numpy(X.view(np.int32)).pin_memory()
    yh = y
    for i in range(2):
        tm.fit(Xh[i * S:(i + 1) * S], yh[i * S:(i + 1) * S], batch_size=B)
    barrier()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for j in range(args.steps):
        i = (args.warmup + j) % (n_train // S)
        tm.fit(Xh[i * S:(i + 1) * S], yh[i * S:(i + 1) * S], batch_size=B)
        tm.last_class_sums.cpu()
    b_.record()
    barrier()
    e2e_ms = a.elapsed_time(b_)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": args.steps * S / (e2e_ms / 1000.0), "unit": "samples/s",
           "h2d_bytes_per_step": int(S * X.shape[1] * 4 + S * kw["n_classes"] * 4),
           "d2h_bytes_per_step": int(B * kw["n_classes"] * 4)}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u32", "data": "synthetic",
            "config": {"workload": name, "global_batch": B, "samples_per_step": S, "parallelism": f"clause-shard{world}",
                       "l2": "flushed between timed steps (2x L2 write)", **_cfgjson(kw)},
            "e2e": e2e,
            "gpu_launches": launches * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": TRAFFIC.get(name) if world == 1 else None, "kernel": kernel,
                         "peak_kind": peak_kind, "algorithmic_bytes_per_launch": alg_bytes,
                         "launch_ms": statistics.mean(upd_ms)},
            "infer": {"value": infer_value, "unit": "samples/s", "samples": ni,
                      "dense_word_tests_per_s": word_tests / (infer_ms / 1000.0),
                      "lop3_peak_per_s": lop3,
                      "int_pipe_frac": None if sparse else word_tests / (infer_ms / 1000.0) / lop3,
                      "kernel": ("k_match_sparse<any> (compacted include words; dense-equivalent rate)" if sparse
                                 else "k_match<0> (one LOP3 per word test)")},
            "clocks": clk.summary(),
        }
        if not args.no_cpu:
            v, done, el, thr, note = cpu_sample(name, kw, B)
            out["cpu_baseline"] = {"value": v, "unit": "samples/s", "cores": thr, "kind": "port",
                                   "sample": f"{done} samples of {name} in {el:.1f}s{note}, oracle/ytm_oracle.c, "
                                             "OpenMP"}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
