"""Generate the golden fixtures of tests/golden/ from the reference's OWN kernels.

Runs on a GPU machine with oracle/_ref/ref_<shape>.so built (oracle/ref_build.py
compiles Mayur1009/YTM src/cutm/cuda/kernel.cu from source).  For every shape in
oracle/ref_build.SHAPES it draws seeded inputs and TA states, runs the
reference kernels, and stores inputs and outputs in tests/golden/<shape>.npz:

  inference shapes (inf_*): encode_batch, pack_clauses,
      calc_class_sums_infer_batch, transform, transform_patchwise
      (kernel.cu:76-204, 319-394), and init_weights where it is deterministic;
  training shapes (tr_*): single iterations of the _fit loop (base.py:305-357)
      with s = 1, q = K-1 and T = 1, where every random draw of the reference is
      forced (u <= 1/s, u <= Q_PROB always hold; update probabilities are 0 or
      1 because no class sum is 0).  Only the patch pick stays random when
      several patches match; the fixture records the pick the reference made.

    python tests/golden/make_golden.py [shape ...]
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.ref_build import SHAPES, derived  # noqa: E402

N_INFER = 6
N_TRAIN_CASES = 12


def gen_inputs(kw, N, rng, density=0.3):
    D = kw["dim"][0] * kw["dim"][1] * kw["dim"][2]
    return (rng.random((N, D)) < density).astype(np.uint32)


def gen_state(kw, lits, rng, n_states=None):
    """TA states u32 [C][L]: mostly excluded (<= half), each clause including a
    few literals that are 1 in some patch of some sample (so clauses fire), a
    few clauses empty, a few with random includes; values cover 0, half, half+1
    and max."""
    d = derived(kw)
    C, L = d["C"], d["L"]
    ns = n_states or kw.get("number_of_ta_states", 256)
    half = ns // 2
    ta = rng.integers(0, half + 1, size=(C, L)).astype(np.uint32)
    ta[:, rng.integers(0, L, size=3)] = 0
    N, P, W = lits.shape
    bits = np.unpackbits(lits.view(np.uint8).reshape(N, P, W * 4), axis=2, bitorder="little")[:, :, :L]
    for c in range(C):
        kind = rng.random()
        if kind < 0.1:
            continue  # empty clause
        if kind < 0.2:
            idx = rng.choice(L, size=rng.integers(1, 6), replace=False)
        else:
            n, p = rng.integers(N), rng.integers(P)
            ones = np.flatnonzero(bits[n, p])
            if len(ones) == 0:
                continue
            idx = rng.choice(ones, size=min(len(ones), int(rng.integers(1, 5))), replace=False)
        ta[c, idx] = rng.integers(half + 1, ns + 1, size=len(idx))
    ta[0, 0] = ns
    return ta


def gen_weights(kw, rng, lo=-4, hi=5):
    d = derived(kw)
    C, K = d["C"], d["K"]
    if kw.get("coalesced", True):
        w = rng.integers(lo, hi, size=(C, K))
    else:
        w = np.zeros((C, K), np.int64)
        cpc = kw["number_of_clauses_per_class"]
        for c in range(C):
            w[c, c // cpc] = rng.integers(lo, hi)
    return w.astype(np.float32)


def make_inference(name, kw, seed):
    from oracle.ref import RefKernels
    rk = RefKernels(name)
    rng = np.random.default_rng(seed)
    X = gen_inputs(kw, N_INFER, rng)
    lits = rk.encode(X)
    ta = gen_state(kw, lits, rng)
    w = gen_weights(kw, rng)
    bias = rng.integers(-3, 4, size=rk.K).astype(np.float32)
    packed, ninc = rk.pack(ta)
    cs = rk.infer(ta, w, lits)
    cs_bias = rk.infer(ta, w, lits, bias=bias)
    tr = rk.transform(ta, lits)
    trp = rk.transform(ta, lits, patchwise=True)
    out = dict(X=X, lits=lits, ta=ta, w=w, bias=bias, packed=packed, ninc=ninc, cs=cs, cs_bias=cs_bias,
               transform=tr.astype(np.uint8), transform_patchwise=trp.astype(np.uint8))
    if not kw.get("coalesced", True):
        out["init_weights"] = rk.init_weights(seed)
    return out


def make_training(name, kw, seed):
    from oracle.ref import RefKernels
    rk = RefKernels(name)
    rng = np.random.default_rng(seed)
    d = derived(kw)
    C, K, P = d["C"], d["K"], d["P"]
    T = kw["T"]
    cases = {k: [] for k in ("lits", "Y", "e", "ta", "w", "pw", "drop", "ta1", "w1", "pw1", "sel", "cs")}
    made = tries = 0
    while made < N_TRAIN_CASES and tries < 2000:
        tries += 1
        N = 3
        X = gen_inputs(kw, N, rng, density=0.4)
        lits = rk.encode(X)
        ta = gen_state(kw, lits, rng)
        w = gen_weights(kw, rng, -3, 4)
        w[w == 0] = 1
        if not kw.get("coalesced", True):
            cpc = kw["number_of_clauses_per_class"]
            for c in range(C):
                w[c, [k for k in range(K) if k != c // cpc]] = 0
        pw = rng.integers(0, 3, size=(C, P)).astype(np.int32)
        labels = rng.integers(0, K, size=N)
        Y = np.where(labels[:, None] == np.arange(K)[None, :], T, -T).astype(np.int32)
        e = int(rng.integers(0, N))
        drop = (rng.random(C) < 0.1).astype(np.uint32) if made % 3 == 2 else np.zeros(C, np.uint32)
        ta1, w1, pw1 = ta.copy(), w.copy(), pw.copy()
        sel, cs = rk.train_step(ta1, w1, pw1, lits, Y, e, drop=drop, seed=seed + tries)
        if np.any(cs == 0):
            continue  # an update probability of 1/2 would make the step random
        for k, v in dict(lits=lits, Y=Y, e=e, ta=ta, w=w, pw=pw, drop=drop, ta1=ta1, w1=w1, pw1=pw1, sel=sel,
                         cs=cs).items():
            cases[k].append(v)
        made += 1
    if made < N_TRAIN_CASES:
        raise RuntimeError(f"{name}: only {made} deterministic cases in {tries} tries")
    return {k: np.stack([np.asarray(v) for v in vs]) for k, vs in cases.items()}


def main(names):
    for i, (name, kw) in enumerate(SHAPES.items()):
        if names and name not in names:
            continue
        seed = 1000 + i
        if name.startswith("acc_"):
            continue  # accuracy shapes: tests/golden/make_accuracy.py
        if derived(kw)["L"] % 4:
            raise ValueError(f"{name}: the reference kernels fault on LITERALS % 4 != 0; not run")
        data = make_training(name, kw, seed) if name.startswith("tr_") else make_inference(name, kw, seed)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **data)
        print(path, os.path.getsize(path))


if __name__ == "__main__":
    main(sys.argv[1:])
