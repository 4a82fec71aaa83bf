"""Accuracy fixtures of the reference's own training, for the accuracy-parity
test (tests/test_gpu_accuracy.py): with independent random numbers, the
engine must reach the same test accuracy after the same epochs.

    python tests/golden/make_accuracy.py --cutm   # on a GPU: the reference's kernel.cu
                                                  # (oracle/_ref, shapes acc_vanilla / acc_coal)
    python tests/golden/make_accuracy.py --pytm   # the reference's numpy TM (needs the
                                                  # reference checkout: src/pytm/base.py)

Data: seeded prototype data (10 classes, 784 features, prototype bits 1 with
p = 0.2, each bit flipped with p = 0.33), 4000 training / 10000 test samples,
2 epochs; 48 seeds for the small models (the standard error of a 48-seed
mean is about 0.15 point, so two such means can be compared at 0.5 point),
12 seeds for configuration 2's 10k-clause model.  Results are merged into
tests/golden/accuracy.json.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

OUT = os.path.join(HERE, "accuracy.json")
N_TRAIN, N_TEST, EPOCHS, P_FLIP, DATA_SEED = 4000, 10000, 2, 0.33, 11
SEEDS = list(range(1, 49))
SEEDS_LARGE = list(range(1, 13))
# reference arguments of each model (BaseTM kwargs; pytm: its own signature)
MODELS = {
    "acc_vanilla": dict(number_of_clauses_per_class=50, T=15, s=3.9, dim=(28, 28, 1), n_classes=10,
                        coalesced=False),
    "acc_coal": dict(number_of_clauses_per_class=400, T=100, s=5.0, dim=(28, 28, 1), n_classes=10),
    "acc_c2": dict(number_of_clauses_per_class=10000, T=1000, s=15.0, dim=(28, 28, 1), n_classes=10),
    "pytm": dict(n_clause=400, T=100, s=5.0, q=1.0, n_class=10, dim=(28, 28, 1)),
}


def data():
    from ytm_b200 import synthetic
    X, y = synthetic.prototypes(N_TRAIN + N_TEST, seed=DATA_SEED, p_flip=P_FLIP)
    return X[:N_TRAIN], y[:N_TRAIN], X[N_TRAIN:], y[N_TRAIN:]


def cutm_reference():
    from oracle.ref import RefKernels
    from oracle.ref_build import SHAPES, derived
    Xtr, ytr, Xte, yte = data()
    out = {}
    for name in ("acc_vanilla", "acc_coal", "acc_c2"):
        kw = SHAPES[name]
        d = derived(kw)
        rk = RefKernels(name)
        ltr, lte = rk.encode(Xtr), rk.encode(Xte)
        T, K = kw["T"], kw["n_classes"]
        Y = np.where(ytr[:, None] == np.arange(K)[None, :], T, -T).astype(np.int32)
        accs = []
        for seed in (SEEDS_LARGE if name == "acc_c2" else SEEDS):
            ta = np.full((d["C"], d["L"]), kw.get("number_of_ta_states", 256) // 2, np.uint32)  # base.py:209
            w = rk.init_weights(seed)
            pw = np.zeros((d["C"], d["P"]), np.int32)
            for ep in range(EPOCHS):
                rk.fit(ta, w, pw, ltr, Y, seed=seed * 1000 + ep)
            cs = rk.infer(ta, w, lte)
            accs.append(float((cs.argmax(1) == yte).mean()))
        out[name] = {"accuracies": accs, "mean": float(np.mean(accs)), "epochs": EPOCHS, "source": "kernel.cu"}
        print(name, out[name], flush=True)
    return out


def _pytm_one(args):
    src, seed = args
    import contextlib
    import io
    sys.path.insert(0, src)
    from pytm.base import BaseTM
    Xtr, ytr, Xte, yte = data()
    tm = BaseTM(seed=seed, **MODELS["pytm"])
    with contextlib.redirect_stderr(io.StringIO()):  # pytm's progress bars
        for _ in range(EPOCHS):
            tm.fit(Xtr.astype(bool), ytr)
        return float((tm.predict(Xte.astype(bool)) == yte).mean())


def pytm_reference(ref_root=None):
    """The reference's numpy TM, one process per seed (pytm is single-threaded)."""
    from multiprocessing import Pool

    from oracle.ref_build import DEFAULT_REF
    src = os.path.join(ref_root or DEFAULT_REF, "src")
    with Pool(os.cpu_count()) as pool:
        accs = pool.map(_pytm_one, [(src, s) for s in SEEDS])
    out = {"pytm": {"accuracies": accs, "mean": float(np.mean(accs)), "epochs": EPOCHS, "source": "pytm/base.py"}}
    print(out, flush=True)
    return out


def main(argv):
    res = json.load(open(OUT)) if os.path.exists(OUT) else {}
    res["data"] = dict(n_train=N_TRAIN, n_test=N_TEST, epochs=EPOCHS, p_flip=P_FLIP, data_seed=DATA_SEED,
                       seeds=SEEDS, seeds_large=SEEDS_LARGE)
    res["models"] = {k: {kk: (list(vv) if isinstance(vv, tuple) else vv) for kk, vv in v.items()}
                     for k, v in MODELS.items()}
    if "--cutm" in argv:
        res.update(cutm_reference())
    if "--pytm" in argv:
        res.update(pytm_reference())
    with open(OUT, "w") as f:
        json.dump(res, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1:])
