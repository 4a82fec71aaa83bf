"""Accuracy parity: trained with independent random numbers, the engine
reaches the test accuracy the reference's own training reaches (its CUDA
kernels for the cutm rules, its numpy TM for the pytm rules) on the same data
after the same epochs.  Fixtures: tests/golden/accuracy.json, made by
tests/golden/make_accuracy.py.

The models of configuration-1 and -2 rules with few clauses are compared on
the mean over 48 seeds of a 10,000-sample test set: the standard error of each
mean is about 0.15 point, so the +-0.5 point bound is about three standard
errors of the difference.  Configuration 2's own model (10k shared clauses)
is compared over 12 seeds, within 0.5 point or three standard errors of the
difference of the means, whichever is larger."""
import json
import os

import numpy as np
import pytest

from ytm_b200 import synthetic

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "accuracy.json")
TOL = 0.005  # 0.5 point on the seed mean


def _tol(ours, ref):
    """TOL, or three standard errors of the difference of the two seed means
    when fewer seeds make that larger."""
    se = np.sqrt(np.var(ours, ddof=1) / len(ours) + np.var(ref, ddof=1) / len(ref))
    return max(TOL, 3 * se)


def _gold():
    if not os.path.exists(GOLD):
        pytest.skip("accuracy fixtures not generated")
    return json.load(open(GOLD))


def _data(g):
    d = g["data"]
    X, y = synthetic.prototypes(d["n_train"] + d["n_test"], seed=d["data_seed"], p_flip=d["p_flip"])
    n = d["n_train"]
    return X[:n], y[:n], X[n:], y[n:]


@pytest.mark.parametrize("name", ["acc_vanilla", "acc_coal", "acc_c2"])
def test_cutm_accuracy_matches_reference_kernels(name):
    from ytm_b200.cutm import MultiClassTM
    g = _gold()
    if name not in g or name not in g["models"]:
        pytest.skip("no reference-kernel accuracy recorded")
    Xtr, ytr, Xte, yte = _data(g)
    kw = {k: (tuple(v) if isinstance(v, list) else v) for k, v in g["models"][name].items()}
    seeds = g["data"]["seeds_large"] if name == "acc_c2" else g["data"]["seeds"]
    assert len(g[name]["accuracies"]) == len(seeds)
    accs = []
    for seed in seeds:
        tm = MultiClassTM(seed=seed, **kw)
        for _ in range(g["data"]["epochs"]):
            tm.fit(Xtr, ytr)  # batch 1, as the reference trains
        accs.append((tm.predict(Xte)[0] == yte).mean())
    tol = TOL if name != "acc_c2" else _tol(accs, g[name]["accuracies"])
    assert abs(np.mean(accs) - g[name]["mean"]) <= tol, (np.mean(accs), g[name]["mean"], tol)


def test_pytm_accuracy_matches_reference_pytm():
    from ytm_b200.pytm import BaseTM
    g = _gold()
    if "pytm" not in g:
        pytest.skip("no pytm accuracy recorded")
    Xtr, ytr, Xte, yte = _data(g)
    kw = {k: (tuple(v) if isinstance(v, list) else v) for k, v in g["models"]["pytm"].items()}
    accs = []
    for seed in g["data"]["seeds"]:
        tm = BaseTM(seed=seed, **kw)
        for _ in range(g["data"]["epochs"]):
            tm.fit(Xtr.astype(bool), ytr)
        accs.append((tm.predict(Xte.astype(bool)) == yte).mean())
    assert abs(np.mean(accs) - g["pytm"]["mean"]) <= TOL, (np.mean(accs), g["pytm"]["mean"])
