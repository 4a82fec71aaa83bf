"""Accuracy parity: trained with independent random numbers, the engine
reaches the test accuracy the reference's own training reaches (its CUDA
kernels for the cutm rules, its numpy TM for the pytm rules) on the same data
after the same epochs.  Fixtures: tests/golden/accuracy.json, made by
tests/golden/make_accuracy.py.  The tolerance is on the mean over 5 seeds of a
2000-sample test set; one run's sampling spread alone is about 0.7 pt."""
import json
import os

import numpy as np
import pytest

from ytm_b200 import synthetic

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "accuracy.json")
TOL = 0.015  # 1.5 points on the 5-seed mean


def _gold():
    if not os.path.exists(GOLD):
        pytest.skip("accuracy fixtures not generated")
    return json.load(open(GOLD))


def _data(g):
    d = g["data"]
    X, y = synthetic.prototypes(d["n_train"] + d["n_test"], seed=d["data_seed"], p_flip=d["p_flip"])
    n = d["n_train"]
    return X[:n], y[:n], X[n:], y[n:]


@pytest.mark.parametrize("name", ["acc_vanilla", "acc_coal"])
def test_cutm_accuracy_matches_reference_kernels(name):
    from ytm_b200.cutm import MultiClassTM
    g = _gold()
    if name not in g:
        pytest.skip("no reference-kernel accuracy recorded")
    Xtr, ytr, Xte, yte = _data(g)
    kw = {k: (tuple(v) if isinstance(v, list) else v) for k, v in g["models"][name].items()}
    accs = []
    for seed in g["data"]["seeds"]:
        tm = MultiClassTM(seed=seed, **kw)
        for _ in range(g["data"]["epochs"]):
            tm.fit(Xtr, ytr)
        accs.append((tm.predict(Xte)[0] == yte).mean())
    assert abs(np.mean(accs) - g[name]["mean"]) <= TOL, (np.mean(accs), g[name])


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
    assert abs(np.mean(accs) - g["pytm"]["mean"]) <= TOL, (np.mean(accs), g["pytm"])
