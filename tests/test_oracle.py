"""CPU tests of the oracle: Philox known answers, the fixtures the reference's
own kernels produced (tests/golden/*.npz), and the mini-batch definition."""
import numpy as np
import pytest

from oracle import oracle as O
from oracle.ref_build import SHAPES
from tests.helpers import golden_names, load_golden, oracle_for


# Known-answer vectors of Philox4x32-10 published with Random123 (Salmon et al.).
@pytest.mark.parametrize("ctr,key,want", [
    ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
    ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
     [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
])
def test_philox_kat(ctr, key, want):
    assert list(O.philox4x32_10(ctr, key)) == want


def test_golden_fixtures_present():
    names = golden_names()
    want = {n for n in SHAPES if not n.startswith("acc_")}
    assert set(names) == want, f"missing fixtures: {want - set(names)}"


@pytest.mark.parametrize("name", golden_names("inf_"))
def test_oracle_matches_reference_inference(name):
    g = load_golden(name)
    o = oracle_for(name)
    np.testing.assert_array_equal(o.encode(g["X"]), g["lits"])
    packed, ninc = o.pack(g["ta"])
    np.testing.assert_array_equal(packed, g["packed"])
    np.testing.assert_array_equal(ninc, g["ninc"])
    w = g["w"].astype(np.int32)
    np.testing.assert_array_equal(o.infer(g["ta"], w, g["lits"]), g["cs"].astype(np.int32))
    np.testing.assert_array_equal(o.infer(g["ta"], w, g["lits"], bias=g["bias"].astype(np.int32)),
                                  g["cs_bias"].astype(np.int32))
    np.testing.assert_array_equal(o.transform(g["ta"], g["lits"]), g["transform"])
    np.testing.assert_array_equal(o.transform_patchwise(g["ta"], g["lits"]), g["transform_patchwise"])
    if "init_weights" in g:
        np.testing.assert_array_equal(o.init_weights(), g["init_weights"].astype(np.int32))


@pytest.mark.parametrize("name", golden_names("tr_"))
def test_oracle_matches_reference_training_step(name):
    """One forced-decision iteration of the reference's _fit loop, restated by
    the oracle with the reference's own patch pick."""
    g = load_golden(name)
    o = oracle_for(name)
    for i in range(g["e"].shape[0]):
        e = int(g["e"][i])
        lits = g["lits"][i][e:e + 1]
        Y = g["Y"][i][e:e + 1]
        ta = np.ascontiguousarray(g["ta"][i])
        w = g["w"][i].astype(np.int32)
        drop = g["drop"][i]
        sel_ref = g["sel"][i][None, :]
        pw = np.ascontiguousarray(g["pw"][i])
        cs, sel, ninc = o.train_eval(0, ta, w, lits, 1, 0, drop=drop, patch_w=pw.copy())
        np.testing.assert_array_equal(cs[0], g["cs"][i].astype(np.int32), err_msg=f"case {i} class sums")
        np.testing.assert_array_equal(sel >= 0, sel_ref >= 0, err_msg=f"case {i} fired clauses")
        o.train_update(0, ta, w, cs, Y, lits, 1, 0, sel_ref, ninc, drop=drop)
        np.testing.assert_array_equal(ta, g["ta1"][i], err_msg=f"case {i} TA states")
        np.testing.assert_array_equal(w, g["w1"][i].astype(np.int32), err_msg=f"case {i} weights")
        pw_exp = g["pw"][i].copy()
        for c in np.flatnonzero(sel_ref[0] >= 0):
            pw_exp[c, sel_ref[0, c]] += 1
        np.testing.assert_array_equal(g["pw1"][i], pw_exp, err_msg=f"case {i} patch weights")


def test_batch_of_one_equals_per_sample_loop():
    """fit(batch_size=1) over N samples == N single-sample batches (the
    reference's loop); batch_size=4 is a different, documented schedule."""
    o2 = O.Oracle(number_of_clauses_per_class=24, T=15, s=3.0, dim=(40, 1, 1), n_classes=4, seed=5)
    rng = np.random.default_rng(3)
    X = (rng.random((20, 40)) < 0.4).astype(np.uint32)
    lits = o2.encode(X)
    Y = O.encode_Y_multiclass(rng.integers(0, 4, 20), 4, 15)
    runs = []
    for bs in (1, 1, 4):
        ta, w = o2.init_state(), o2.init_weights()
        pw = np.zeros((o2.C, o2.P), np.int32)
        if len(runs) == 1:
            for i in range(20):
                o2.train_batch(ta, w, pw, lits[i:i + 1], Y[i:i + 1], i)
        else:
            o2.fit(ta, w, pw, lits, Y, 0, batch_size=bs)
        runs.append((ta, w, pw))
    for a, b in zip(runs[0], runs[1]):
        np.testing.assert_array_equal(a, b)
    assert any(not np.array_equal(a, b) for a, b in zip(runs[0], runs[2]))


def test_smask_rate():
    """The literal mask is Bernoulli(1/s)."""
    o = O.Oracle(number_of_clauses_per_class=4, T=10, s=10.0, dim=(4, 1, 1), n_classes=2, seed=9)
    ones = sum(bin(o.smask_word(c, t, 0, 0)).count("1") for c in range(4) for t in range(500))
    rate = ones / (4 * 500 * 32)
    assert abs(rate - 0.1) < 0.005


def _smask_spec(o, clause, t, k, w):
    """Count-and-place literal mask, restated from its definition with the
    oracle's Philox4x32-7: count n = first index with r0 < cdf[n]; n distinct
    positions (or 32-n holes when n > 16) from 5-bit fields of r1..r3, then of
    further draws at sub-indices 4w+1, ..."""
    seed = o.cfg.seed
    key = [seed & 0xFFFFFFFF, ((seed >> 32) ^ (t >> 32)) & 0xFFFFFFFF]

    def draw(sub):
        return [int(v) for v in O.philox4x32([clause, t & 0xFFFFFFFF, sub, 2 | (k << 2)], key, 7)]

    cdf = list(o.cfg.s_cdf)
    r = draw(4 * w)
    n = 0
    while n < 32 and r[0] >= cdf[n]:
        n += 1
    holes = n > 16
    need = 32 - n if holes else n
    fields = []
    for word in r[1:]:
        fields += [(word >> (5 * i)) & 31 for i in range(6)]
    sub, m = 4 * w, 0
    while need:
        if not fields:
            sub += 1
            for word in draw(sub):
                fields += [(word >> (5 * i)) & 31 for i in range(6)]
        b = 1 << fields.pop(0)
        if not m & b:
            m |= b
            need -= 1
    return (~m & 0xFFFFFFFF) if holes else m


@pytest.mark.parametrize("s", [1.0, 1.3, 2.0, 10.0, 20.0])
def test_smask_matches_its_definition(s):
    o = O.Oracle(number_of_clauses_per_class=4, T=10, s=s, dim=(4, 1, 1), n_classes=3, seed=2**40 + 17)
    for clause, t, k, w in [(0, 0, 0, 0), (3, 7, 2, 5), (1, 2**32 + 9, 1, 30), (2, 123456, 0, 1023)]:
        assert o.smask_word(clause, t, k, w) == _smask_spec(o, clause, t, k, w)
    if s == 1.0:
        assert o.smask_word(0, 1, 0, 0) == 0xFFFFFFFF


def test_smask_distribution():
    """Count of set literals ~ Binomial(32, 1/s); every position equally
    likely; about one Philox call per word (chi-square-free bounds at 20k
    words)."""
    from math import comb
    s = 6.0
    p = 1 / s
    o = O.Oracle(number_of_clauses_per_class=4, T=10, s=s, dim=(4, 1, 1), n_classes=2, seed=5)
    O.Oracle.smask_count(True)
    words = [o.smask_word(c, t, 1, w) for c in range(4) for t in range(1000) for w in range(5)]
    calls = O.Oracle.smask_count(False)
    n = len(words)
    counts = np.bincount([bin(x).count("1") for x in words], minlength=33)
    for j in range(12):
        want = comb(32, j) * p ** j * (1 - p) ** (32 - j) * n
        assert abs(counts[j] - want) < 5 * np.sqrt(want) + 5
    pos = np.array([[(x >> b) & 1 for b in range(32)] for x in words]).mean(0)
    assert np.all(np.abs(pos - p) < 5 * np.sqrt(p * (1 - p) / n))
    assert n <= calls < 1.01 * n


def test_oracle_threads():
    O.set_threads(2)
    assert O.get_threads() == 2


def _run_spec(o, clause, t, k, w, mi):
    """Type Ib run counts restated from their definition: bit b of literal
    j's 16-bit uniform is bit j of word b & 3 of the Philox4x32-7 call b >> 2
    at sub-index 0x40000000 | 4w | (b >> 2); its count is the first d with
    u < cdf[d]."""
    seed = o.cfg.seed
    key = [seed & 0xFFFFFFFF, ((seed >> 32) ^ (t >> 32)) & 0xFFFFFFFF]
    calls = [[int(v) for v in O.philox4x32([clause, t & 0xFFFFFFFF, 0x40000000 | (w << 2) | i, 2 | (k << 2)],
                                            key, 7)] for i in range(4)]
    cdf = list(o.cfg.run_cdf16[mi])
    m = 8 * (mi + 1)
    out = []
    for j in range(32):
        u = sum(((calls[b >> 2][b & 3] >> j) & 1) << b for b in range(16))
        d = 0
        while d < m and u >= cdf[d]:
            d += 1
        out.append(d)
    return out


@pytest.mark.parametrize("s", [1.0, 3.0, 10.0, 20.0])
def test_type1b_run_counts(s):
    """Definition, and the count distribution Binomial(m, 1/s) of each run size."""
    from math import comb
    o = O.Oracle(number_of_clauses_per_class=4, T=10, s=s, dim=(4, 1, 1), n_classes=3, seed=3 + 2**36)
    for mi in range(8):
        m = 8 * (mi + 1)
        assert list(o.run_counts(2, 2**32 + 5, 1, 7, mi)) == _run_spec(o, 2, 2**32 + 5, 1, 7, mi)
        d = np.concatenate([o.run_counts(c, t, 2, w, mi) for c in range(3) for t in range(60) for w in range(4)])
        if s == 1.0:
            assert (d == m).all()
            continue
        p = 1 / s
        hist = np.bincount(d, minlength=m + 1)
        for j in range(min(m, 12) + 1):
            want = comb(m, j) * p ** j * (1 - p) ** (m - j) * len(d)
            assert abs(hist[j] - want) < 5 * np.sqrt(want) + 6, (mi, j, hist[j], want)


def test_negative_class_set_draw():
    """Coalesced models of at least 32 classes with K * Q <= 2 draw each
    (clause, sample)'s selected negative classes as a set: the count follows
    Binomial(K, Q) and every class is selected with probability Q, as the
    reference's per-class test u < Q (kernel.cu:573) gives."""
    from scipy.stats import binom, chisquare
    K = 40
    o = O.Oracle(number_of_clauses_per_class=4, T=10, s=3.0, dim=(16, 1, 1), n_classes=K, seed=5)
    assert o.cfg.q_select == 1
    Q = 1.0 / (K - 1)
    S = np.array([o.qselect_set(c, 2**32 - 3 + t) for c in range(8) for t in range(2500)])
    n = S.sum(1)
    obs = np.bincount(n, minlength=6)[:6].astype(float)
    obs[5] += (n > 5).sum()
    exp = binom.pmf(np.arange(6), K, Q) * len(n)
    exp[5] = binom.sf(4, K, Q) * len(n)
    assert chisquare(obs, exp).pvalue > 1e-3
    per = S.sum(0).astype(float)
    assert chisquare(per, np.full(K, per.sum() / K)).pvalue > 1e-3
    assert abs(per.sum() / (len(n) * K) - Q) < 4 * np.sqrt(Q / (len(n) * K))
    # the same (clause, sample) gives the same set
    assert np.array_equal(o.qselect_set(3, 77), o.qselect_set(3, 77))
