"""GPU parity tests: the CUDA engine (through the C ABI) against the reference
kernels' fixtures and against the oracle.  Everything integer: bit-exact."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle.ref_build import SHAPES
from tests.helpers import golden_names, lib_kwargs, load_golden, oracle_kwargs
from ytm_b200 import _lib
from ytm_b200.engine import CudaEngine

pytestmark = pytest.mark.gpu


def engine_for(kw, seed=0, rank=0, world=1):
    cfg = _lib.make_config(**lib_kwargs(kw, seed))
    if world > 1:
        cfg = _lib.shard_config(cfg, rank, world)
    return CudaEngine(cfg, "cuda:0")


def dev(a, dtype=np.uint32):
    a = np.ascontiguousarray(a, dtype=dtype)
    return torch.from_numpy(a.view(np.int32)).cuda()


def host(t):
    return t.cpu().numpy()


# ------------------------------------------------------------ golden: reference

@pytest.mark.parametrize("name", golden_names("inf_"))
def test_inference_matches_reference_kernels(name):
    g = load_golden(name)
    e = engine_for(SHAPES[name])
    lits = e.encode(dev(g["X"]))
    np.testing.assert_array_equal(host(lits).view(np.uint32), g["lits"])
    e.set_ta_state(g["ta"])
    np.testing.assert_array_equal(e.get_ta_state(), g["ta"])
    inc, ninc = e.include_mask()
    np.testing.assert_array_equal(host(inc).view(np.uint32), g["packed"])
    np.testing.assert_array_equal(host(ninc), g["ninc"])
    e.weights.copy_(torch.from_numpy(g["w"].astype(np.int32)))
    np.testing.assert_array_equal(host(e.infer(lits)), g["cs"].astype(np.int32))
    e.bias.copy_(torch.from_numpy(g["bias"].astype(np.int32)))
    np.testing.assert_array_equal(host(e.infer(lits)), g["cs_bias"].astype(np.int32))
    np.testing.assert_array_equal(host(e.transform(lits)), g["transform"])
    np.testing.assert_array_equal(host(e.transform_patchwise(lits)), g["transform_patchwise"])
    if "init_weights" in g:
        e.reset_weights()
        np.testing.assert_array_equal(host(e.weights), g["init_weights"].astype(np.int32))


@pytest.mark.parametrize("name", golden_names("tr_"))
def test_training_step_matches_reference_kernels(name):
    g = load_golden(name)
    e = engine_for(SHAPES[name])
    for i in range(g["e"].shape[0]):
        s = int(g["e"][i])
        lits = dev(g["lits"][i][s:s + 1])
        Y = dev(g["Y"][i][s:s + 1], np.int32)
        e.set_ta_state(g["ta"][i])
        e.weights.copy_(torch.from_numpy(g["w"][i].astype(np.int32)))
        e.patch_w.copy_(torch.from_numpy(g["pw"][i]))
        drop = dev(g["drop"][i])
        cs = e.train_eval(lits, 0, drop, add_bias=True)
        np.testing.assert_array_equal(host(cs)[0], g["cs"][i].astype(np.int32), err_msg=f"case {i}")
        sel = host(e.selection(1))
        np.testing.assert_array_equal(sel[0] >= 0, g["sel"][i] >= 0, err_msg=f"case {i} fired")
        sel_ref = dev(g["sel"][i][None, :], np.int32)
        e.train_update(cs, Y, lits, 0, drop, sel_override=sel_ref)
        np.testing.assert_array_equal(e.get_ta_state(), g["ta1"][i], err_msg=f"case {i} TA states")
        np.testing.assert_array_equal(host(e.weights), g["w1"][i].astype(np.int32), err_msg=f"case {i} weights")
        if g["pw"][i].shape[1] == 1:  # a single patch: the pick is forced
            np.testing.assert_array_equal(host(e.patch_w), g["pw1"][i], err_msg=f"case {i} patch weights")


# ------------------------------------------------------------ oracle parity

TRAIN_CASES = {
    "vanilla": (dict(number_of_clauses_per_class=12, T=15, s=4.0, dim=(40, 1, 1), n_classes=3, coalesced=False), 1),
    "coalesced_b1": (dict(number_of_clauses_per_class=40, T=30, s=6.0, dim=(50, 1, 1), n_classes=5), 1),
    "coalesced_b7": (dict(number_of_clauses_per_class=40, T=30, s=6.0, dim=(50, 1, 1), n_classes=5), 7),
    "coalesced_b40": (dict(number_of_clauses_per_class=33, T=30, s=6.0, dim=(70, 1, 1), n_classes=4), 40),
    "conv": (dict(number_of_clauses_per_class=30, T=20, s=3.0, dim=(8, 8, 1), n_classes=3, patch_dim=(4, 4)), 1),
    "conv_rgb_b3": (dict(number_of_clauses_per_class=20, T=20, s=5.0, dim=(7, 7, 3), n_classes=3,
                         patch_dim=(4, 3)), 3),
    "states4096": (dict(number_of_clauses_per_class=24, T=40, s=8.0, dim=(33, 1, 1), n_classes=4,
                        number_of_ta_states=4096), 2),
    "states16": (dict(number_of_clauses_per_class=24, T=10, s=2.0, dim=(33, 1, 1), n_classes=9,
                      number_of_ta_states=16), 1),
    "maxinc_nopol": (dict(number_of_clauses_per_class=24, T=10, s=3.0, dim=(40, 1, 1), n_classes=4,
                          max_included_literals=4, negative_polarity=False), 2),
    "noneg_noloc": (dict(number_of_clauses_per_class=16, T=10, s=3.0, dim=(8, 8, 1), n_classes=2,
                         patch_dim=(4, 4), encode_loc=False, append_negated=False), 1),
    "many_classes": (dict(number_of_clauses_per_class=70, T=50, s=10.0, dim=(30, 1, 1), n_classes=70), 2),
    # 289 patches: three 128-patch tiles of the sparse match, the last ragged
    "conv_tiles_b2": (dict(number_of_clauses_per_class=20, T=20, s=3.0, dim=(19, 19, 2), n_classes=3,
                           patch_dim=(3, 3)), 2),
    # 37 literal words: more include words per clause than lanes
    "conv_wide_b4": (dict(number_of_clauses_per_class=20, T=20, s=3.0, dim=(12, 12, 16), n_classes=3,
                          patch_dim=(6, 6)), 4),
    # every negative class selected (q = K - 1): about a dozen events per
    # clause and sample, so runs of 8, 16 and 32 Type Ib events form inside
    # the run windows (batch 40: one ragged window; batch 1:
    # the fused kernel; batch 12: the warp-per-clause kernel)
    "runs_b40": (dict(number_of_clauses_per_class=30, T=400, s=4.0, dim=(40, 1, 1), n_classes=24, q=23.0), 40),
    "runs_b12": (dict(number_of_clauses_per_class=30, T=400, s=4.0, dim=(40, 1, 1), n_classes=24, q=23.0), 12),
    "runs_b1": (dict(number_of_clauses_per_class=30, T=400, s=4.0, dim=(40, 1, 1), n_classes=40, q=39.0), 1),
    # negative-class selection drawn as a set (coalesced, K >= 32, K * Q <= 2):
    # the CTA-per-clause, warp-per-clause and fused kernels
    "qset_b40": (dict(number_of_clauses_per_class=12, T=40, s=5.0, dim=(40, 1, 1), n_classes=48, q=1.5), 40),
    "qset_b12": (dict(number_of_clauses_per_class=12, T=40, s=5.0, dim=(40, 1, 1), n_classes=33), 12),
    "qset_b1": (dict(number_of_clauses_per_class=12, T=40, s=5.0, dim=(40, 1, 1), n_classes=36, q=2.0), 1),
    "runs_conv_b3": (dict(number_of_clauses_per_class=16, T=300, s=6.0, dim=(8, 8, 1), n_classes=20, q=19.0,
                          patch_dim=(4, 4)), 3),
}


@pytest.mark.parametrize("case", sorted(TRAIN_CASES))
def test_training_matches_oracle(case):
    kw, bs = TRAIN_CASES[case]
    seed = 1234
    o = O.Oracle(**oracle_kwargs(kw, seed))
    e = engine_for(kw, seed)
    rng = np.random.default_rng(7)
    N = 24
    D = kw["dim"][0] * kw["dim"][1] * kw["dim"][2]
    X = (rng.random((N, D)) < 0.35).astype(np.uint32)
    labels = rng.integers(0, kw["n_classes"], N)
    Y = O.encode_Y_multiclass(labels, kw["n_classes"], kw["T"])
    lits_h = o.encode(X)
    lits = e.encode(dev(X))
    np.testing.assert_array_equal(host(lits).view(np.uint32), lits_h)
    ta, w = o.init_state(), o.init_weights()
    pw = np.zeros((o.C, o.P), np.int32)
    np.testing.assert_array_equal(host(e.weights), w)
    drop_h = (rng.random(o.C) < 0.1).astype(np.uint32) if case == "coalesced_b7" else None
    drop = None if drop_h is None else dev(drop_h)
    Yd = dev(Y, np.int32)
    t = 0
    for epoch in range(2):
        for i in range(0, N, bs):
            B = min(bs, N - i)
            cs_o, sel_o = o.train_batch(ta, w, pw, lits_h[i:i + B], Y[i:i + B], t, drop=drop_h)
            cs = e.train_eval(lits[i:i + B], t, drop, add_bias=True)
            np.testing.assert_array_equal(host(cs), cs_o, err_msg=f"class sums, batch at {i}")
            np.testing.assert_array_equal(host(e.selection(B)), sel_o, err_msg=f"patch picks, batch at {i}")
            e.train_update(cs, Yd[i:i + B], lits[i:i + B], t, drop)
            t += B
        np.testing.assert_array_equal(e.get_ta_state(), ta, err_msg=f"TA states after epoch {epoch}")
        np.testing.assert_array_equal(host(e.weights), w, err_msg=f"weights after epoch {epoch}")
        np.testing.assert_array_equal(host(e.patch_w), pw, err_msg=f"patch weights after epoch {epoch}")
    # something happened
    assert not np.array_equal(ta, o.init_state())
    # inference on the trained state
    np.testing.assert_array_equal(host(e.infer(lits)), o.infer(ta, w, lits_h))
    np.testing.assert_array_equal(host(e.transform(lits)), o.transform(ta, lits_h))
    np.testing.assert_array_equal(host(e.transform_patchwise(lits)), o.transform_patchwise(ta, lits_h))


CONVERGED_CASES = {
    # name: (model, batch, oracle/engine modes); batch 150 spans two feedback
    # chunks, batches of at most 32 take the warp-per-clause kernel
    "coalesced_b150": (dict(number_of_clauses_per_class=40, T=8, s=4.0, dim=(40, 1, 1), n_classes=5), 150, {}),
    "coalesced_b8": (dict(number_of_clauses_per_class=40, T=8, s=4.0, dim=(40, 1, 1), n_classes=5), 8, {}),
    "vanilla_b16": (dict(number_of_clauses_per_class=12, T=6, s=4.0, dim=(40, 1, 1), n_classes=4, coalesced=False),
                    16, {}),
    "pytm_rules_b20": (dict(number_of_clauses_per_class=40, T=8, s=4.0, dim=(40, 1, 1), n_classes=5), 20,
                       dict(one_negative=True)),
}


@pytest.mark.parametrize("case", sorted(CONVERGED_CASES))
def test_training_to_convergence_matches_oracle(case):
    """Twelve epochs on separable prototype data with a small T: the class sums
    saturate at +-T, so most (sample, class) pairs get a zero update
    probability (the feedback decides only the active pairs, and classes none
    of whose active samples fired take the parallel Type Ib path) while about
    a fifth of the clauses fire.  The engine must stay bit-exact with the
    oracle, and the run must reach that regime."""
    kw, bs, modes = CONVERGED_CASES[case]
    seed, N, D, K = 77, 300, 40, kw["n_classes"]
    o = O.Oracle(**oracle_kwargs(kw, seed), **modes)
    cfg = _lib.make_config(**lib_kwargs(kw, seed), **modes)
    e = CudaEngine(cfg, "cuda:0")
    rng = np.random.default_rng(5)
    proto = rng.random((K, D)) < 0.3
    labels = rng.integers(0, K, N)
    X = (proto[labels] ^ (rng.random((N, D)) < 0.03)).astype(np.uint32)
    Y = O.encode_Y_multiclass(labels, K, kw["T"])
    lits_h, lits, Yd = o.encode(X), e.encode(dev(X)), dev(Y, np.int32)
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    t = 0
    for epoch in range(12):
        inactive, fired = [], []
        for i in range(0, N, bs):
            B = min(bs, N - i)
            cs_o, sel_o = o.train_batch(ta, w, pw, lits_h[i:i + B], Y[i:i + B], t)
            cs = e.train_eval(lits[i:i + B], t, None, add_bias=True)
            np.testing.assert_array_equal(host(cs), cs_o, err_msg=f"class sums, epoch {epoch}, batch at {i}")
            e.train_update(cs, Yd[i:i + B], lits[i:i + B], t, None)
            t += B
            v = np.clip(cs_o, -kw["T"], kw["T"])
            inactive.append(np.mean((Y[i:i + B] - v) / (2.0 * Y[i:i + B]) <= 0))
            fired.append(np.mean(sel_o >= 0))
        np.testing.assert_array_equal(e.get_ta_state(), ta, err_msg=f"TA states after epoch {epoch}")
        np.testing.assert_array_equal(host(e.weights), w, err_msg=f"weights after epoch {epoch}")
        np.testing.assert_array_equal(host(e.patch_w), pw, err_msg=f"patch weights after epoch {epoch}")
    assert np.mean(inactive) > 0.7, "the run did not reach the converged regime"
    assert 0.05 < np.mean(fired) < 0.9


def test_sharded_engines_match_oracle():
    """Two clause shards on one GPU, class sums summed between the halves of
    each batch, equal the unsharded oracle (the multi-GPU schedule)."""
    kw = dict(number_of_clauses_per_class=50, T=30, s=5.0, dim=(40, 1, 1), n_classes=4)
    seed = 99
    o = O.Oracle(seed=seed, **{k: v for k, v in kw.items()})
    parts = [engine_for(kw, seed, r, 3) for r in range(3)]
    rng = np.random.default_rng(5)
    X = (rng.random((30, 40)) < 0.4).astype(np.uint32)
    Y = O.encode_Y_multiclass(rng.integers(0, 4, 30), 4, 30)
    lits_h = o.encode(X)
    ta, w = o.init_state(), o.init_weights()
    pw = np.zeros((o.C, o.P), np.int32)
    lits, Yd = dev(lits_h), dev(Y, np.int32)
    t = 0
    for i in range(0, 30, 5):
        o.train_batch(ta, w, pw, lits_h[i:i + 5], Y[i:i + 5], t)
        cs = sum(p.train_eval(lits[i:i + 5], t, None, add_bias=(r == 0)) for r, p in enumerate(parts))
        for p in parts:
            p.train_update(cs, Yd[i:i + 5], lits[i:i + 5], t, None)
        t += 5
    np.testing.assert_array_equal(np.concatenate([p.get_ta_state() for p in parts]), ta)
    np.testing.assert_array_equal(np.concatenate([host(p.weights) for p in parts]), w)


# ------------------------------------------------------------ full-size properties

def test_state_roundtrip_config5_size():
    """state_from_u32 -> state_to_u32 is the identity on a 13-plane model with
    W = 1024 (config-5 literal width, fewer clauses)."""
    kw = dict(number_of_clauses_per_class=512, T=20000, s=20.0, dim=(16384, 1, 1), n_classes=100,
              number_of_ta_states=4096)
    e = engine_for(kw)
    rng = np.random.default_rng(0)
    ta = rng.integers(0, e.cfg.state_top + 1, size=(e.C, e.L), dtype=np.uint32)
    e.set_ta_state(ta)
    np.testing.assert_array_equal(e.get_ta_state(), ta)
    inc, ninc = e.include_mask()
    np.testing.assert_array_equal(host(ninc), (ta > 2048).sum(1))


def test_infer_equals_transform_times_weights_config1_size():
    """Config-1 model (20000 clauses, W = 49): class sums == clause outputs x
    weights over non-empty clauses, on 2048 samples."""
    kw = dict(number_of_clauses_per_class=2000, T=50, s=10.0, dim=(28, 28, 1), n_classes=10, coalesced=False)
    e = engine_for(kw, seed=4)
    rng = np.random.default_rng(1)
    ta = rng.integers(0, 129, size=(e.C, e.L), dtype=np.uint32)
    X = (rng.random((2048, 784)) < 0.2).astype(np.uint32)
    lits = e.encode(dev(X))
    lh = host(lits).view(np.uint32)
    for c in range(e.C):  # each clause includes 1-3 literals true in some sample
        if c % 7 == 0:
            continue
        bits = np.unpackbits(lh[rng.integers(2048), 0].view(np.uint8), bitorder="little")[:e.L]
        ones = np.flatnonzero(bits)
        ta[c, rng.choice(ones, size=rng.integers(1, 4), replace=False)] = 200
    e.set_ta_state(ta)
    out = host(e.transform(lits)).astype(np.int64)
    cs = host(e.infer(lits)).astype(np.int64)
    nonempty = (ta > 128).any(1)
    W = host(e.weights).astype(np.int64)
    np.testing.assert_array_equal(cs, (out * nonempty[None, :]) @ W)
    assert 0 < out.mean() < 1


@pytest.mark.parametrize("case", ["vanilla", "coalesced_b1", "states4096", "states16", "maxinc_nopol",
                                  "many_classes", "drop", "conv", "conv_rgb_b3", "noneg_noloc", "runs_b1",
                                  "runs_conv_b3"])
def test_fused_batch1_matches_oracle(case):
    """ytm_train_fit_b1 (one fused launch per sample) == the oracle's
    per-sample loop."""
    kw, _ = TRAIN_CASES["coalesced_b1" if case == "drop" else case]
    seed = 4321
    o = O.Oracle(**oracle_kwargs(kw, seed))
    e = engine_for(kw, seed)
    rng = np.random.default_rng(8)
    N = 40
    D = kw["dim"][0] * kw["dim"][1] * kw["dim"][2]
    X = (rng.random((N, D)) < 0.35).astype(np.uint32)
    Y = O.encode_Y_multiclass(rng.integers(0, kw["n_classes"], N), kw["n_classes"], kw["T"])
    lits_h = o.encode(X)
    lits = dev(lits_h)
    drop_h = (rng.random(o.C) < 0.15).astype(np.uint32) if case == "drop" else None
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    t = 0
    for ep in range(3):
        t = o.fit(ta, w, pw, lits_h, Y, t, batch_size=1, drop=drop_h)
        e.train_fit_b1(lits, dev(Y, np.int32), ep * N, None if drop_h is None else dev(drop_h))
        np.testing.assert_array_equal(e.get_ta_state(), ta, err_msg=f"epoch {ep}")
        np.testing.assert_array_equal(host(e.weights), w)
        np.testing.assert_array_equal(host(e.patch_w), pw)
    assert not np.array_equal(ta, o.init_state())


@pytest.mark.parametrize("path", ["batch", "fused"])
def test_sample_counter_crossing_2_32(path):
    """Decisions key on the sample counter's high word: batches whose samples
    straddle t = 2^32 must match the oracle too."""
    kw = dict(number_of_clauses_per_class=30, T=20, s=4.0, dim=(40, 1, 1), n_classes=4)
    seed = 77
    o = O.Oracle(**oracle_kwargs(kw, seed))
    e = engine_for(kw, seed)
    rng = np.random.default_rng(3)
    X = (rng.random((12, 40)) < 0.4).astype(np.uint32)
    Y = O.encode_Y_multiclass(rng.integers(0, 4, 12), 4, 20)
    lits_h = o.encode(X)
    lits, Yd = dev(lits_h), dev(Y, np.int32)
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    t0 = 2 ** 32 - 5
    if path == "batch":
        o.train_batch(ta, w, pw, lits_h, Y, t0)
        cs = e.train_eval(lits, t0, None, add_bias=True)
        e.train_update(cs, Yd, lits, t0, None)
    else:
        o.fit(ta, w, pw, lits_h, Y, t0, batch_size=1)
        e.train_fit_b1(lits, Yd, t0, None)
    np.testing.assert_array_equal(e.get_ta_state(), ta)
    np.testing.assert_array_equal(host(e.weights), w)


@pytest.mark.parametrize("case,p_inc", [("conv_wide_b4", 0.02), ("conv_wide_b4", 0.3), ("conv_tiles_b2", 0.05),
                                        ("conv_tiles_b2", 0.0)])
def test_patch_match_on_random_states(case, p_inc):
    """Patch picks and class sums of one training batch from random TA
    states with a given share of included literals (dense and sparse include
    words, empty clauses, more include words than lanes)."""
    kw, bs = TRAIN_CASES[case]
    o = O.Oracle(**oracle_kwargs(kw, 5))
    e = engine_for(kw, 5)
    rng = np.random.default_rng(int(p_inc * 100) + 1)
    ta = np.where(rng.random((o.C, o.L)) < p_inc, rng.integers(o.half_state + 1, 2 * o.half_state, (o.C, o.L)),
                  rng.integers(0, o.half_state + 1, (o.C, o.L))).astype(np.uint32)
    ta[::7] = rng.integers(0, o.half_state + 1, (len(ta[::7]), o.L))  # every 7th clause empty
    e.set_ta_state(ta)
    D = kw["dim"][0] * kw["dim"][1] * kw["dim"][2]
    X = (rng.random((bs, D)) < 0.5).astype(np.uint32)
    lits_h = o.encode(X)
    Y = O.encode_Y_multiclass(rng.integers(0, kw["n_classes"], bs), kw["n_classes"], kw["T"])
    w, pw = o.init_weights(), np.zeros((o.C, o.P), np.int32)
    cs_o, sel_o = o.train_batch(ta.copy(), w, pw, lits_h, Y, 99, drop=None)
    cs = e.train_eval(dev(lits_h), 99, None, add_bias=True)
    np.testing.assert_array_equal(host(cs), cs_o)
    np.testing.assert_array_equal(host(e.selection(bs)), sel_o)
    assert (sel_o >= 0).any() and (sel_o < 0).any() if p_inc > 0 else (sel_o >= 0).all()
    # inference and transforms on the same states and samples (any-patch match)
    ta_now = e.get_ta_state()
    X2 = (rng.random((37, D)) < 0.5).astype(np.uint32)
    l2 = o.encode(X2)
    np.testing.assert_array_equal(host(e.infer(dev(l2))), o.infer(ta_now, host(e.weights), l2))
    np.testing.assert_array_equal(host(e.transform(dev(l2))), o.transform(ta_now, l2))


def test_type1b_runs_take_the_run_path():
    """On a case with long Type Ib runs the feedback's device counters show
    run pieces (four Philox calls per word for a piece of 8 to 64 events
    instead of one per event), and the state still equals the oracle's."""
    kw, bs = TRAIN_CASES["runs_b40"]
    o = O.Oracle(**oracle_kwargs(kw, 5))
    e = engine_for(kw, 5)
    rng = np.random.default_rng(11)
    X = (rng.random((40, 40)) < 0.35).astype(np.uint32)
    Y = O.encode_Y_multiclass(rng.integers(0, kw["n_classes"], 40), kw["n_classes"], kw["T"])
    lits_h = o.encode(X)
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    lits, Yd = dev(lits_h), dev(Y, np.int32)
    ctr = torch.zeros(6, dtype=torch.int64, device="cuda")
    for t in (0, 40):
        o.train_batch(ta, w, pw, lits_h, Y, t)
        cs = e.train_eval(lits, t, None, add_bias=True)
        e.train_update(cs, Yd, lits, t, None, counters=ctr)
    np.testing.assert_array_equal(e.get_ta_state(), ta)
    calls, events = int(ctr[1]), int(ctr[3])
    assert events > 0 and calls < 0.75 * events * o.W, (calls, events)


@pytest.mark.parametrize("K,bs", [(24, 150), (300, 100)])
def test_type1b_runs_over_chunks(K, bs):
    """Runs inside their windows when a batch spans several feedback chunks:
    24 classes, batch 150 (128-sample windows: chunks of 128 and 22); 300
    classes, batch 100 (above 256 classes the windows and chunks are 64
    samples: 64 and 36)."""
    kw = dict(number_of_clauses_per_class=20 if K < 100 else 6, T=400, s=4.0, dim=(40, 1, 1), n_classes=K,
              q=float(K - 1))
    o = O.Oracle(**oracle_kwargs(kw, 8))
    e = engine_for(kw, 8)
    rng = np.random.default_rng(13)
    N = 2 * bs
    X = (rng.random((N, 40)) < 0.35).astype(np.uint32)
    Y = O.encode_Y_multiclass(rng.integers(0, K, N), K, kw["T"])
    lits_h = o.encode(X)
    lits, Yd = dev(lits_h), dev(Y, np.int32)
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    for i in range(0, N, bs):
        o.train_batch(ta, w, pw, lits_h[i:i + bs], Y[i:i + bs], i)
        cs = e.train_eval(lits[i:i + bs], i, None, add_bias=True)
        e.train_update(cs, Yd[i:i + bs], lits[i:i + bs], i, None)
    np.testing.assert_array_equal(e.get_ta_state(), ta)
    np.testing.assert_array_equal(host(e.weights), w)
