"""GPU tests of the reference-facing API (ytm_b200.cutm mirrors
src/cutm/{multiclass,multioutput,base}.py): fit/predict/score, encode,
transforms, getters, state dict and pickle, against the oracle."""
import io
import lzma
import pickle

import numpy as np
import pytest

from oracle import oracle as O
from ytm_b200 import synthetic
from ytm_b200.cutm import MultiClassTM, MultiOutputTM

pytestmark = pytest.mark.gpu

KW = dict(number_of_clauses_per_class=40, T=20, s=4.0, dim=(8, 8, 1), n_classes=3, patch_dim=(5, 5), seed=3)


def data(n=60, seed=0):
    rng = np.random.default_rng(seed)
    return (rng.random((n, 64)) < 0.35).astype(np.uint32), rng.integers(0, 3, n).astype(np.uint32)


@pytest.mark.parametrize("bs", [1, 8])
def test_multiclass_fit_predict_matches_oracle(bs):
    X, y = data()
    tm = MultiClassTM(**KW)
    assert (tm.number_of_clauses, tm.number_of_patches) == (40, 16)
    enc = tm.encode(X)
    tm.fit(enc, y, is_X_encoded=True, batch_size=bs, block_size=16)
    tm.fit(X, y, batch_size=bs)  # raw inputs, encoded on the device
    o = O.Oracle(**KW)
    lits = o.encode(X)
    np.testing.assert_array_equal(enc, lits)
    Y = O.encode_Y_multiclass(y, 3, KW["T"])
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    t = o.fit(ta, w, pw, lits, Y, 0, batch_size=bs)
    o.fit(ta, w, pw, lits, Y, t, batch_size=bs)
    np.testing.assert_array_equal(tm.get_ta_state(), ta)
    np.testing.assert_array_equal(tm.get_weights(), w.astype(np.float32))
    np.testing.assert_array_equal(tm.get_patch_weights(), pw)
    np.testing.assert_array_equal(tm.get_literals(), (ta > 128).astype(np.uint32))
    preds, cs = tm.predict(X)
    assert cs.dtype == np.float32 and preds.shape == (60,)
    np.testing.assert_array_equal(cs, o.infer(ta, w, lits).astype(np.float32))
    np.testing.assert_array_equal(preds, np.argmax(cs, axis=1))
    np.testing.assert_array_equal(tm.transform(X), o.transform(ta, lits))
    np.testing.assert_array_equal(tm.transform_patchwise(enc, is_X_encoded=True), o.transform_patchwise(ta, lits))


def test_non_coalesced_getter_shapes():
    tm = MultiClassTM(number_of_clauses_per_class=10, T=5, s=3.0, dim=(16, 1, 1), n_classes=4, coalesced=False,
                      seed=1)
    assert tm.get_ta_state().shape == (4, 10, 32)
    assert tm.get_weights().shape == (4, 10, 4)
    assert tm.get_patch_weights().shape == (4, 10, 1)
    assert tm.get_bias_weights().shape == (4,)


def test_multioutput_matches_oracle():
    rng = np.random.default_rng(2)
    X = (rng.random((40, 64)) < 0.35).astype(np.uint32)
    Ym = (rng.random((40, 3)) < 0.4).astype(np.uint32)
    tm = MultiOutputTM(**KW)
    tm.fit(X, Ym, batch_size=4)
    o = O.Oracle(**KW)
    lits = o.encode(X)
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    o.fit(ta, w, pw, lits, O.encode_Y_multioutput(Ym, KW["T"]), 0, batch_size=4)
    np.testing.assert_array_equal(tm.get_ta_state(), ta)
    preds, cs = tm.predict(X)
    np.testing.assert_array_equal(cs, o.infer(ta, w, lits).astype(np.float32))
    np.testing.assert_array_equal(preds, (cs >= 0).astype(np.uint32))


def test_pickle_lzma_roundtrip_and_continue():
    """Scripts save models with pickle + LZMAFile (pneumonia_mnist.py:119-120)."""
    X, y = data()
    tm = MultiClassTM(**KW)
    tm.fit(X[:30], y[:30], batch_size=2)
    buf = io.BytesIO()
    with lzma.LZMAFile(buf, "wb") as f:
        pickle.dump(tm, f)
    buf.seek(0)
    with lzma.LZMAFile(buf, "rb") as f:
        tm2 = pickle.load(f)
    np.testing.assert_array_equal(tm2.get_ta_state(), tm.get_ta_state())
    np.testing.assert_array_equal(tm2.predict(X)[1], tm.predict(X)[1])
    tm.fit(X[30:], y[30:], batch_size=2)
    tm2.fit(X[30:], y[30:], batch_size=2)  # the sample counter travels: same decisions
    np.testing.assert_array_equal(tm2.get_ta_state(), tm.get_ta_state())


def test_state_dict_in_reference_layout():
    tm = MultiClassTM(**KW)
    sd = tm.get_state_dict()
    assert sd["ta_state"].dtype == np.uint32 and sd["ta_state"].shape == (40 * tm.number_of_literals,)
    assert sd["clause_weights"].dtype == np.float32 and sd["patch_weights"].dtype == np.int32
    rng = np.random.default_rng(0)
    sd["ta_state"] = rng.integers(0, 257, sd["ta_state"].shape).astype(np.uint32)
    tm.load_state_dict({"state": sd})
    np.testing.assert_array_equal(tm.get_state_dict()["ta_state"], sd["ta_state"])
    sd["ta_state"][0] = 10_000
    with pytest.raises(ValueError):
        tm.load_state_dict({"state": sd})


def test_learns_config1_like_data():
    """Vanilla TM on prototype data (config 1 distribution, fewer clauses):
    one epoch at batch 1 gives high test accuracy."""
    X, y = synthetic.prototypes(3000, seed=11)
    tm = MultiClassTM(number_of_clauses_per_class=100, T=50, s=10.0, dim=(28, 28, 1), n_classes=10,
                      coalesced=False, seed=5)
    tm.fit(X[:2000], y[:2000])
    acc = (tm.predict(X[2000:])[0] == y[2000:]).mean()
    assert acc > 0.9, acc


def test_bad_inputs_raise():
    tm = MultiClassTM(**KW)
    with pytest.raises(AssertionError):
        tm.encode(np.zeros((3, 64), np.int64))
    with pytest.raises(AssertionError):
        tm.fit(np.zeros((3, 64), np.uint32), np.zeros((3, 2), np.uint32))
    with pytest.raises(NotImplementedError):
        MultiClassTM(bias=True, **KW)


def _binarize_rgb(X, levels):
    """ThermometerBinarizer(levels).binarize_rgb, tm_utils/binarizer.py:17-21."""
    thr = (np.arange(1, levels + 1) * 255 / (levels + 1)).reshape(1, 1, 1, 1, levels)
    out = (X[:, :, :, :, None] >= thr).reshape(X.shape[0], X.shape[1], X.shape[2], X.shape[3] * levels)
    return np.asarray(out, dtype=np.uint32)


@pytest.mark.parametrize("levels,ch,patch", [(8, 3, (5, 5)), (4, 1, (9, 9)), (3, 2, (4, 6))])
def test_thermometer_encoding_on_device(levels, ch, patch):
    rng = np.random.default_rng(levels)
    imgs = rng.integers(0, 256, size=(7, 9, 9, ch), dtype=np.uint8)
    imgs[0, 0, 0, :] = 255
    imgs[0, 0, 1, :] = 0
    tm = MultiClassTM(number_of_clauses_per_class=8, T=10, s=3.0, dim=(9, 9, ch * levels), n_classes=2,
                      patch_dim=patch, seed=1)
    want = tm.encode(_binarize_rgb(imgs, levels).reshape(7, -1))
    np.testing.assert_array_equal(tm.encode_thermometer(imgs, levels), want)
    o = O.Oracle(number_of_clauses_per_class=8, T=10, s=3.0, dim=(9, 9, ch * levels), n_classes=2, patch_dim=patch)
    np.testing.assert_array_equal(want, o.encode(_binarize_rgb(imgs, levels).reshape(7, -1)))
    lits = tm.encode_thermometer(imgs, levels, on_device=True)
    tm.fit(lits, np.array([0, 1, 0, 1, 1, 0, 1]), is_X_encoded=True)
    assert tm.predict(lits, is_X_encoded=True)[1].shape == (7, 2)


def test_pytm_front_end_matches_oracle_pytm_rules():
    """ytm_b200.pytm.BaseTM follows pytm's rules (one other class per sample,
    true class first, empty clauses counted at prediction) — checked bit for
    bit against the oracle run in the same mode."""
    from ytm_b200.pytm import BaseTM
    rng = np.random.default_rng(4)
    X = rng.random((80, 30)) < 0.4
    y = rng.integers(0, 5, 80)
    tm = BaseTM(n_clause=40, T=12, s=3.0, q=1.0, n_class=5, dim=(30, 1, 1), n_ta_states=64, seed=9)
    assert tm.states.dtype == np.uint8 and (tm.states == 31).all()
    tm.fit(X, y)
    tm.fit(X, y, shuffle=True)
    o = O.Oracle(number_of_clauses_per_class=40, T=12, s=3.0, dim=(30, 1, 1), n_classes=5, number_of_ta_states=63,
                 seed=9, one_negative=True, count_empty=True)
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, 1), np.int32)
    lits = o.encode(X.astype(np.uint32))
    Y = O.encode_Y_multiclass(y, 5, 12)
    t = o.fit(ta, w, pw, lits, Y, 0)
    iota = np.arange(80)
    np.random.default_rng(9).shuffle(iota)
    o.fit(ta, w, pw, lits[iota], Y[iota], t)
    np.testing.assert_array_equal(tm.states, ta.astype(np.uint8))
    np.testing.assert_array_equal(tm.weights, w.astype(np.float32))
    preds, cs = tm.predict(X, return_cs=True)
    np.testing.assert_array_equal(cs, o.infer(ta, w, lits).astype(np.float32))
    assert (ta != 31).any()  # training moved the states


def test_empty_and_single_sample_inputs():
    tm = MultiClassTM(**KW)
    X0 = np.zeros((0, 64), np.uint32)
    assert tm.encode(X0).shape == (0, tm.number_of_patches, tm.number_of_literal_chunks)
    preds, cs = tm.predict(X0)
    assert preds.shape == (0,) and cs.shape == (0, 3)
    tm.fit(X0, np.zeros(0, np.uint32))
    assert tm.sample_counter == 0
    X1, y1 = data(1)
    tm.fit(X1, y1)
    tm.fit(X1, y1, batch_size=4)
    assert tm.sample_counter == 2
    assert tm.transform(X1).shape == (1, tm.number_of_clauses)
    assert tm.transform_patchwise(X1).shape == (1, tm.number_of_clauses, tm.number_of_patches)


def test_match_early_exit_counts_and_parity():
    """The dense match tiles stop once every (sample, clause) pair of a tile has
    a violation: clauses 0..127 include a literal that is 0 in every sample
    and sits in the first 32-word chunk, so their tiles stop after one of the
    four chunks; the other clauses match often and run to the end.  Class sums
    equal the oracle's, and the device counters show the skipped chunks."""
    import ctypes as ct

    import torch
    from ytm_b200 import _lib
    kw = dict(number_of_clauses_per_class=200, T=20, s=4.0, dim=(2048, 1, 1), n_classes=4, seed=5)
    tm = MultiClassTM(**kw)
    rng = np.random.default_rng(1)
    N = 200
    X = (rng.random((N, 2048)) < 0.9).astype(np.uint32)
    X[:, :32] = 0
    C, L = tm.engine.C, 2 * 2048
    assert C == 200
    ta = rng.integers(0, 128, size=(C, L), dtype=np.uint32)  # 8-bit states: include at >= 128
    for c in range(C):
        if c < 128:
            ta[c, c % 32] = 200  # x_(c mod 32), always 0: violated in word 0
        else:
            ta[c, rng.integers(100, 1024, size=2)] = 200  # mostly 1
    tm.engine.set_ta_state(ta)
    tm._model_version += 1
    lib = _lib.load()
    out = (ct.c_uint64 * 2)()
    st = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.ytm_match_counters(out, st))
    _, cs = tm.predict(X)
    _lib.check(lib.ytm_match_counters(out, st))
    tiles, chunks = int(out[0]), int(out[1])
    o = O.Oracle(**kw)
    np.testing.assert_array_equal(cs, o.infer(ta, o.init_weights(), o.encode(X)).astype(np.float32))
    row_tiles, clause_tiles = -(-N // 64), -(-C // 64)
    assert tiles == row_tiles * clause_tiles
    # clause tiles 0 and 1 hold clauses 0..127: one chunk each; the rest run all 4
    assert chunks == row_tiles * (2 * 1 + (clause_tiles - 2) * 4)
