"""Convolutional models fed packed bit images (input_images = 1): the patch
literal words are formed on the fly inside the match, feedback and fused
batch-1 kernels instead of being read from the reference's per-patch literal
tensor (encode_batch, kernel.cu:76-152).  Everything must be bit-identical to
the oracle fed that tensor."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import bits_of, lib_kwargs, oracle_kwargs
from tests.test_gpu_parity import TRAIN_CASES
from ytm_b200 import _lib, synthetic
from ytm_b200.engine import CudaEngine

pytestmark = pytest.mark.gpu

SHAPES = {
    "conv": dict(dim=(8, 8, 1), patch_dim=(4, 4)),
    "rgb": dict(dim=(7, 7, 3), patch_dim=(4, 3)),
    "nonsq": dict(dim=(9, 7, 2), patch_dim=(4, 4)),
    "noloc": dict(dim=(8, 8, 1), patch_dim=(4, 4), encode_loc=False),
    "noneg_noloc": dict(dim=(8, 8, 1), patch_dim=(4, 4), encode_loc=False, append_negated=False),
    "noneg": dict(dim=(12, 10, 3), patch_dim=(5, 3), append_negated=False),
    "c3": dict(dim=(28, 28, 1), patch_dim=(10, 10)),
    "c4": dict(dim=(32, 32, 24), patch_dim=(10, 10)),
}


def dev(a, dtype=np.uint32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype).view(np.int32)).cuda()


def host(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_image_literals_are_the_encoded_literals(shape):
    """One clause per literal, each including only its own literal: the
    per-patch clause outputs from bit images are then exactly the literal bits
    of every patch, which must equal ytm_encode's (== the reference's
    encode_batch fixtures, checked elsewhere)."""
    geo = SHAPES[shape]
    probe = _lib.make_config(clauses_per_class=1, T=10, s=3.0, n_classes=2, **geo)
    L = probe.literals
    cfg = _lib.make_config(clauses_per_class=L, T=10, s=3.0, n_classes=2, **geo)
    e = CudaEngine(cfg, "cuda:0")
    ta = np.zeros((L, L), np.uint32)
    ta[np.arange(L), np.arange(L)] = cfg.number_of_ta_states // 2 + 1
    e.set_ta_state(ta)
    rng = np.random.default_rng(3)
    D = geo["dim"][0] * geo["dim"][1] * geo["dim"][2]
    X = (rng.random((3, D)) < 0.4).astype(np.uint32)
    lits = e.encode(dev(X))
    img = e.pack_images(dev(X))
    assert img.shape == (3, cfg.image_words)
    want = bits_of(host(lits).view(np.uint32), L)  # [N, P, L]
    got = host(e.transform_patchwise(img)).view(np.uint32)  # [N, C=L, P]
    np.testing.assert_array_equal(got.transpose(0, 2, 1), want)
    np.testing.assert_array_equal(host(e.transform_patchwise(lits)), host(e.transform_patchwise(img)))


def test_thermometer_images_match_thermometer_literals():
    kw = dict(synthetic.MODELS["c4"], number_of_clauses_per_class=32)
    cfg = _lib.make_config(**lib_kwargs(kw, 1))
    e = CudaEngine(cfg, "cuda:0")
    rng = np.random.default_rng(9)
    raw = torch.from_numpy(rng.integers(0, 256, (5, 32 * 32 * 3), dtype=np.uint8)).cuda()
    lits = e.encode_thermometer(raw, 8)
    img = e.pack_images_thermometer(raw, 8)
    ta = np.where(rng.random((e.C, e.L)) < 0.002, 200, 50).astype(np.uint32)
    e.set_ta_state(ta)
    np.testing.assert_array_equal(host(e.infer(img)), host(e.infer(lits)))
    np.testing.assert_array_equal(host(e.transform(img)), host(e.transform(lits)))


CASES = {name: TRAIN_CASES[name] for name in ("conv", "conv_rgb_b3", "noneg_noloc", "conv_tiles_b2", "conv_wide_b4")}
CASES["c4_b2"] = (dict(synthetic.MODELS["c4"], number_of_clauses_per_class=48), 2)
CASES["c3_b1"] = (dict(synthetic.MODELS["c3"], number_of_clauses_per_class=40), 1)


def _data(kw, N, seed):
    rng = np.random.default_rng(seed)
    D = kw["dim"][0] * kw["dim"][1] * kw["dim"][2]
    X = (rng.random((N, D)) < 0.3).astype(np.uint32)
    Y = O.encode_Y_multiclass(rng.integers(0, kw["n_classes"], N), kw["n_classes"], kw["T"])
    return X, Y


@pytest.mark.parametrize("case", sorted(CASES))
def test_training_from_images_matches_oracle(case):
    kw, bs = CASES[case]
    seed = 4242
    o = O.Oracle(**oracle_kwargs(kw, seed))
    e = CudaEngine(_lib.make_config(**lib_kwargs(kw, seed)), "cuda:0")
    X, Y = _data(kw, 12, 21)
    lits_h = o.encode(X)
    img = e.pack_images(dev(X))
    Yd = dev(Y, np.int32)
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    t = 0
    for ep in range(2):
        for i in range(0, len(X), bs):
            B = min(bs, len(X) - i)
            cs_o, sel_o = o.train_batch(ta, w, pw, lits_h[i:i + B], Y[i:i + B], t)
            cs = e.train_eval(img[i:i + B], t, None, add_bias=True)
            np.testing.assert_array_equal(host(cs), cs_o, err_msg=f"class sums, batch at {i}")
            np.testing.assert_array_equal(host(e.selection(B)), sel_o, err_msg=f"picks, batch at {i}")
            e.train_update(cs, Yd[i:i + B], img[i:i + B], t, None)
            t += B
        np.testing.assert_array_equal(e.get_ta_state(), ta, err_msg=f"TA states after epoch {ep}")
        np.testing.assert_array_equal(host(e.weights), w)
        np.testing.assert_array_equal(host(e.patch_w), pw)
    assert not np.array_equal(ta, o.init_state())
    np.testing.assert_array_equal(host(e.infer(img)), o.infer(ta, w, lits_h))
    np.testing.assert_array_equal(host(e.transform(img)), o.transform(ta, lits_h))


@pytest.mark.parametrize("case", ["conv", "conv_rgb_b3", "noneg_noloc", "c3_b1"])
def test_fused_batch1_from_images_matches_oracle(case):
    kw, _ = CASES[case]
    seed = 99
    o = O.Oracle(**oracle_kwargs(kw, seed))
    e = CudaEngine(_lib.make_config(**lib_kwargs(kw, seed)), "cuda:0")
    X, Y = _data(kw, 25, 5)
    lits_h = o.encode(X)
    img = e.pack_images(dev(X))
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    for ep in range(2):
        o.fit(ta, w, pw, lits_h, Y, ep * len(X), batch_size=1)
        e.train_fit_b1(img, dev(Y, np.int32), ep * len(X), None)
        np.testing.assert_array_equal(e.get_ta_state(), ta, err_msg=f"epoch {ep}")
        np.testing.assert_array_equal(host(e.weights), w)
        np.testing.assert_array_equal(host(e.patch_w), pw)
    assert not np.array_equal(ta, o.init_state())


def test_api_conv_fit_uses_images():
    """MultiClassTM feeds convolutional models packed bit images; results
    equal training on encoded literals (is_X_encoded=True)."""
    from ytm_b200.cutm import MultiClassTM
    kw = dict(number_of_clauses_per_class=30, T=20, s=3.0, dim=(10, 10, 2), n_classes=3, patch_dim=(4, 4))
    X, Y = _data(dict(kw), 40, 8)
    y = Y.argmax(1)
    a = MultiClassTM(seed=5, **kw)
    b = MultiClassTM(seed=5, **kw)
    assert a._input_device(X).dim() == 2
    a.fit(X, y, batch_size=4)
    b.fit(b.encode(X), y, is_X_encoded=True, batch_size=4)
    np.testing.assert_array_equal(a.get_ta_state(), b.get_ta_state())
    np.testing.assert_array_equal(a.predict(X)[1], b.predict(b.encode(X), is_X_encoded=True)[1])
    a.fit(X, y, batch_size=1)
    b.fit(b.encode(X), y, is_X_encoded=True, batch_size=1)
    np.testing.assert_array_equal(a.get_ta_state(), b.get_ta_state())
