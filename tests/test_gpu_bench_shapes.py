"""GPU parity at the benchmark configurations' exact shapes (literal width,
patch grid, state planes, class count, batch), with fewer clauses and samples
so that the CPU oracle stays fast.  These shapes reach code paths the small
parity cases do not:

* config 4 (dim 32x32x24, 10x10 patches: W = 153, P = 529): the sparse patch
  match with more than 48 KB of dynamic shared memory, and the fused batch-1
  kernel's convolutional scan at that width;
* config 5 (16384 features, 4096 states = 13 planes, 100 classes, batch 128):
  the 256-thread feedback CTAs over W = 1024 with a 64-sample chunk (two
  chunks per batch);
* config 1 at full size (20,000 clauses, batch 1 fused path, 313 blocks);
* config 3 (28x28, 10x10 patches: W = 9, P = 361) through the fused path.

Everything is compared bit for bit: TA states, weights, patch weights, class
sums, patch picks, then inference and transforms on the trained state."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import lib_kwargs, oracle_kwargs
from ytm_b200 import _lib, synthetic
from ytm_b200.engine import CudaEngine

pytestmark = pytest.mark.gpu


def dev(a, dtype=np.uint32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype).view(np.int32)).cuda()


def host(t):
    return t.cpu().numpy()


def pair(kw, seed):
    o = O.Oracle(**oracle_kwargs(kw, seed))
    e = CudaEngine(_lib.make_config(**lib_kwargs(kw, seed)), "cuda:0")
    return o, e


def model(name, clauses, **over):
    kw = dict(synthetic.MODELS[name])
    kw["number_of_clauses_per_class"] = clauses
    kw.update(over)
    return kw


def check_inference(o, e, ta, lits_h, n=None):
    lits_h = lits_h[:n] if n else lits_h
    lits = dev(lits_h)
    w = host(e.weights)
    np.testing.assert_array_equal(host(e.infer(lits)), o.infer(ta, w, lits_h), err_msg="class sums")
    np.testing.assert_array_equal(host(e.transform(lits)), o.transform(ta, lits_h), err_msg="transform")


def train_batches(o, e, lits_h, Y, bs, epochs=1):
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    np.testing.assert_array_equal(host(e.weights), w)
    lits, Yd = dev(lits_h), dev(Y, np.int32)
    N, t = lits_h.shape[0], 0
    for ep in range(epochs):
        for i in range(0, N, bs):
            B = min(bs, N - i)
            cs_o, sel_o = o.train_batch(ta, w, pw, lits_h[i:i + B], Y[i:i + B], t)
            cs = e.train_eval(lits[i:i + B], t, None, add_bias=True)
            np.testing.assert_array_equal(host(cs), cs_o, err_msg=f"class sums, epoch {ep}, batch at {i}")
            np.testing.assert_array_equal(host(e.selection(B)), sel_o, err_msg=f"picks, epoch {ep}, batch at {i}")
            e.train_update(cs, Yd[i:i + B], lits[i:i + B], t, None)
            t += B
        np.testing.assert_array_equal(host(e.weights), w, err_msg=f"weights after epoch {ep}")
        np.testing.assert_array_equal(e.get_ta_state(), ta, err_msg=f"TA states after epoch {ep}")
        np.testing.assert_array_equal(host(e.patch_w), pw, err_msg=f"patch weights after epoch {ep}")
    assert not np.array_equal(ta, o.init_state())
    return ta


def train_fused(o, e, lits_h, Y, epochs=1):
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    lits, Yd = dev(lits_h), dev(Y, np.int32)
    N, t = lits_h.shape[0], 0
    for ep in range(epochs):
        t = o.fit(ta, w, pw, lits_h, Y, t, batch_size=1)
        e.train_fit_b1(lits, Yd, ep * N, None)
        np.testing.assert_array_equal(host(e.weights), w, err_msg=f"weights after epoch {ep}")
        np.testing.assert_array_equal(e.get_ta_state(), ta, err_msg=f"TA states after epoch {ep}")
        np.testing.assert_array_equal(host(e.patch_w), pw, err_msg=f"patch weights after epoch {ep}")
    assert not np.array_equal(ta, o.init_state())
    return ta


def data(name, kw, n, seed):
    X, y = synthetic.make(name, n, seed=seed)
    return X, O.encode_Y_multiclass(y, kw["n_classes"], kw["T"])


# -------------------------------------------------------------- config 4 width

@pytest.mark.parametrize("bs", [1, 4])
def test_config4_shape_batches(bs):
    kw = model("c4", 64)
    o, e = pair(kw, 2024)
    assert (o.W, o.P) == (153, 529)
    X, Y = data("c4", kw, 8, 11)
    lits_h = o.encode(X)
    np.testing.assert_array_equal(host(e.encode(dev(X))).view(np.uint32), lits_h)
    ta = train_batches(o, e, lits_h, Y, bs)
    check_inference(o, e, ta, lits_h)


def test_config4_shape_fused_batch1():
    kw = model("c4", 64)
    o, e = pair(kw, 77)
    X, Y = data("c4", kw, 6, 12)
    lits_h = o.encode(X)
    ta = train_fused(o, e, lits_h, Y, epochs=2)
    check_inference(o, e, ta, lits_h)


# -------------------------------------------------------------- config 5 width

def test_config5_shape_two_chunks():
    kw = model("c5", 256)
    o, e = pair(kw, 5005)
    assert (o.W, o.K, e.NB) == (1024, 100, 13)
    X, Y = data("c5", kw, 256, 13)
    lits_h = o.encode(X)
    ta = train_batches(o, e, lits_h, Y, 128)
    check_inference(o, e, ta, lits_h, 64)


def test_config5_shape_ragged_small_batch():
    """A 40-sample batch (one ragged chunk) and a 24-sample batch (the
    warp-per-clause feedback) at config-5 width."""
    kw = model("c5", 96)
    o, e = pair(kw, 6006)
    X, Y = data("c5", kw, 64, 14)
    lits_h = o.encode(X)
    ta = train_batches(o, e, lits_h, Y, 40)
    check_inference(o, e, ta, lits_h, 32)


# -------------------------------------------------------------- config 1 size

def test_config1_full_size_fused():
    kw = dict(synthetic.MODELS["c1"])
    o, e = pair(kw, 42)
    assert o.C == 20000
    X, Y = data("c1", kw, 50, 15)
    lits_h = o.encode(X)
    ta = train_fused(o, e, lits_h, Y)
    check_inference(o, e, ta, lits_h)


# -------------------------------------------------------------- config 3 shape

def test_config3_shape_fused():
    kw = model("c3", 96)
    o, e = pair(kw, 31)
    assert (o.W, o.P) == (9, 361)
    X, Y = data("c3", kw, 30, 16)
    lits_h = o.encode(X)
    ta = train_fused(o, e, lits_h, Y, epochs=2)
    check_inference(o, e, ta, lits_h)
