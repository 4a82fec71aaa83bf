"""ytm_infer_noalloc: inference for callers that cannot allocate device memory
(an embedding runtime that hands out all device memory itself, or a service
that forbids allocation after start-up).  It must give exactly what ytm_infer gives, call
after call, although all calls share one fixed scratch array.

Named test_zz_* so that pytest collects it last."""
import ctypes as ct

import numpy as np
import pytest
import torch

from ytm_b200 import _lib
from ytm_b200.engine import CudaEngine

pytestmark = pytest.mark.gpu


def _p(t):
    return ct.c_void_p(t.data_ptr())


def _model(seed, patch_dim=(24, 24), count_empty=False):
    cfg = _lib.make_config(clauses_per_class=300, T=50, s=10.0, dim=(28, 28, 1), n_classes=10, patch_dim=patch_dim,
                           seed=seed, count_empty=count_empty)
    eng = CudaEngine(cfg, "cuda:0")
    rng = np.random.default_rng(seed)
    half = cfg.number_of_ta_states // 2
    ta = rng.integers(0, half + 1, size=(eng.C, eng.L), dtype=np.uint32)
    for c in range(eng.C):  # a few includes per clause so that some clauses fire
        if c % 9:
            ta[c, rng.choice(eng.L, size=rng.integers(1, 3), replace=False)] = half + 5
    eng.set_ta_state(ta)
    eng.weights.copy_(torch.from_numpy(rng.integers(-20, 21, size=(eng.C, eng.K)).astype(np.int32)))
    eng.bias.copy_(torch.from_numpy(rng.integers(-3, 4, size=eng.K).astype(np.int32)))
    return eng, rng


def _noalloc(eng, lits):
    lib = _lib.load()
    N = lits.shape[0]
    cs = torch.full((N, eng.K), 12345, dtype=torch.int32, device=eng.device)
    stream = ct.c_void_p(torch.cuda.current_stream(eng.device).cuda_stream)
    rc = lib.ytm_infer_noalloc(ct.byref(eng.cfg), _p(eng.state), _p(eng.weights), _p(eng.bias), _p(lits), N,
                               _p(cs), stream)
    _lib.check(rc, "ytm_infer_noalloc")
    return cs


@pytest.mark.parametrize("patch_dim,count_empty", [((24, 24), False), (None, True)])
def test_noalloc_matches_workspace_inference_twice(patch_dim, count_empty):
    """Convolutional model (25 patches), and a single-patch model that counts
    empty clauses (pytm's inference rule)."""
    eng, rng = _model(21, patch_dim, count_empty)
    for n in (96, 40):  # second call smaller: stale scratch from the first must not leak in
        X = (rng.random((n, 784)) < 0.3).astype(np.uint32)
        lits = eng.encode(torch.from_numpy(X.view(np.int32)).cuda())
        want = eng.infer(lits).cpu().numpy()
        got = _noalloc(eng, lits).cpu().numpy()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got, want)  # integer class sums: exact
        assert np.abs(want).sum() > 0


def test_noalloc_rejects_oversize_call():
    eng, _ = _model(5)
    lib = _lib.load()
    per_sample = ((eng.C + 31) // 32) * 4
    N = (16 << 20) // per_sample + 1
    lits = torch.zeros((1, eng.P, eng.W), dtype=torch.int32, device=eng.device)
    cs = torch.zeros((1, eng.K), dtype=torch.int32, device=eng.device)
    # the size check fails before any launch, so the 1-row buffers are never read
    rc = lib.ytm_infer_noalloc(ct.byref(eng.cfg), _p(eng.state), _p(eng.weights), None, _p(lits), N, _p(cs),
                               None)
    assert rc == 1
    assert b"fixed scratch" in lib.ytm_last_error()
