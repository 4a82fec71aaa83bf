"""CPU tests of the C ABI: the library loads, exports exactly what
include/ytm.h declares, and derives the same sizes as the oracle."""
import os
import re

import pytest

from oracle.ref_build import SHAPES, derived
from tests.helpers import lib_kwargs, oracle_for
from ytm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "ytm.h")).read()
    return set(re.findall(r"^\s*(?:const\s+)?[a-z0-9_]+\s*\*?\s*(ytm_[a-z0-9_]+)\s*\(", src, re.M))


def test_header_matches_binding():
    assert declared() == set(_lib.EXPORTS)


def test_library_exports_all_symbols():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.ytm_version().startswith(b"ytm-b200")


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_config_matches_oracle(name):
    kw = SHAPES[name]
    cfg = _lib.make_config(**lib_kwargs(kw, seed=3))
    o = oracle_for(name, seed=3)
    d = derived(kw)
    assert (cfg.clauses, cfg.n_classes, cfg.literals, cfg.words, cfg.patches) == (d["C"], d["K"], d["L"], d["W"], d["P"])
    assert (cfg.clauses, cfg.literals, cfg.words, cfg.patches) == (o.C, o.L, o.W, o.P)
    assert cfg.state_top == o.state_top and cfg.half_state == o.half_state
    assert list(cfg.s_count_cdf) == list(o.cfg.s_cdf) and cfg.q_threshold == o.cfg.q_thr
    assert cfg.q_select == o.cfg.q_select and list(cfg.q_count_cdf) == list(o.cfg.q_cdf)
    for mi in range(8):
        cdf = list(cfg.run_cdf16[mi])
        assert cdf == list(o.cfg.run_cdf16[mi])
        lo, hi = cfg.run_range[mi] & 0xFFFF, cfg.run_range[mi] >> 16
        assert all(v == 0 for v in cdf[:lo]) and all(0 < v < 65536 for v in cdf[lo:hi])
        assert all(v == 65536 for v in cdf[hi:])
    # include iff state > half  <=>  stored value has the top plane set
    assert cfg.half_state + 1 + cfg.state_offset == 1 << (cfg.planes - 1)
    assert cfg.state_top + cfg.state_offset == (1 << cfg.planes) - 1


def test_config_errors():
    with pytest.raises(_lib.YTMError):
        _lib.make_config(clauses_per_class=0, T=1, s=1.0, dim=(4, 1, 1), n_classes=2)
    with pytest.raises(_lib.YTMError):
        _lib.make_config(clauses_per_class=4, T=1, s=1.0, dim=(4, 4, 1), n_classes=2, patch_dim=(5, 5))
    with pytest.raises(_lib.YTMError):  # location literals outside the vector
        _lib.make_config(clauses_per_class=4, T=1, s=1.0, dim=(28, 28, 1), n_classes=2, patch_dim=(3, 3),
                         encode_loc=False)


def test_shard_partition():
    cfg = _lib.make_config(clauses_per_class=1001, T=10, s=3.0, dim=(8, 1, 1), n_classes=3)
    parts = [_lib.shard_config(cfg, r, 4) for r in range(4)]
    assert parts[0].clause_lo == 0
    for a, b in zip(parts, parts[1:]):
        assert a.clause_lo + a.clause_count == b.clause_lo
    assert parts[-1].clause_lo + parts[-1].clause_count == cfg.clauses
    with pytest.raises(_lib.YTMError):
        _lib.shard_config(cfg, 4, 4)


def test_workspace_sizes_grow_with_batch():
    cfg = _lib.make_config(clauses_per_class=100, T=10, s=3.0, dim=(28, 28, 1), n_classes=10, patch_dim=(10, 10))
    lib = _lib.load()
    a = lib.ytm_workspace_bytes(cfg, _lib.YTM_OP_TRAIN, 1)
    b = lib.ytm_workspace_bytes(cfg, _lib.YTM_OP_TRAIN, 8)
    assert 0 < a < b and a % 256 == 0


def test_config_struct_size_matches_binding():
    import ctypes as ct
    assert _lib.load().ytm_config_size() == ct.sizeof(_lib.Config)


def test_entry_points_reject_bad_arguments_without_a_gpu():
    """Argument checks run before any CUDA call: null pointers, negative
    sizes and out-of-range shards come back as status codes."""
    import ctypes as ct
    lib = _lib.load()
    cfg = _lib.make_config(clauses_per_class=8, T=5, s=3.0, dim=(16, 1, 1), n_classes=2)
    assert lib.ytm_infer(ct.byref(cfg), None, None, None, None, 4, None, None, None) == 1
    assert lib.ytm_encode(ct.byref(cfg), None, -1, None, None, None) == 1
    assert lib.ytm_train_eval(ct.byref(cfg), None, None, None, None, None, 0, 0, 0, None, None, None, None) == 1
    assert lib.ytm_peer_allreduce_i32(None, None, 4, 0, None) == 1
    assert lib.ytm_infer(ct.byref(cfg), None, None, None, None, 0, None, None, None) == 0  # N = 0: nothing to do
    assert lib.ytm_last_error()  # the last failure left a message


def test_negative_class_set_draw_table():
    """The negative-class selection is drawn as a set only for coalesced
    models of at least 32 classes with K * Q <= 2; its count table is the
    Binomial(K, Q) CDF scaled to 2^32 (floor, saturated)."""
    from scipy.stats import binom
    cfg = _lib.make_config(clauses_per_class=8, T=10, s=3.0, dim=(16, 1, 1), n_classes=100, seed=1)
    assert cfg.q_select == 1
    Q = 1.0 / 99
    for n in range(32):
        want = min(int(binom.cdf(n, 100, Q) * 2**32), 2**32 - 1)
        assert abs(int(cfg.q_count_cdf[n]) - want) <= 2, n
    assert _lib.make_config(clauses_per_class=8, T=10, s=3.0, dim=(16, 1, 1), n_classes=10, seed=1).q_select == 0
    assert _lib.make_config(clauses_per_class=8, T=10, s=3.0, dim=(16, 1, 1), n_classes=100, seed=1,
                            coalesced=False).q_select == 0
    assert _lib.make_config(clauses_per_class=8, T=10, s=3.0, dim=(16, 1, 1), n_classes=40, seed=1,
                            q=39.0).q_select == 0
