"""ctypes front end of the CPU oracle (oracle/ytm_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg as the checker.  The product (``ytm_b200``) never
imports it.

Arrays are numpy, host memory, in the reference's own layouts
(Mayur1009/YTM src/cutm/base.py:189-192): TA states u32 [C][L], weights
[C][K] (int32 here; the reference's float32 weights hold whole numbers),
patch weights i32 [C][P], encoded literals u32 [N][P][W].
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libytm_oracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE, "libytm_oracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ct.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class OrcCfg(ct.Structure):
    _fields_ = [
        ("clauses_per_class", ct.c_int32), ("T", ct.c_int32),
        ("s", ct.c_double), ("q", ct.c_double),
        ("D0", ct.c_int32), ("D1", ct.c_int32), ("D2", ct.c_int32), ("K", ct.c_int32),
        ("P0", ct.c_int32), ("P1", ct.c_int32),
        ("n_states", ct.c_int32), ("max_included", ct.c_int32), ("append_negated", ct.c_int32),
        ("init_neg_weights", ct.c_int32), ("negative_polarity", ct.c_int32),
        ("encode_loc", ct.c_int32), ("coalesced", ct.c_int32),
        ("seed", ct.c_uint64),
        ("banks", ct.c_int32), ("C", ct.c_int32), ("L", ct.c_int32), ("W", ct.c_int32), ("P", ct.c_int32),
        ("max_state", ct.c_int32), ("half_state", ct.c_int32), ("state_top", ct.c_int32),
        ("s_cdf", ct.c_uint32 * 32), ("q_thr", ct.c_uint64), ("q_cdf", ct.c_uint32 * 32), ("q_select", ct.c_int32), ("run_cdf16", (ct.c_uint32 * 65) * 8),
        ("one_negative", ct.c_int32), ("count_empty", ct.c_int32),
    ]


_P = ct.c_void_p
_I32 = ct.c_int32
_I64 = ct.c_int64
_U64 = ct.c_uint64


def _declare(L):
    L.orc_cfg_init.argtypes = [ct.POINTER(OrcCfg), _I32, _I32, ct.c_double, _I32, _I32, _I32, _I32,
                               ct.c_double, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _U64]
    L.orc_cfg_init.restype = ct.c_int
    L.orc_set_threads.argtypes = [ct.c_int]
    L.orc_cfg_set_modes.argtypes = [ct.POINTER(OrcCfg), ct.c_int32, ct.c_int32]
    L.orc_get_threads.restype = ct.c_int
    L.orc_philox4x32_10.argtypes = [_P, _P, _P]
    L.orc_philox4x32.argtypes = [_P, _P, ct.c_int, _P]
    L.orc_smask_word.argtypes = [ct.POINTER(OrcCfg), ct.c_uint32, _U64, ct.c_uint32, ct.c_uint32]
    L.orc_smask_word.restype = ct.c_uint32
    L.orc_run_counts.argtypes = [ct.POINTER(OrcCfg), ct.c_uint32, _U64, ct.c_uint32, ct.c_uint32, ct.c_int, _P]
    L.orc_qselect_set.argtypes = [ct.POINTER(OrcCfg), ct.c_uint32, _U64, _P]
    L.orc_smask_count.argtypes = [ct.c_int]
    L.orc_smask_count.restype = ct.c_uint64
    L.orc_update_threshold.argtypes = [_I32, _I32]
    L.orc_update_threshold.restype = _U64
    L.orc_encode.argtypes = [ct.POINTER(OrcCfg), _P, _I64, _P]
    L.orc_pack.argtypes = [ct.POINTER(OrcCfg), _P, _I32, _P, _P]
    L.orc_infer.argtypes = [ct.POINTER(OrcCfg), _P, _P, _P, _P, _I64, _P]
    L.orc_transform.argtypes = [ct.POINTER(OrcCfg), _P, _P, _I64, _P]
    L.orc_transform_patchwise.argtypes = [ct.POINTER(OrcCfg), _P, _P, _I64, _P]
    L.orc_init_weights.argtypes = [ct.POINTER(OrcCfg), _I32, _I32, _P]
    L.orc_train_eval.argtypes = [ct.POINTER(OrcCfg), _I32, _I32, _P, _P, _P, _P, _P, _I32, _U64, _I32,
                                 _P, _P, _P, _P]
    L.orc_train_update.argtypes = [ct.POINTER(OrcCfg), _I32, _I32, _P, _P, _P, _P, _P, _P, _I32, _U64,
                                   _P, _P]
    L.orc_train_batch.argtypes = [ct.POINTER(OrcCfg), _P, _P, _P, _P, _P, _P, _I32, _U64, _P, _P, _P]


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ct.c_void_p)


def _c(a, dtype):
    """Contiguous array of dtype (the C side reads raw memory)."""
    return np.ascontiguousarray(a, dtype=dtype)


def philox4x32_10(ctr, key):
    c = _c(ctr, np.uint32)
    k = _c(key, np.uint32)
    out = np.zeros(4, np.uint32)
    lib().orc_philox4x32_10(_ptr(c), _ptr(k), _ptr(out))
    return out


def philox4x32(ctr, key, rounds):
    c = _c(ctr, np.uint32)
    k = _c(key, np.uint32)
    out = np.zeros(4, np.uint32)
    lib().orc_philox4x32(_ptr(c), _ptr(k), int(rounds), _ptr(out))
    return out


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return int(lib().orc_get_threads())


class Oracle:
    """One model's sizes and hyper-parameters, mirroring BaseTM.__init__
    (base.py:42-125) with the same keyword defaults (base.py:60-74)."""

    def __init__(self, number_of_clauses_per_class, T, s, dim, n_classes, q=1.0, patch_dim=None,
                 number_of_ta_states=256, max_included_literals=None, append_negated=True,
                 init_neg_weights=True, negative_polarity=True, encode_loc=True, coalesced=True,
                 seed=0, one_negative=False, count_empty=False):
        if patch_dim is None:
            patch_dim = (dim[0], dim[1])
        self.cfg = OrcCfg()
        rc = lib().orc_cfg_init(ct.byref(self.cfg), int(number_of_clauses_per_class), int(T), float(s),
                                int(dim[0]), int(dim[1]), int(dim[2]), int(n_classes), float(q),
                                int(patch_dim[0]), int(patch_dim[1]), int(number_of_ta_states),
                                -1 if max_included_literals is None else int(max_included_literals),
                                int(append_negated), int(init_neg_weights), int(negative_polarity),
                                int(encode_loc), int(coalesced), int(seed) & (2**64 - 1))
        if rc != 0:
            raise ValueError("invalid oracle configuration")
        lib().orc_cfg_set_modes(ct.byref(self.cfg), int(bool(one_negative)), int(bool(count_empty)))
        c = self.cfg
        self.C, self.K, self.L, self.W, self.P = c.C, c.K, c.L, c.W, c.P
        self.half_state, self.state_top = c.half_state, c.state_top

    def _cfg(self):
        return ct.byref(self.cfg)

    def encode(self, X):
        X = _c(X, np.uint32)
        N = X.shape[0]
        out = np.zeros((N, self.P, self.W), np.uint32)
        lib().orc_encode(self._cfg(), _ptr(X), N, _ptr(out))
        return out

    def pack(self, ta):
        ta = _c(ta, np.uint32).reshape(-1, self.L)
        nc = ta.shape[0]
        packed = np.zeros((nc, self.W), np.uint32)
        ninc = np.zeros(nc, np.int32)
        lib().orc_pack(self._cfg(), _ptr(ta), nc, _ptr(packed), _ptr(ninc))
        return packed, ninc

    def infer(self, ta, weights, lits, bias=None):
        ta = _c(ta, np.uint32)
        w = _c(weights, np.int32)
        lits = _c(lits, np.uint32)
        b = None if bias is None else _c(bias, np.int32)
        N = lits.shape[0]
        cs = np.zeros((N, self.K), np.int32)
        lib().orc_infer(self._cfg(), _ptr(ta), _ptr(w), _ptr(b), _ptr(lits), N, _ptr(cs))
        return cs

    def transform(self, ta, lits):
        ta, lits = _c(ta, np.uint32), _c(lits, np.uint32)
        N = lits.shape[0]
        out = np.zeros((N, self.C), np.uint32)
        lib().orc_transform(self._cfg(), _ptr(ta), _ptr(lits), N, _ptr(out))
        return out

    def transform_patchwise(self, ta, lits):
        ta, lits = _c(ta, np.uint32), _c(lits, np.uint32)
        N = lits.shape[0]
        out = np.zeros((N, self.C, self.P), np.uint32)
        lib().orc_transform_patchwise(self._cfg(), _ptr(ta), _ptr(lits), N, _ptr(out))
        return out

    def init_state(self):
        return np.full((self.C, self.L), self.cfg.n_states // 2, np.uint32)

    def init_weights(self, lo=0, n=None):
        n = self.C - lo if n is None else n
        w = np.zeros((n, self.K), np.int32)
        lib().orc_init_weights(self._cfg(), int(lo), int(n), _ptr(w))
        return w

    def smask_word(self, clause, t, k, w):
        return int(lib().orc_smask_word(self._cfg(), clause, t, k, w))

    def run_counts(self, clause, t, k, w, mi):
        """Per-literal decrement counts of a Type Ib run piece of 8 (mi + 1)
        events for word w (u32 [32])."""
        out = np.zeros(32, np.uint32)
        lib().orc_run_counts(self._cfg(), clause, t, k, w, int(mi), _ptr(out))
        return out

    def qselect_set(self, clause, t):
        """The negative-class selection of (clause, sample t) drawn as a set
        (configurations with q_select): bool [K]."""
        out = np.zeros(self.cfg.K, np.uint8)
        lib().orc_qselect_set(self._cfg(), clause, t, _ptr(out))
        return out.astype(bool)

    @staticmethod
    def smask_count(on: bool) -> int:
        """Start (on) or stop counting the Philox4x32-7 calls of the literal
        masks; returns the count since the previous call and resets it."""
        return int(lib().orc_smask_count(int(bool(on))))

    # -- training -----------------------------------------------------------
    def train_eval(self, lo, ta, w, lits, B, t0, drop=None, bias=None, add_bias=False, patch_w=None):
        """Part 1 of a batch for the shard starting at global clause `lo`
        (ta, w, drop, patch_w shard-local).  Returns (cs, sel, ninc); patch_w
        is updated in place."""
        nc = ta.shape[0]
        assert ta.flags.c_contiguous and ta.dtype == np.uint32
        w = _c(w, np.int32)
        lits = _c(lits, np.uint32)
        if patch_w is None:
            patch_w = np.zeros((nc, self.P), np.int32)
        assert patch_w.flags.c_contiguous and patch_w.dtype == np.int32
        d = None if drop is None else _c(drop, np.uint32)
        bb = None if bias is None else _c(bias, np.int32)
        cs = np.zeros((B, self.K), np.int32)
        sel = np.zeros((B, nc), np.int32)
        ninc = np.zeros(nc, np.int32)
        lib().orc_train_eval(self._cfg(), int(lo), nc, _ptr(ta), _ptr(w), _ptr(bb), _ptr(d), _ptr(lits),
                             int(B), int(t0), int(bool(add_bias)), _ptr(cs), _ptr(patch_w), _ptr(sel),
                             _ptr(ninc))
        return cs, sel, ninc

    def train_update(self, lo, ta, w, cs, Y, lits, B, t0, sel, ninc, drop=None):
        """Part 2 of a batch; ta and w (shard-local, contiguous) change in place."""
        nc = ta.shape[0]
        assert ta.flags.c_contiguous and ta.dtype == np.uint32
        assert w.flags.c_contiguous and w.dtype == np.int32
        d = None if drop is None else _c(drop, np.uint32)
        cs, Y = _c(cs, np.int32), _c(Y, np.int32)
        lits, sel, ninc = _c(lits, np.uint32), _c(sel, np.int32), _c(ninc, np.int32)
        lib().orc_train_update(self._cfg(), int(lo), nc, _ptr(ta), _ptr(w), _ptr(cs), _ptr(Y), _ptr(d),
                               _ptr(lits), int(B), int(t0), _ptr(sel), _ptr(ninc))

    def train_batch(self, ta, w, patch_w, lits, Y, t0, drop=None, sel_override=None):
        """A whole batch (all clauses); ta, w, patch_w change in place.
        Returns (cs, sel) as used by the feedback."""
        for a, dt in ((ta, np.uint32), (w, np.int32), (patch_w, np.int32)):
            assert a.flags.c_contiguous and a.dtype == dt
        lits, Y = _c(lits, np.uint32), _c(Y, np.int32)
        B = lits.shape[0]
        d = None if drop is None else _c(drop, np.uint32)
        so = None if sel_override is None else _c(sel_override, np.int32)
        cs = np.zeros((B, self.K), np.int32)
        sel = np.zeros((B, self.C), np.int32)
        lib().orc_train_batch(self._cfg(), _ptr(ta), _ptr(w), _ptr(patch_w), _ptr(d), _ptr(lits), _ptr(Y),
                              int(B), int(t0), _ptr(so), _ptr(cs), _ptr(sel))
        return cs, sel

    def fit(self, ta, w, patch_w, lits, Y, t0=0, batch_size=1, drop=None):
        """Train over all samples in order with the given batch size; returns
        the sample counter after the last batch."""
        N = lits.shape[0]
        t = t0
        for i in range(0, N, batch_size):
            self.train_batch(ta, w, patch_w, lits[i:i + batch_size], Y[i:i + batch_size], t, drop=drop)
            t += min(batch_size, N - i)
        return t


def encode_Y_multiclass(Y, K, T):
    """multiclass.py:35-37: +T for the true class, -T otherwise."""
    Y = np.asarray(Y)
    return np.where(Y[:, None] == np.arange(K)[None, :], T, -T).astype(np.int32)


def encode_Y_multioutput(Y, T):
    """multioutput.py:36."""
    return np.where(np.asarray(Y) == 1, T, -T).astype(np.int32)
