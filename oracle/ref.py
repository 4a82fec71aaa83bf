"""ctypes front end of oracle/_ref/ref_<shape>.so — the reference's own CUDA
kernels (Mayur1009/YTM src/cutm/cuda/kernel.cu) compiled from its source by
oracle/ref_build.py.  TEST INFRASTRUCTURE ONLY; needs a GPU to run.
"""
from __future__ import annotations

import ctypes as ct
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
_P = ct.c_void_p


def available(name: str) -> bool:
    return os.path.exists(os.path.join(REF_DIR, f"ref_{name}.so"))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ct.c_void_p)


class RefKernels:
    def __init__(self, name: str):
        path = os.path.join(REF_DIR, f"ref_{name}.so")
        L = ct.CDLL(path)
        L.ref_sizes.argtypes = [_P]
        L.ref_encode.argtypes = [_P, ct.c_int, _P]
        L.ref_pack.argtypes = [_P, _P, _P]
        L.ref_infer.argtypes = [_P, _P, _P, ct.c_int, _P]
        L.ref_transform.argtypes = [_P, _P, ct.c_int, ct.c_int, _P]
        L.ref_init_weights.argtypes = [ct.c_ulonglong, _P]
        L.ref_train_step.argtypes = [_P, _P, _P, _P, _P, ct.c_int, ct.c_int, _P, ct.c_ulonglong, _P, _P]
        L.ref_fit.argtypes = [_P, _P, _P, _P, _P, ct.c_int, ct.c_ulonglong]
        self.L = L
        s = np.zeros(5, np.int32)
        L.ref_sizes(_ptr(s))
        self.C, self.K, self.Lits, self.W, self.P = (int(v) for v in s)

    @staticmethod
    def _ok(rc, what):
        if rc != 0:
            raise RuntimeError(f"reference {what} failed: CUDA error {rc}")

    def encode(self, X):
        X = np.ascontiguousarray(X, np.uint32)
        out = np.zeros((X.shape[0], self.P, self.W), np.uint32)
        self._ok(self.L.ref_encode(_ptr(X), X.shape[0], _ptr(out)), "encode")
        return out

    def pack(self, ta):
        ta = np.ascontiguousarray(ta, np.uint32)
        packed = np.zeros((self.C, self.W), np.uint32)
        ninc = np.zeros(self.C, np.int32)
        self._ok(self.L.ref_pack(_ptr(ta), _ptr(packed), _ptr(ninc)), "pack")
        return packed, ninc

    def infer(self, ta, w, lits, bias=None):
        ta = np.ascontiguousarray(ta, np.uint32)
        w = np.ascontiguousarray(w, np.float32)
        lits = np.ascontiguousarray(lits, np.uint32)
        N = lits.shape[0]
        cs = np.zeros((N, self.K), np.float32)
        if bias is not None:
            cs[:] = np.asarray(bias, np.float32)[None, :]
        self._ok(self.L.ref_infer(_ptr(ta), _ptr(w), _ptr(lits), N, _ptr(cs)), "infer")
        return cs

    def transform(self, ta, lits, patchwise=False):
        ta = np.ascontiguousarray(ta, np.uint32)
        lits = np.ascontiguousarray(lits, np.uint32)
        N = lits.shape[0]
        shape = (N, self.C, self.P) if patchwise else (N, self.C)
        out = np.zeros(shape, np.uint32)
        self._ok(self.L.ref_transform(_ptr(ta), _ptr(lits), N, int(patchwise), _ptr(out)), "transform")
        return out

    def init_weights(self, seed=0):
        w = np.zeros((self.C, self.K), np.float32)
        self._ok(self.L.ref_init_weights(seed, _ptr(w)), "init_weights")
        return w

    def train_step(self, ta, w, patch_w, lits, Y, e, drop=None, seed=0):
        """One sample of _fit (base.py:305-357); ta, w, patch_w updated in place."""
        for a, dt in ((ta, np.uint32), (w, np.float32), (patch_w, np.int32)):
            assert a.flags.c_contiguous and a.dtype == dt
        lits = np.ascontiguousarray(lits, np.uint32)
        Y = np.ascontiguousarray(Y, np.int32)
        d = None if drop is None else np.ascontiguousarray(drop, np.uint32)
        sel = np.zeros(self.C, np.int32)
        cs = np.zeros(self.K, np.float32)
        self._ok(self.L.ref_train_step(_ptr(ta), _ptr(w), _ptr(patch_w), _ptr(lits), _ptr(Y), lits.shape[0], int(e),
                                       _ptr(d), seed, _ptr(sel), _ptr(cs)), "train_step")
        return sel, cs

    def fit(self, ta, w, patch_w, lits, Y, seed=0):
        """One epoch of the reference's _fit loop on the device; ta, w, patch_w
        updated in place."""
        for a, dt in ((ta, np.uint32), (w, np.float32), (patch_w, np.int32)):
            assert a.flags.c_contiguous and a.dtype == dt
        lits = np.ascontiguousarray(lits, np.uint32)
        Y = np.ascontiguousarray(Y, np.int32)
        self._ok(self.L.ref_fit(_ptr(ta), _ptr(w), _ptr(patch_w), _ptr(lits), _ptr(Y), lits.shape[0], seed), "fit")
