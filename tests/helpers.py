"""Shared test helpers: golden fixtures, oracle/engine pairs, kwargs mapping."""
from __future__ import annotations

import glob
import os

import numpy as np

from oracle import oracle as O
from oracle.ref_build import SHAPES

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_names(prefix=""):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, f"{prefix}*.npz")))


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def oracle_kwargs(kw, seed=0):
    return dict(number_of_clauses_per_class=kw["number_of_clauses_per_class"], T=kw["T"], s=kw["s"],
                dim=kw["dim"], n_classes=kw["n_classes"], q=kw.get("q", 1.0), patch_dim=kw.get("patch_dim"),
                number_of_ta_states=kw.get("number_of_ta_states", 256),
                max_included_literals=kw.get("max_included_literals"),
                append_negated=kw.get("append_negated", True), init_neg_weights=kw.get("init_neg_weights", True),
                negative_polarity=kw.get("negative_polarity", True), encode_loc=kw.get("encode_loc", True),
                coalesced=kw.get("coalesced", True), seed=seed)


def lib_kwargs(kw, seed=0):
    d = oracle_kwargs(kw, seed)
    d["clauses_per_class"] = d.pop("number_of_clauses_per_class")
    return d


def oracle_for(name, seed=0):
    return O.Oracle(**oracle_kwargs(SHAPES[name], seed))


def bits_of(lits, L):
    N = lits.shape[0]
    return np.unpackbits(np.ascontiguousarray(lits).view(np.uint8).reshape(N, -1, lits.shape[-1] * 4),
                         axis=2, bitorder="little")[:, :, :L]
