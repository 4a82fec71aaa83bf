"""pytm.base.BaseTM (reference src/pytm/base.py:5-166) on the B200 engine.

Same constructor, fit and predict signatures and the same rules as the
reference's numpy TM:
  * TA states 0..n_ta_states-1, a literal included iff its state exceeds
    n_ta_states/2 - 1, all states starting there (base.py:19-20, 32-33) — the
    engine's state range 0..max with max = n_ta_states - 1;
  * shared clauses with +-1 weights for every class (base.py:35-37);
  * per sample, feedback for the true class and then for ONE other class drawn
    uniformly (base.py:134-143), each clause updating with probability
    (T - v)/2T resp. (T + v)/2T (base.py:119);
  * prediction counts clauses without includes (base.py:59-67).
The draws come from the engine's Philox stream instead of numpy's generator,
so runs match pytm's rules, not its random sequence.  `q` is accepted and,
as in the reference, unused.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from .. import _lib
from ..engine import CudaEngine


class BaseTM:
    def __init__(self, n_clause, T, s, q, n_class, dim, n_ta_states=256, seed=None, device=None):
        self.n_clause = n_clause
        self.T = T
        self.s = s
        self.s_inv = 1 / s
        self.q = q
        self.n_class = n_class
        self.dim = dim
        self.n_ta_states = n_ta_states
        assert self.n_ta_states <= 256, "n_ta_states must be less than or equal to 256."
        assert self.n_ta_states >= 3, "n_ta_states must be at least 3."
        self.half_state = (self.n_ta_states // 2) - 1
        self.max_state = self.n_ta_states - 1
        self.n_features = int(np.prod(dim))
        self.n_literals = 2 * self.n_features
        self.rng = np.random.default_rng(seed)  # shuffling, as base.py:153-154
        key = int(seed) if seed is not None else int.from_bytes(os.urandom(8), "little") >> 1
        self._cfg = _lib.make_config(clauses_per_class=n_clause, T=T, s=s, dim=(self.n_features, 1, 1),
                                     n_classes=n_class, q=1.0, number_of_ta_states=self.n_ta_states - 1,
                                     init_neg_weights=True, coalesced=True, seed=key, one_negative=True,
                                     count_empty=True)
        self.engine = CudaEngine(self._cfg, device)
        self.sample_counter = 0

    # states / weights in the reference's dtypes and shapes (base.py:27-28)
    @property
    def states(self) -> np.ndarray:
        return self.engine.get_ta_state().astype(np.uint8)

    @property
    def weights(self) -> np.ndarray:
        return self.engine.weights.cpu().numpy().astype(np.float32)

    def _lits(self, X) -> torch.Tensor:
        X = np.asarray(X).reshape(np.asarray(X).shape[0], -1)
        assert X.shape[1] == self.n_features, "X has the wrong number of features."
        Xd = torch.from_numpy(np.ascontiguousarray(X != 0, dtype=np.uint32).view(np.int32)).to(self.engine.device)
        return self.engine.encode(Xd)

    def fit(self, X, y, shuffle: bool = False) -> None:
        """One pass over the samples, one at a time (base.py:145-156)."""
        y = np.asarray(y)
        iota = np.arange(X.shape[0])
        if shuffle:
            self.rng.shuffle(iota)
        lits = self._lits(np.asarray(X)[iota])
        Y = np.where(y[iota][:, None] == np.arange(self.n_class)[None, :], self.T, -self.T).astype(np.int32)
        Yd = torch.from_numpy(Y).to(self.engine.device)
        self.engine.train_fit_b1(lits, Yd, self.sample_counter, None)
        self.sample_counter += X.shape[0]

    def predict(self, X, return_cs: bool = False):
        """Class sums over all firing clauses, argmax (base.py:158-166)."""
        cs = self.engine.infer(self._lits(X)).cpu().numpy().astype(np.float32)
        preds = np.argmax(cs, axis=1)
        if return_cs:
            return preds, cs
        return preds
