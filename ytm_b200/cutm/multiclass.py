"""MultiClassTM — reference src/cutm/multiclass.py:6-59 on the B200 engine."""
from __future__ import annotations

import numpy as np
import torch

from .base import BaseTM


class MultiClassTM(BaseTM):
    def __init__(self, number_of_clauses_per_class: int, T: int, s: float, dim: tuple[int, int, int],
                 n_classes: int, **opt_args):
        super().__init__(number_of_clauses_per_class=number_of_clauses_per_class, T=T, s=s, dim=dim,
                         n_classes=n_classes, **opt_args)

    def encode_Y(self, Y) -> np.ndarray:
        """+T for the true class, -T for the others (multiclass.py:35-37)."""
        Y = np.asarray(Y)
        return np.where(Y[:, None] == np.arange(self.number_of_outputs)[None, :], self.T, -self.T).astype(np.int32)

    def fit(self, X, Y, is_X_encoded: bool = False, **opt_args):
        Yn = Y.cpu().numpy() if isinstance(Y, torch.Tensor) else np.asarray(Y)
        assert Yn.ndim == 1, "Y must be 1D array (samples,)"
        assert X.shape[0] == Yn.shape[0], "X and Y must have the same number of samples."
        encoded_Y = self.encode_Y(Yn)
        encoded_X = self._literals_device(X, is_X_encoded)
        self._fit(encoded_X, encoded_Y, **opt_args)

    def score(self, X, is_X_encoded: bool, block_size: int | None = None):
        lits = self._literals_device(X, is_X_encoded)
        return self._score_device(lits).cpu().numpy().astype(np.float32)

    def predict(self, X, is_X_encoded: bool = False, block_size: int | None = None):
        class_sums = self.score(X, is_X_encoded, block_size=block_size)
        preds = np.argmax(class_sums, axis=1)
        return preds, class_sums
