"""MultiOutputTM — reference src/cutm/multioutput.py:6-57 on the B200 engine."""
from __future__ import annotations

import numpy as np
import torch

from .base import BaseTM


class MultiOutputTM(BaseTM):
    def __init__(self, number_of_clauses_per_class: int, T: int, s: float, dim: tuple[int, int, int],
                 n_classes: int, **opt_args):
        super().__init__(number_of_clauses_per_class=number_of_clauses_per_class, T=T, s=s, dim=dim,
                         n_classes=n_classes, **opt_args)

    def fit(self, X, Y, is_X_encoded: bool = False, **opt_args) -> None:
        Yn = Y.cpu().numpy() if isinstance(Y, torch.Tensor) else np.asarray(Y)
        assert Yn.ndim == 2, f"Y must be 2D array (samples, outputs), got {Yn.ndim}D"
        assert X.shape[0] == Yn.shape[0], "X and Y must have the same number of samples"
        encoded_Y = np.where(Yn == 1, self.T, -self.T).astype(np.int32)  # multioutput.py:36
        encoded_X = self._literals_device(X, is_X_encoded)
        self._fit(encoded_X, encoded_Y, **opt_args)

    def score(self, X, is_X_encoded: bool, block_size: int | None = None):
        lits = self._literals_device(X, is_X_encoded)
        return self._score_device(lits).cpu().numpy().astype(np.float32)

    def predict(self, X, is_X_encoded: bool = False, block_size: int | None = None):
        class_sums = self.score(X, is_X_encoded, block_size=block_size)
        preds = (class_sums >= 0).astype(np.uint32)  # multioutput.py:56
        return preds, class_sums
