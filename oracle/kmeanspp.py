"""CPU oracle for k-means++ seeding -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/`` may import it.

It restates scikit-learn 1.9.0's greedy k-means++
(``sklearn/cluster/_kmeans.py``, ``_kmeans_plusplus``), which is what
``skmetal.accelerate(KMeans(init="k-means++"))`` runs on a machine without
Metal (``skmetal/estimators/_registry.py:50-51``):

* the first centre is ``random_state.choice(n, p=w / w.sum())``;
* ``n_local_trials = 2 + int(log(k))`` unless given;
* for every further centre: ``u = random_state.uniform(size=n_local_trials)``,
  targets ``u * pot``, candidates = ``searchsorted(cumsum(w * closest), targets)``
  (left side) clipped to ``n - 1``; each candidate's squared distances to all
  rows, ``min`` with the current closest distances, potentials
  ``sum(w * new)``; the first candidate of smallest potential is kept;
* squared distances as ``_euclidean_distances_upcast`` forms them for float32
  data: ``(-2 x.y + |x|^2) + |y|^2`` in float64, rounded to float32, then
  ``max(., 0)``.

Arithmetic of the restatement (which the GPU path follows): the cumulative sum
and every potential are accumulated in float64. scikit-learn accumulates both
in float32 (``np.cumsum`` of a float32 array, a float32 matrix-vector
product), whose rounding depends on the order and on the BLAS build, so for
large n its candidate positions can move by a few rows; this restatement is
the float64 form of the same algorithm with the same random stream.
"""

from __future__ import annotations

import numpy as np


def sq_dist_to(X: np.ndarray, y: np.ndarray) -> np.ndarray:
    """float32 squared distances of every row of X to the row y, formed as
    scikit-learn's float32 path does (float64 inside, rounded to float32)."""
    X64 = X.astype(np.float64)
    y64 = y.astype(np.float64)
    xx = np.einsum("ij,ij->i", X64, X64)
    yy = float(y64 @ y64)
    d = -2.0 * (X64 @ y64)
    d += yy
    d += xx
    return np.maximum(d.astype(np.float32), np.float32(0))


def kmeans_plusplus(X: np.ndarray, k: int, random_state: np.random.RandomState,
                    sample_weight: np.ndarray | None = None, n_local_trials: int | None = None):
    """Centres (k x d float32) and their row indices, drawing from
    ``random_state`` in scikit-learn's order."""
    n, d = X.shape
    w = np.ones(n, dtype=X.dtype) if sample_weight is None else np.asarray(sample_weight, dtype=X.dtype)
    if n_local_trials is None:
        n_local_trials = 2 + int(np.log(k))
    centers = np.empty((k, d), dtype=X.dtype)
    indices = np.full(k, -1, dtype=np.int64)
    cid = random_state.choice(n, p=w / w.sum())
    centers[0] = X[cid]
    indices[0] = cid
    closest = sq_dist_to(X, X[cid])
    w64 = w.astype(np.float64)
    pot = float(np.dot(closest.astype(np.float64), w64))
    for c in range(1, k):
        targets = random_state.uniform(size=n_local_trials) * pot
        cs = np.cumsum(w64 * closest.astype(np.float64))
        cand = np.searchsorted(cs, targets)
        np.clip(cand, None, n - 1, out=cand)
        best_t, best_pot, best_new = -1, np.inf, None
        for t, ci in enumerate(cand):
            new = np.minimum(closest, sq_dist_to(X, X[ci]))
            p = float(np.dot(new.astype(np.float64), w64))
            if p < best_pot:
                best_t, best_pot, best_new = t, p, new
        ci = int(cand[best_t])
        centers[c] = X[ci]
        indices[c] = ci
        closest, pot = best_new, best_pot
    return centers, indices
