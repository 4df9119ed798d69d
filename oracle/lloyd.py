"""CPU oracle for the KMeans Lloyd path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it. The shipped estimator and C-ABI library never call into it.

It restates, in numpy, the algorithm that the reference's ``KMeans`` path runs
on this platform. ``skmetal.accelerate(KMeans(...))`` returns scikit-learn's
``KMeans`` unchanged when Metal is absent (``skmetal/estimators/_registry.py:50-51``,
``skmetal/_dispatch.py:26-47``), so the reference semantics are those of
scikit-learn 1.9.0 (pinned ``scikit-learn>=1.5,<2.0`` at ``pyproject.toml:30``):

* centring of X and of the init array by the column mean
  (``sklearn/cluster/_kmeans.py:1487-1493``);
* the Lloyd loop with strict-convergence check, scaled tolerance on the sum of
  squared centre shifts and the final E-step (``sklearn/cluster/_kmeans.py:705-758``);
* one iteration: bias ``||c||^2``, ``-2 X C^T``, strict-``<`` argmin with the
  first index winning, per-cluster sums and weights
  (``sklearn/cluster/_k_means_lloyd.pyx:23-218``);
* empty-cluster relocation to the points farthest from their assigned centre,
  chosen with ``np.argpartition`` (``sklearn/cluster/_k_means_common.pyx:167-211``);
* averaging with empty clusters placed on the heaviest cluster
  (``sklearn/cluster/_k_means_common.pyx:274-295``) and the per-centre shift
  (``sklearn/cluster/_k_means_common.pyx:298-311``);
* inertia as the sum of direct squared differences
  (``sklearn/cluster/_k_means_common.pyx:94-124``).

Two arithmetic modes are offered. ``"fp32"`` follows scikit-learn's float32
arithmetic (its sums are order-dependent there, so it is reproduced to
rounding, not to the bit). ``"fp64"`` carries every sum and distance in float64
and is the yardstick for classifying label disagreements as near-ties.

The restatement is pinned against scikit-learn itself by
``tests/test_oracle.py`` (end-to-end on the committed golden fixtures and on
live ``sklearn.cluster.KMeans``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

__all__ = [
    "center_data",
    "tolerance",
    "row_norms_sq",
    "assign",
    "lloyd_iter",
    "inertia",
    "kmeans_lloyd",
    "LloydStep",
    "LloydResult",
    "near_tie_gap",
]


def center_data(X: np.ndarray, init: np.ndarray | None = None):
    """Column mean of X and the centred copies (``_kmeans.py:1487-1493``), float32."""
    X = np.asarray(X, dtype=np.float32)
    mean = X.mean(axis=0)
    Xc = X - mean
    initc = None if init is None else np.asarray(init, dtype=np.float32) - mean
    return mean, Xc, initc


def tolerance(X: np.ndarray, tol: float) -> float:
    """Dataset-scaled tolerance ``mean(var(X, axis=0)) * tol`` (``_kmeans.py:285-294``)."""
    if tol == 0:
        return 0.0
    return float(np.mean(np.var(X, axis=0)) * tol)


def row_norms_sq(A: np.ndarray) -> np.ndarray:
    return np.einsum("ij,ij->i", A, A)


def assign(X: np.ndarray, C: np.ndarray, mode: str = "fp32") -> tuple[np.ndarray, np.ndarray]:
    """Labels and the argmin value of ``||c||^2 - 2 x.c`` (``_k_means_lloyd.pyx:190-213``).

    ``np.argmin`` returns the first index among equal minima, which is the
    strict-``<`` scan of the reference.
    """
    dt = np.float32 if mode == "fp32" else np.float64
    Xd = X.astype(dt, copy=False)
    Cd = C.astype(dt, copy=False)
    cn = row_norms_sq(Cd)
    labels = np.empty(X.shape[0], dtype=np.int32)
    best = np.empty(X.shape[0], dtype=dt)
    step = 65536
    for s in range(0, X.shape[0], step):
        D = cn[None, :] + (-2.0 * (Xd[s:s + step] @ Cd.T)).astype(dt, copy=False)
        lab = np.argmin(D, axis=1)
        labels[s:s + step] = lab
        best[s:s + step] = D[np.arange(D.shape[0]), lab]
    return labels, best


def near_tie_gap(X: np.ndarray, C: np.ndarray, la: np.ndarray, lb: np.ndarray) -> np.ndarray:
    """Relative float64 distance gap between labels ``la`` and ``lb`` for each row.

    ``|d(x, c_la) - d(x, c_lb)| / max(d(x, c_la), d(x, c_lb), tiny)`` with exact
    (float64, direct-difference) squared distances.
    """
    Xd = X.astype(np.float64)
    Cd = C.astype(np.float64)
    da = ((Xd - Cd[la]) ** 2).sum(axis=1)
    db = ((Xd - Cd[lb]) ** 2).sum(axis=1)
    return np.abs(da - db) / np.maximum(np.maximum(da, db), 1e-300)


@dataclass
class LloydStep:
    labels: np.ndarray           # E-step labels against centers_old (int32)
    centers_new: np.ndarray      # M-step centres (float32)
    weight: np.ndarray           # per-cluster weight after relocation (float32)
    center_shift: np.ndarray     # per-centre euclidean shift (float32)
    counts: np.ndarray           # per-cluster counts before relocation (int64)
    empty: np.ndarray            # empty cluster ids (ascending)
    far: np.ndarray              # rows relocated to ``empty`` (same order)


def lloyd_iter(X: np.ndarray, centers_old: np.ndarray, mode: str = "fp32",
               relocation_order: str = "argpartition", sample_weight: np.ndarray | None = None) -> LloydStep:
    """One E+M step of ``lloyd_iter_chunked_dense`` on already-centred X.

    ``relocation_order`` selects how the farthest points are paired with the
    ascending empty-cluster ids: ``"argpartition"`` is the reference's own call
    (``_k_means_common.pyx:186-187``), whose order among the farthest points is
    left unspecified by numpy; ``"sorted"`` pairs them by decreasing distance,
    ties to the lower row index (the order the CUDA path uses).

    With ``sample_weight`` (float32, one per row) a row adds ``x * w`` (the
    float32 product, ``_k_means_lloyd.pyx:_update_chunk_dense``) to its
    cluster's sum and ``w`` to its weight; a cluster of weight 0 is empty, and
    a relocated row carries its weighted values and its weight
    (``_k_means_common.pyx:_relocate_empty_clusters_dense``). ``counts`` stays
    the number of rows per cluster.
    """
    X = np.asarray(X, dtype=np.float32)
    centers_old = np.asarray(centers_old, dtype=np.float32)
    k, d = centers_old.shape
    labels, _ = assign(X, centers_old, mode)
    counts = np.bincount(labels, minlength=k).astype(np.int64)
    acc = np.float32 if mode == "fp32" else np.float64
    if sample_weight is None:
        w = np.ones(X.shape[0], dtype=np.float32)
        Xw = X
    else:
        w = np.asarray(sample_weight, dtype=np.float32)
        Xw = X * w[:, None]  # float32 products
    sums = np.zeros((k, d), dtype=np.float64)
    np.add.at(sums, labels, Xw.astype(np.float64))
    sums = sums.astype(acc)
    weight = np.bincount(labels, weights=w.astype(np.float64), minlength=k).astype(acc)

    empty = np.where(weight == 0)[0].astype(np.int32)
    far = np.zeros(0, dtype=np.int64)
    if empty.size:
        dist = ((X - centers_old[labels]) ** 2).sum(axis=1)  # float32, as the reference
        if np.max(dist) != 0:
            m = empty.size
            if relocation_order == "argpartition":
                far = np.argpartition(dist, -m)[:-m - 1:-1]
            else:
                order = np.lexsort((np.arange(dist.size), -dist.astype(np.float64)))
                far = order[:m]
            for new_id, fi in zip(empty, far):
                old_id = labels[fi]
                sums[old_id] -= Xw[fi].astype(acc)
                sums[new_id] = Xw[fi].astype(acc)
                weight[new_id] = w[fi]
                weight[old_id] -= w[fi]
        else:
            empty = np.zeros(0, dtype=np.int32)

    centers_new = np.empty((k, d), dtype=acc)
    heavy = int(np.argmax(weight))
    for j in range(k):
        if weight[j] > 0:
            centers_new[j] = sums[j] * (acc(1.0) / weight[j])
    for j in range(k):
        if not weight[j] > 0:
            centers_new[j] = centers_new[heavy]
    centers_new = centers_new.astype(np.float32)
    shift = np.sqrt(((centers_new.astype(acc) - centers_old.astype(acc)) ** 2).sum(axis=1)).astype(np.float32)
    return LloydStep(labels, centers_new, weight.astype(np.float32), shift, counts, empty, np.asarray(far))


def inertia(X: np.ndarray, C: np.ndarray, labels: np.ndarray, mode: str = "fp64",
            sample_weight: np.ndarray | None = None) -> float:
    """Sum of (weighted) squared direct differences to the assigned centre
    (``_k_means_common.pyx:94-124``)."""
    dt = np.float32 if mode == "fp32" else np.float64
    diff = X.astype(dt) - C.astype(dt)[labels]
    if sample_weight is None:
        return float(np.einsum("ij,ij->", diff, diff))
    return float(np.einsum("ij,ij->i", diff, diff) @ np.asarray(sample_weight, dtype=dt))


@dataclass
class LloydResult:
    labels: np.ndarray
    inertia: float
    centers: np.ndarray          # un-centred (mean added back), float32
    n_iter: int
    strict_convergence: bool
    history: list = field(default_factory=list)  # per-iteration dicts


def kmeans_lloyd(X: np.ndarray, init: np.ndarray, max_iter: int = 300, tol: float = 1e-4,
                 mode: str = "fp32", relocation_order: str = "argpartition",
                 keep_centers: bool = False, sample_weight: np.ndarray | None = None) -> LloydResult:
    """Full ``KMeans(algorithm="lloyd", n_init=1, init=array).fit`` restated.

    Follows ``_kmeans.py:1487-1496`` (centring) and ``:705-758`` (loop).
    """
    X = np.asarray(X, dtype=np.float32)
    tol_scaled = tolerance(X, tol)
    mean, Xc, centers = center_data(X, init)
    labels_old = np.full(X.shape[0], -1, dtype=np.int32)
    history = []
    strict = False
    i = 0
    for i in range(max_iter):
        step = lloyd_iter(Xc, centers, mode, relocation_order, sample_weight)
        n_changed = int(np.count_nonzero(step.labels != labels_old))
        rec = {"n_changed": n_changed, "n_empty": int(step.empty.size),
               "shift_tot": float((step.center_shift.astype(np.float64) ** 2).sum())}
        if keep_centers:
            rec["centers_in"] = centers.copy()
            rec["labels"] = step.labels.copy()
            rec["centers_out"] = step.centers_new.copy()
            rec["counts"] = step.counts.copy()
        history.append(rec)
        centers = step.centers_new
        labels = step.labels
        if n_changed == 0:
            strict = True
            break
        if float((step.center_shift ** 2).sum()) <= tol_scaled:
            break
        labels_old = labels
    if not strict:
        labels, _ = assign(Xc, centers, mode)
    inert = inertia(Xc, centers, labels, "fp64", sample_weight)
    return LloydResult(labels, inert, (centers + mean).astype(np.float32), i + 1, strict, history)
