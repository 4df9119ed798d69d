"""Seeded synthetic KMeans workloads (the five benchmark configurations).

The reference publishes no dataset for its KMeans benchmark; its own timing
script draws ``make_blobs`` data (``benchmarks/benchmark_suite.py:63-64``).
These generators pin five workloads by shape, value distribution and seed so
that the bench, the parity tests and the CPU baseline all see the same bytes.

Every generator returns ``(X, init)`` as C-contiguous float32 arrays (``init``
is ``None`` for the predict workload, which returns ``(X, centers)``).
Generation order is fixed: changing it changes every downstream number.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = ["Workload", "WORKLOADS", "make_workload", "make_rows", "gaussian_mixture", "scaled"]


@dataclass(frozen=True)
class Workload:
    name: str
    n: int
    d: int
    k: int
    max_iter: int
    seed: int
    kind: str  # "fit" or "predict"
    description: str


WORKLOADS = {
    "c1": Workload("c1", 100_000, 32, 8, 50, 0, "fit",
                   "8-component isotropic Gaussian mixture, centres U(-10,10)^32, std 1, equal sizes"),
    "c2": Workload("c2", 500_000, 100, 50, 100, 1, "fit",
                   "50-component isotropic Gaussian mixture, centres U(-10,10)^100, std 1, equal sizes"),
    "c3": Workload("c3", 2_000_000, 128, 1024, 25, 2, "fit",
                   "i.i.d. N(0,1) rows L2-normalised (large-k codebook)"),
    "c4": Workload("c4", 50_000_000, 64, 256, 20, 3, "fit",
                   "256-component Gaussian mixture, centres U(-5,5)^64, std U(0.5,2), Dirichlet(1) sizes"),
    "c5": Workload("c5", 400_000_000, 8, 16, 1, 4, "predict",
                   "i.i.d. U[0,1)^8 rows, 16 fixed centres U[0,1)^8 (seed 5)"),
}

_CHUNK = 1_000_000  # rows per generation chunk for the large workloads


def gaussian_mixture(n: int, d: int, k: int, seed: int, spread: float = 10.0) -> tuple[np.ndarray, np.ndarray]:
    """Equal-size isotropic mixture: centres U(-spread, spread)^d, unit std, rows shuffled.

    ``init`` is ``k`` distinct rows of ``X`` chosen by the same generator.
    """
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-spread, spread, (k, d))
    labels = np.repeat(np.arange(k), -(-n // k))[:n]
    rng.shuffle(labels)
    X = (centres[labels] + rng.standard_normal((n, d))).astype(np.float32)
    init = np.ascontiguousarray(X[rng.choice(n, k, replace=False)])
    return X, init


def _unit_rows(n: int, d: int, k: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d), dtype=np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True).astype(np.float32)
    init = np.ascontiguousarray(X[rng.choice(n, k, replace=False)])
    return X, init


def _dirichlet_plan(n: int, d: int, k: int, seed: int):
    """Mixture parameters, every row's component and the init row indices of
    the C4 recipe (the main stream of ``default_rng(seed)``)."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-5.0, 5.0, (k, d)).astype(np.float32)
    sigma = rng.uniform(0.5, 2.0, k).astype(np.float32)
    p = rng.dirichlet(np.ones(k))
    sizes = rng.multinomial(n, p)
    labels = np.repeat(np.arange(k, dtype=np.int32), sizes)
    rng.shuffle(labels)
    # k seed-chosen rows of the first chunk (an unbiased sample: the rows'
    # components are shuffled), so that the init needs no other chunk
    init_idx = rng.choice(min(n, _CHUNK), k, replace=False)
    return centres, sigma, labels, init_idx


def _dirichlet_rows(plan, d: int, lo: int, hi: int) -> np.ndarray:
    """Rows [lo, hi) of the C4 recipe: chunk c (rows [c * _CHUNK, ...)) draws
    its noise from its own stream default_rng([seed, c + 1]), so any row range
    is generated without the rows before it."""
    centres, sigma, labels, _, seed = plan
    X = np.empty((hi - lo, d), dtype=np.float32)
    for c in range(lo // _CHUNK, -(-hi // _CHUNK)):
        s0, e0 = c * _CHUNK, min(labels.shape[0], (c + 1) * _CHUNK)
        a, b = max(lo, s0), min(hi, e0)
        if a >= b:
            continue
        noise = np.random.default_rng([seed, c + 1]).standard_normal((b - s0, d), dtype=np.float32)[a - s0:]
        lab = labels[a:b]
        X[a - lo:b - lo] = centres[lab] + sigma[lab, None] * noise
    return X


def _dirichlet_mixture(n: int, d: int, k: int, seed: int, lo: int = 0, hi: int | None = None):
    hi = n if hi is None else hi
    centres, sigma, labels, init_idx = _dirichlet_plan(n, d, k, seed)
    plan = (centres, sigma, labels, init_idx, seed)
    X = _dirichlet_rows(plan, d, lo, hi)
    head = X if lo == 0 and hi >= min(n, _CHUNK) else _dirichlet_rows(plan, d, 0, min(n, _CHUNK))
    init = np.ascontiguousarray(head[init_idx])
    return X, init


def _uniform_predict(n: int, d: int, k: int, seed: int, lo: int = 0, hi: int | None = None):
    """Rows [lo, hi) of U[0,1)^d (chunk c from default_rng([seed, c + 1])) and
    the k centres U[0,1)^d from default_rng(seed + 1)."""
    hi = n if hi is None else hi
    X = np.empty((hi - lo, d), dtype=np.float32)
    for c in range(lo // _CHUNK, -(-hi // _CHUNK)):
        s0, e0 = c * _CHUNK, min(n, (c + 1) * _CHUNK)
        a, b = max(lo, s0), min(hi, e0)
        if a >= b:
            continue
        X[a - lo:b - lo] = np.random.default_rng([seed, c + 1]).random((b - s0, d), dtype=np.float32)[a - s0:]
    centers = np.random.default_rng(seed + 1).random((k, d), dtype=np.float32)
    return X, centers


def scaled(name: str, n: int) -> Workload:
    """The workload ``name`` with ``n`` rows (same distribution, same seed)."""
    w = WORKLOADS[name]
    return Workload(w.name, n, w.d, w.k, w.max_iter, w.seed, w.kind, w.description)


def make_workload(w: Workload | str) -> tuple[np.ndarray, np.ndarray]:
    """Generate ``(X, init)`` (fit workloads) or ``(X, centers)`` (predict)."""
    if isinstance(w, str):
        w = WORKLOADS[w]
    return make_rows(w, 0, w.n)


def make_rows(w: Workload | str, lo: int, hi: int) -> tuple[np.ndarray, np.ndarray]:
    """Rows ``[lo, hi)`` of the workload's X and its init (or centres): the
    same values as ``make_workload(w)[0][lo:hi]``. The C4 and C5 recipes
    generate only the requested rows (plus the init's chunk), so every rank of
    a sharded run holds just its shard."""
    if isinstance(w, str):
        w = WORKLOADS[w]
    if w.name in ("c1", "c2", "c3"):
        X, init = (gaussian_mixture(w.n, w.d, w.k, w.seed) if w.name != "c3" else _unit_rows(w.n, w.d, w.k, w.seed))
        return (X if (lo, hi) == (0, w.n) else np.ascontiguousarray(X[lo:hi])), init
    if w.name == "c4":
        return _dirichlet_mixture(w.n, w.d, w.k, w.seed, lo, hi)
    if w.name == "c5":
        return _uniform_predict(w.n, w.d, w.k, w.seed, lo, hi)
    raise KeyError(w.name)
