"""Generate the golden KMeans fixtures from the reference itself.

Run in a checkout where the reference package is importable (its source tree
on PYTHONPATH), e.g.::

    PYTHONPATH=/path/to/skmetal python tests/golden/make_golden.py

For every case it draws the inputs with ``skmetal_b200._synthetic`` (seeded),
fits ``skmetal.accelerate(KMeans(n_clusters=k, init=init, n_init=1,
max_iter=M, tol=tol, algorithm="lloyd"))`` -- the reference's public API,
which on a machine without Apple Metal is scikit-learn's Lloyd path
(``skmetal/estimators/_registry.py:50-51``) -- once with ``max_iter=M`` and
once with ``max_iter=1`` (one Lloyd step plus the final E-step), and stores
the outputs with a SHA-256 of the inputs in ``golden_kmeans.npz``. The inputs
are not stored: tests regenerate them and check the hash.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from skmetal_b200._synthetic import _dirichlet_mixture, _unit_rows, gaussian_mixture  # noqa: E402

# name: (generator, k, max_iter, tol)
CASES = {
    "c1_small": ("mixture:4000:32:8:0", 8, 50, 0.0),
    "c2_small": ("mixture:6000:100:50:1", 50, 30, 0.0),
    "c3_small": ("unit:3000:128:64:2", 64, 10, 0.0),
    # the C3 codebook shape: k = 1024 (several 256-cluster blocks of the
    # tensor-core E-step), d = 128
    "c3_k1024": ("unit:20000:128:1024:2", 1024, 4, 0.0),
    # k = 300: two uneven cluster blocks, d not a multiple of 8
    "k300_odd": ("mixture:9000:37:300:4", 300, 6, 0.0),
    "c4_small": ("dirichlet:5000:64:256:3", 256, 8, 0.0),
    "tol_rel": ("mixture:3000:32:8:0", 8, 100, 1e-4),
    "relocation": ("reloc", 20, 10, 0.0),
    "odd_shape": ("odd", 7, 20, 0.0),
}


def case_inputs(gen: str):
    """(X, init) of a case, float32 C-contiguous."""
    if gen == "reloc":
        # k = 20 on 5 blobs with a duplicate-heavy init: empty clusters appear
        X, _ = gaussian_mixture(4000, 10, 5, seed=11)
        init = np.ascontiguousarray(np.repeat(X[:4], 5, axis=0))
        return X, init
    if gen == "reloc1":
        # 6 blobs, 7 initial centres of which the last duplicates the first:
        # exactly one cluster is empty in each of the first two iterations
        X, _ = gaussian_mixture(20000, 16, 6, seed=23)
        init = np.ascontiguousarray(np.concatenate([X[:6], X[:1]]))
        return X, init
    if gen == "odd":
        rng = np.random.default_rng(257)
        X = (rng.standard_normal((257, 9)) * 3).astype(np.float32)
        init = np.ascontiguousarray(X[rng.choice(257, 7, replace=False)])
        return X, init
    kind, n, d, k, seed = gen.split(":")
    n, d, k, seed = int(n), int(d), int(k), int(seed)
    if kind == "mixture":  # the C1 / C2 recipe at a smaller n
        return gaussian_mixture(n, d, k, seed)
    if kind == "unit":  # the C3 recipe
        return _unit_rows(n, d, k, seed)
    if kind == "dirichlet":  # the C4 recipe
        return _dirichlet_mixture(n, d, k, seed)
    raise KeyError(gen)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    from sklearn.cluster import KMeans
    import sklearn
    from skmetal import accelerate

    out = {}
    meta = {"sklearn": sklearn.__version__, "numpy": np.__version__, "cases": {}}
    for name, (gen, k, max_iter, tol) in CASES.items():
        X, init = case_inputs(gen)
        assert init.shape[0] == k
        for tag, mi in (("full", max_iter), ("step1", 1)):
            est = accelerate(KMeans(n_clusters=k, init=init, n_init=1, max_iter=mi, tol=tol, algorithm="lloyd"))
            est.fit(X)
            out[f"{name}/{tag}/labels"] = est.labels_.astype(np.int32)
            out[f"{name}/{tag}/centers"] = est.cluster_centers_.astype(np.float32)
            out[f"{name}/{tag}/inertia"] = np.float64(est.inertia_)
            out[f"{name}/{tag}/n_iter"] = np.int32(est.n_iter_)
        meta["cases"][name] = {"gen": gen, "k": k, "max_iter": max_iter, "tol": tol, "n": int(X.shape[0]),
                               "d": int(X.shape[1]), "sha256": digest(X, init)}
        print(name, X.shape, "n_iter", int(out[f"{name}/full/n_iter"]), "inertia", float(out[f"{name}/full/inertia"]))
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "golden_kmeans.npz", **out)
    print("wrote", HERE / "golden_kmeans.npz")


if __name__ == "__main__":
    main()
