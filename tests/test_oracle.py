"""The CPU oracle pinned against the reference (no GPU needed).

* The reference's own golden vector: ``tests/test_kernels.py:94-98`` of the
  reference (4 rows, 2 centres -> labels [0, 0, 1, 1]).
* Fixtures produced by the reference's public API
  (``skmetal.accelerate(KMeans(...)).fit``, i.e. scikit-learn's Lloyd path on
  a machine without Metal) by ``tests/golden/make_golden.py``: full fits and
  single Lloyd steps on seeded inputs of the C1-C4 recipes, a relocation case,
  a relative-tolerance case and an odd shape. The oracle must reproduce them
  under the same criteria the GPU is held to (label agreement with near-ties
  only, centres within rtol 1e-4, inertia within rtol 1e-5).
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import lloyd as ora
from parity import CENTER_RTOL, INERTIA_RTOL, check_labels

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_kmeans.npz"


def _golden():
    z = np.load(GOLDEN)
    meta = json.loads(str(z["meta"]))
    return z, meta


def _inputs(name):
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN.parent / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    z, meta = _golden()
    c = meta["cases"][name]
    X, init = mg.case_inputs(c["gen"])
    assert mg.digest(X, init) == c["sha256"], "input generator drifted from the fixtures"
    return X, init, c, z


CASES = sorted(_golden()[1]["cases"])


def test_reference_golden_assign():
    # reference tests/test_kernels.py:94-98
    X = np.array([[0.0, 0.0], [1.0, 1.0], [10.0, 10.0], [9.0, 9.0]], dtype=np.float32)
    C = np.array([[0.0, 0.0], [10.0, 10.0]], dtype=np.float32)
    labels, _ = ora.assign(X, C)
    np.testing.assert_array_equal(labels, [0, 0, 1, 1])


@pytest.mark.parametrize("name", CASES)
def test_oracle_full_fit_matches_reference(name):
    X, init, c, z = _inputs(name)
    res = ora.kmeans_lloyd(X, init, max_iter=c["max_iter"], tol=c["tol"], mode="fp32")
    want = z[f"{name}/full/labels"]
    assert res.n_iter == int(z[f"{name}/full/n_iter"])
    mean, Xc, _ = ora.center_data(X)
    check_labels(Xc, res.centers - mean, res.labels, want, f"{name} labels")
    scale = float(np.abs(X).max())
    np.testing.assert_allclose(res.centers, z[f"{name}/full/centers"], rtol=CENTER_RTOL, atol=1e-5 * scale)
    assert res.inertia == pytest.approx(float(z[f"{name}/full/inertia"]), rel=INERTIA_RTOL)


@pytest.mark.parametrize("name", CASES)
def test_oracle_single_step_matches_reference(name):
    """One Lloyd step from the explicit init (max_iter=1: the step, then the
    final E-step against the new centres)."""
    X, init, c, z = _inputs(name)
    mean, Xc, Cc = ora.center_data(X, init)
    step = ora.lloyd_iter(Xc, Cc, "fp32")
    centres = step.centers_new + mean
    scale = float(np.abs(X).max())
    np.testing.assert_allclose(centres, z[f"{name}/step1/centers"], rtol=CENTER_RTOL, atol=1e-5 * scale)
    labels, _ = ora.assign(Xc, step.centers_new)
    check_labels(Xc, step.centers_new, labels, z[f"{name}/step1/labels"], f"{name} step labels")
    assert int(z[f"{name}/step1/n_iter"]) == 1


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_weighted_oracle_matches_sklearn(seed):
    """The weighted restatement (sample_weight) against scikit-learn's own
    weighted Lloyd on well-separated data, including rows of weight zero."""
    from sklearn.cluster import KMeans

    rng = np.random.default_rng(seed)
    n, d, k = 3000, 8, 6
    C = rng.uniform(-10, 10, (k, d))
    X = (C[rng.integers(0, k, n)] + rng.normal(size=(n, d))).astype(np.float32)
    w = rng.uniform(0.2, 3.0, n).astype(np.float32)
    if seed == 2:
        w[:500] = 0.0
    init = X[rng.choice(n, k, replace=False)]
    sk = KMeans(n_clusters=k, init=init, n_init=1, max_iter=50, tol=0, algorithm="lloyd").fit(X, sample_weight=w)
    r = ora.kmeans_lloyd(X, init, 50, 0.0, sample_weight=w)
    np.testing.assert_array_equal(sk.labels_, r.labels)
    np.testing.assert_allclose(sk.cluster_centers_, r.centers, rtol=1e-5, atol=1e-5)
    assert sk.inertia_ == pytest.approx(r.inertia, rel=1e-5)
