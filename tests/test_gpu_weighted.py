"""Weighted Lloyd on the GPU (KMeans.fit(X, sample_weight=w)) against the
oracle's restatement of scikit-learn's weighted Lloyd (oracle/lloyd.py,
pinned to scikit-learn by tests/test_oracle.py), plus the identities that
exact fixed-point sums make bitwise: unit weights are the unweighted fit, and
integer weights are repeated rows."""

import numpy as np
import pytest

from oracle import lloyd as ora
from skmetal_b200 import _bridge

pytestmark = pytest.mark.gpu


def _blobs(n, d, k, seed, spread=10.0, noise=1.0):
    """k separated blobs and an init of one row from each blob, so that the
    fit converges to the same clustering in float32 and float64 (a random
    init that puts two centres in one blob makes the trajectory chaotic)."""
    rng = np.random.default_rng(seed)
    C = rng.uniform(-spread, spread, size=(k, d))
    lab = rng.permutation(np.arange(n) % k)
    X = (C[lab] + noise * rng.normal(size=(n, d))).astype(np.float32)
    init = np.stack([X[np.flatnonzero(lab == j)[0]] for j in range(k)]).astype(np.float32)
    return X, init, rng


# noise levels chosen so that the fits take several iterations yet stay on the
# same trajectory in float32 and float64 (checked with the oracle in both modes)
@pytest.mark.parametrize("n,d,k,seed,noise", [(20000, 8, 6, 0, 5.0), (30000, 100, 20, 1, 12.0),
                                              (12000, 37, 300, 2, 5.0)])
def test_weighted_fit_matches_oracle(n, d, k, seed, noise):
    X, init, rng = _blobs(n, d, k, seed, noise=noise)
    w = rng.uniform(0.2, 3.0, size=n).astype(np.float32)
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, 40, 0.0, sample_weight=w)
    ref = ora.kmeans_lloyd(X, init, 40, 0.0, mode="fp64", relocation_order="sorted", sample_weight=w)
    assert np.mean(lab == ref.labels) >= 0.9999
    np.testing.assert_allclose(c, ref.centers, rtol=1e-4, atol=1e-4)
    assert inertia == pytest.approx(ref.inertia, rel=1e-5)
    assert n_iter == ref.n_iter


def test_unit_weights_are_the_unweighted_fit():
    X, init, _ = _blobs(50000, 32, 16, 3)
    a = _bridge.kmeans_fit(X, init, 30, 0.0)
    b = _bridge.kmeans_fit(X, init, 30, 0.0, sample_weight=np.ones(X.shape[0], np.float32))
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert a[3] == b[3]
    assert a[2] == pytest.approx(b[2], rel=1e-12)


def test_integer_weights_are_repeated_rows():
    """Weights 1, 2 and 4 (exact float32 products) against the rows repeated,
    without centring (repeating rows moves the mean)."""
    X, init, rng = _blobs(20000, 16, 10, 4)
    w = (2.0 ** rng.integers(0, 3, size=X.shape[0])).astype(np.float32)
    cw, lw, iw, nw = _bridge.kmeans_fit(X, init, 25, 0.0, sample_weight=w, center=False)
    Xr = np.repeat(X, w.astype(np.int64), axis=0)
    cr, lr, ir, nr = _bridge.kmeans_fit(Xr, init, 25, 0.0, center=False)
    np.testing.assert_allclose(cw, cr, rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(np.repeat(lw, w.astype(np.int64)), lr)
    assert nw == nr
    assert iw == pytest.approx(ir, rel=1e-9)


def test_zero_weights_and_weight_empty_clusters():
    """Rows of weight 0 add nothing; a cluster holding only such rows is
    empty and is relocated (oracle: scikit-learn's weight-based rule)."""
    X, init, rng = _blobs(15000, 12, 8, 5)
    w = rng.uniform(0.5, 2.0, size=X.shape[0]).astype(np.float32)
    w[rng.random(X.shape[0]) < 0.3] = 0.0
    # one init centre sits on a zero-weight row far from everything else
    X[0] = 200.0
    w[0] = 0.0
    init[0] = X[0]
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, 30, 0.0, sample_weight=w)
    ref = ora.kmeans_lloyd(X, init, 30, 0.0, mode="fp64", relocation_order="sorted", sample_weight=w)
    assert np.mean(lab == ref.labels) >= 0.9999
    np.testing.assert_allclose(c, ref.centers, rtol=1e-4, atol=1e-4)
    assert inertia == pytest.approx(ref.inertia, rel=1e-5)


def test_weighted_dataset_fit_and_inertia():
    X, init, rng = _blobs(20000, 24, 12, 6)
    w = rng.uniform(0.1, 5.0, size=X.shape[0]).astype(np.float32)
    ds = _bridge.Dataset(X)
    try:
        lab = np.empty(X.shape[0], np.int32)
        c1, i1, n1 = ds.fit(init, 30, 0.0, labels_out=lab, sample_weight=w)
    finally:
        ds.close()
    c2, l2, i2, n2 = _bridge.kmeans_fit(X, init, 30, 0.0, sample_weight=w)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(lab, l2)
    # weighted inertia entry point on the fitted centres
    iw = _bridge.kmeans_inertia_weighted(X, c2, l2.astype(np.uint32), w, X.shape[0], X.shape[1], c2.shape[0])
    ref = ora.inertia(X.astype(np.float64), c2.astype(np.float64), l2, "fp64", w)
    assert iw == pytest.approx(ref, rel=1e-5)


def test_bad_weights_raise():
    X, init, _ = _blobs(1000, 4, 3, 7)
    for bad in (np.full(1000, -1.0, np.float32), np.zeros(1000, np.float32),
                np.where(np.arange(1000) == 5, np.nan, 1.0).astype(np.float32)):
        with pytest.raises(RuntimeError):
            _bridge.kmeans_fit(X, init, 5, 0.0, sample_weight=bad)


def test_estimator_sample_weight_matches_sklearn():
    """accelerate(KMeans).fit(X, sample_weight=w) and score(X, sample_weight=w)
    against scikit-learn's weighted Lloyd on well-separated blobs, with an
    explicit init and with k-means++ seeding (the same random stream)."""
    from sklearn.cluster import KMeans

    import skmetal_b200 as skmetal

    X, init, rng = _blobs(8000, 10, 5, 8)
    w = rng.uniform(0.2, 3.0, size=X.shape[0]).astype(np.float32)
    for kw in (dict(init=init, n_init=1), dict(init="k-means++", n_init=1, random_state=3)):
        cpu = KMeans(n_clusters=5, max_iter=50, tol=0, **kw).fit(X, sample_weight=w)
        gpu = skmetal.accelerate(KMeans(n_clusters=5, max_iter=50, tol=0, **kw)).fit(X, sample_weight=w)
        np.testing.assert_array_equal(gpu.labels_, cpu.labels_)
        np.testing.assert_allclose(gpu.cluster_centers_, cpu.cluster_centers_, rtol=1e-4, atol=1e-4)
        assert gpu.inertia_ == pytest.approx(cpu.inertia_, rel=1e-5)
        assert gpu.score(X, sample_weight=w) == pytest.approx(cpu.score(X, sample_weight=w), rel=1e-5)
