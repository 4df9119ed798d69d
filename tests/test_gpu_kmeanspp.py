"""GPU k-means++ seeding through the C ABI, against the oracle's float64
restatement of scikit-learn's greedy k-means++ (oracle/kmeanspp.py) on the
same random stream, and against scikit-learn itself where its float32
accumulation cannot move a candidate (small n)."""

import numpy as np
import pytest

from oracle import lloyd as ora
from oracle.kmeanspp import kmeans_plusplus as oracle_pp
from skmetal_b200 import _bridge

pytestmark = pytest.mark.gpu


def _exact_mean_centred(X):
    """X centred by its exact column mean rounded to float32 (the fit's centring)."""
    mean = (X.astype(np.float64).sum(axis=0, dtype=np.float64) / X.shape[0]).astype(np.float32)
    return X - mean


@pytest.mark.parametrize("n,d,k,seed", [(500, 2, 5, 0), (3000, 13, 17, 1), (5000, 64, 40, 2), (2049, 100, 8, 3),
                                        (4097, 7, 64, 4)])
def test_plusplus_matches_oracle(n, d, k, seed):
    rng = np.random.default_rng(seed)
    X = (rng.normal(size=(n, d)) * rng.uniform(0.5, 3.0, size=(1, d)) + rng.normal(size=(1, d)) * 5).astype(np.float32)
    centers, idx = _bridge.kmeans_plusplus(X, k, np.random.RandomState(seed))
    _, ref_idx = oracle_pp(_exact_mean_centred(X), k, np.random.RandomState(seed))
    np.testing.assert_array_equal(idx, ref_idx)
    np.testing.assert_array_equal(centers, X[idx])


def test_plusplus_weighted_and_uncentred():
    rng = np.random.default_rng(7)
    X = rng.normal(size=(3000, 9)).astype(np.float32)
    w = rng.uniform(0.1, 3.0, size=3000).astype(np.float32)
    centers, idx = _bridge.kmeans_plusplus(X, 12, np.random.RandomState(3), sample_weight=w, center=False)
    _, ref_idx = oracle_pp(X, 12, np.random.RandomState(3), sample_weight=w)
    np.testing.assert_array_equal(idx, ref_idx)


def test_plusplus_matches_sklearn_small():
    """scikit-learn's own seeding (float32 cumulative sums) picks the same rows
    on small inputs; its data is centred by numpy's float32 mean, so the
    GPU is given the same centred copy without further centring."""
    from sklearn.cluster import kmeans_plusplus as sk_pp

    rng = np.random.default_rng(11)
    for trial in range(6):
        n, d, k = int(rng.integers(200, 1500)), int(rng.integers(2, 30)), int(rng.integers(2, 12))
        X = (rng.normal(size=(n, d)) * 2.0).astype(np.float32)
        _, Xc, _ = ora.center_data(X)
        _, idx = _bridge.kmeans_plusplus(np.ascontiguousarray(Xc), k, np.random.RandomState(trial), center=False)
        _, sk_idx = sk_pp(Xc, k, random_state=np.random.RandomState(trial))
        np.testing.assert_array_equal(idx, sk_idx)


def test_plusplus_on_dataset_and_duplicates():
    rng = np.random.default_rng(5)
    base = rng.normal(size=(40, 6)).astype(np.float32)
    X = np.repeat(base, 50, axis=0)  # many identical rows: zero distances, ties in the sums
    ds = _bridge.Dataset(X)
    try:
        c1, i1 = _bridge.kmeans_plusplus(ds, 30, np.random.RandomState(1))
    finally:
        ds.close()
    c2, i2 = _bridge.kmeans_plusplus(X, 30, np.random.RandomState(1))
    np.testing.assert_array_equal(i1, i2)
    _, ref = oracle_pp(_exact_mean_centred(X), 30, np.random.RandomState(1))
    np.testing.assert_array_equal(i1, ref)


def test_plusplus_rejects_bad_arguments():
    X = np.zeros((10, 3), dtype=np.float32)
    with pytest.raises(ValueError):
        _bridge.kmeans_plusplus(X, 11, np.random.RandomState(0))
    with pytest.raises(RuntimeError):
        _bridge.kmeans_plusplus(X, 3, np.random.RandomState(0), n_local_trials=17)
