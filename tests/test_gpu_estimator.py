"""The public API on the GPU: ``skmetal_b200.accelerate(KMeans(...))``.

Ports of the reference's own KMeans cases, run against this package's
estimator (the reference compares its accelerated estimator with
scikit-learn's CPU one; here the GPU path is the one under test):

* ``tests/test_correctness.py:139-170`` -- fitted attributes against
  scikit-learn (rtol 1e-3, atol 1e-4; centres Hungarian-matched, ``labels_``
  unpermuted; ``n_iter_`` and ``n_features_in_`` skipped);
* ``tests/test_comprehensive.py:127-138`` (per-estimator threshold), ``:160-197``
  (``n_init``), ``:319-336`` (k > n, empty clusters), ``:360-384`` (transformer
  API), ``:409-419`` (refit), ``:549`` (attributes);
* ``tests/test_large_matrix.py:206-216`` (100k x 50, k = 20) and ``:326-329``.

Plus what the port adds: NaN input raises scikit-learn's ``ValueError``
(detected on the device), and X in pageable and in page-locked host memory
give the same bits (the staged upload)."""

import numpy as np
import pytest
from sklearn import datasets
from sklearn.cluster import KMeans

import skmetal_b200 as skmetal
from skmetal_b200 import _bridge
from skmetal_b200._config import get_config

pytestmark = pytest.mark.gpu


def _match_clusters(gpu_centers, cpu_centers):
    from scipy.optimize import linear_sum_assignment
    from sklearn.metrics import pairwise_distances

    row_ind, col_ind = linear_sum_assignment(pairwise_distances(gpu_centers, cpu_centers))
    out = np.empty_like(gpu_centers)
    out[col_ind] = gpu_centers[row_ind]
    return out


def _check_attrs(gpu_obj, cpu_obj, rtol=1e-3, atol=1e-4):
    skip = {"n_iter_", "n_features_in_", "n_features_out_"}
    checked = []
    for attr in dir(cpu_obj):
        if attr.startswith("_") or attr in skip or not attr.endswith("_"):
            continue
        g, c = getattr(gpu_obj, attr, None), getattr(cpu_obj, attr, None)
        if g is None or c is None or callable(g) or isinstance(g, str):
            continue
        if isinstance(g, np.ndarray):
            if attr == "cluster_centers_":
                g = _match_clusters(g, c)
            np.testing.assert_allclose(g, c, rtol=rtol, atol=atol, err_msg=attr)
        else:
            assert abs(g - c) <= atol + rtol * abs(c), attr
        checked.append(attr)
    return checked


def test_estimator_correctness_kmeans():
    """test_correctness.py:139-170, the KMeans row: make_blobs(2000, 10 centres,
    50 features, random_state=42), KMeans(random_state=42)."""
    X, _ = datasets.make_blobs(n_samples=2000, centers=10, n_features=50, random_state=42)
    X = X.astype(np.float32)
    cpu = KMeans(random_state=42).fit(X)
    gpu = skmetal.accelerate(KMeans(random_state=42))
    gpu.fit(X)
    assert type(gpu).__name__ == "MetalKMeans"
    checked = _check_attrs(gpu._estimator, cpu)
    assert {"cluster_centers_", "labels_", "inertia_"} <= set(checked)


def test_per_estimator_threshold_still_fits():
    """test_comprehensive.py:127-138: the reference routes to its CPU path
    under a huge per-estimator threshold; this build has no CPU path for
    KMeans and must still produce results."""
    thresh = get_config().thresholds
    thresh["KMeans"] = (10**9, 10**9)
    get_config().thresholds = thresh
    X, _ = datasets.make_classification(n_samples=2000, n_features=50, n_classes=2, random_state=42)
    model = skmetal.accelerate(KMeans(n_clusters=5, random_state=42, n_init=1))
    model.fit(X.astype(np.float32))
    assert model.cluster_centers_.shape == (5, 50)


@pytest.mark.parametrize("init", ["k-means++", "random"])
def test_n_init_auto(init):
    """test_comprehensive.py:160-174; n_init='auto' resolves like scikit-learn."""
    X, _ = datasets.make_blobs(n_samples=2000, n_features=10, centers=5, random_state=42)
    X = X.astype(np.float32)
    model = skmetal.accelerate(KMeans(n_clusters=5, init=init, n_init="auto", random_state=42))
    model.fit(X)
    cpu = KMeans(n_clusters=5, init=init, n_init="auto", random_state=42).fit(X)
    assert model.cluster_centers_.shape == (5, 10)
    assert model._n_init == cpu._n_init
    assert model.inertia_ == pytest.approx(cpu.inertia_, rel=1e-5)


def test_n_init_multiple_deterministic():
    """test_comprehensive.py:176-185."""
    X, _ = datasets.make_blobs(n_samples=2000, n_features=10, centers=5, random_state=42)
    X = X.astype(np.float32)
    m1 = skmetal.accelerate(KMeans(n_clusters=5, random_state=42, n_init=3)).fit(X)
    m2 = skmetal.accelerate(KMeans(n_clusters=5, random_state=42, n_init=3)).fit(X)
    assert np.array_equal(m1.labels_, m2.labels_)
    np.testing.assert_array_equal(m1.cluster_centers_, m2.cluster_centers_)


def test_k_greater_than_n_raises():
    """test_comprehensive.py:319-326 (scikit-learn raises for k > n)."""
    X = np.random.default_rng(0).standard_normal((5, 10)).astype(np.float32)
    with pytest.raises(ValueError):
        skmetal.accelerate(KMeans(n_clusters=10, random_state=42, n_init=1)).fit(X)


def test_empty_cluster_recovery():
    """test_comprehensive.py:328-336: k = 20 on 5 blobs, and the same result
    as scikit-learn from the same initial centres."""
    X, _ = datasets.make_blobs(n_samples=1000, n_features=10, centers=5, random_state=42)
    X = X.astype(np.float32)
    model = skmetal.accelerate(KMeans(n_clusters=20, random_state=42, n_init=1))
    model.fit(X)
    assert len(np.unique(model.labels_)) <= 20
    assert model.cluster_centers_.shape == (20, 10)
    cpu = KMeans(n_clusters=20, random_state=42, n_init=1).fit(X)
    assert model.inertia_ == pytest.approx(cpu.inertia_, rel=1e-4)


def test_fit_predict_equals_labels():
    """test_comprehensive.py:360-366."""
    X, _ = datasets.make_blobs(n_samples=500, n_features=10, centers=5, random_state=42)
    X = X.astype(np.float32)
    model = skmetal.accelerate(KMeans(n_clusters=5, random_state=42, n_init=1))
    labels = model.fit_predict(X)
    assert labels.shape == (500,)
    assert np.array_equal(labels, model.labels_)
    assert np.array_equal(model.predict(X), model.labels_)


def test_fit_transform():
    """test_comprehensive.py:368-384: shape, non-negative, fit_transform ==
    transform after fit (rtol 1e-5), and equal to scikit-learn's transform."""
    X, _ = datasets.make_blobs(n_samples=500, n_features=10, centers=5, random_state=42)
    X = X.astype(np.float32)
    model = skmetal.accelerate(KMeans(n_clusters=5, random_state=42, n_init=1))
    dists_ft = model.fit_transform(X)
    assert dists_ft.shape == (500, 5) and np.all(dists_ft >= 0)
    model.fit(X)
    dists_t = model.transform(X)
    np.testing.assert_allclose(dists_ft, dists_t, rtol=1e-5, atol=1e-6)
    cpu = KMeans(n_clusters=5, random_state=42, n_init=1).fit(X)
    np.testing.assert_allclose(dists_t, cpu.transform(X), rtol=1e-4, atol=1e-4)
    assert model.score(X) == pytest.approx(cpu.score(X), rel=1e-5)


def test_refit_changes_centres():
    """test_comprehensive.py:409-419."""
    X1, _ = datasets.make_blobs(n_samples=200, n_features=10, centers=5, random_state=42)
    X2, _ = datasets.make_blobs(n_samples=200, n_features=10, centers=5, random_state=99)
    model = skmetal.accelerate(KMeans(n_clusters=5, random_state=42, n_init=1))
    model.fit(X1.astype(np.float32))
    c1 = model.cluster_centers_.copy()
    model.fit(X2.astype(np.float32))
    assert not np.allclose(c1, model.cluster_centers_, rtol=1e-3)


def test_attributes_present():
    """test_comprehensive.py:549."""
    X, _ = datasets.make_classification(n_samples=500, n_features=20, n_classes=2, random_state=42)
    model = skmetal.accelerate(KMeans(random_state=42)).fit(X.astype(np.float32))
    for attr in ["cluster_centers_", "labels_", "inertia_", "n_iter_", "n_features_in_"]:
        assert hasattr(model, attr), attr


def test_large_kmeans_fit_and_transform():
    """test_large_matrix.py:206-216 (100k x 50, k = 20) and :326-329."""
    X, _ = datasets.make_blobs(n_samples=100_000, n_features=50, centers=20, random_state=42)
    X = X.astype(np.float32)
    model = skmetal.accelerate(KMeans(n_clusters=20, random_state=42, n_init=1))
    model.fit(X)
    assert len(np.unique(model.labels_)) >= 19
    assert model.cluster_centers_.shape == (20, 50)
    assert np.all(np.isfinite(model.cluster_centers_))
    dists = model.transform(X[:1000])
    assert dists.shape == (1000, 20) and np.all(dists >= 0)
    cpu = KMeans(n_clusters=20, random_state=42, n_init=1).fit(X)
    assert model.inertia_ == pytest.approx(cpu.inertia_, rel=1e-4)


def test_nan_input_raises_value_error():
    """NaN is found on the device (the host does not scan X) and raised as
    scikit-learn's ValueError, by fit and by predict."""
    X, _ = datasets.make_blobs(n_samples=300, n_features=6, centers=3, random_state=0)
    X = X.astype(np.float32)
    model = skmetal.accelerate(KMeans(n_clusters=3, random_state=0, n_init=1)).fit(X)
    bad = X.copy()
    bad[17, 3] = np.nan
    with pytest.raises(ValueError):
        model.predict(bad)
    with pytest.raises(ValueError):
        skmetal.accelerate(KMeans(n_clusters=3, random_state=0, n_init=1)).fit(bad)
    bad[17, 3] = np.inf
    with pytest.raises(ValueError):
        model.transform(bad)


@pytest.mark.parametrize("d", [32, 37])
def test_pageable_and_pinned_uploads_agree(d):
    """X of 24-28 MB in ordinary host memory goes through the library's
    pinned staging ring (several chunks, d = 37: padded rows); the same
    bytes page-locked go directly. The fits must be bit-identical."""
    import torch

    from skmetal_b200._synthetic import gaussian_mixture

    X, init = gaussian_mixture(190_000, d, 12, seed=d)
    a = _bridge.kmeans_fit(X, init, 15, 0.0)
    Xp = torch.empty(X.shape, dtype=torch.float32, pin_memory=True).numpy()
    Xp[...] = X
    b = _bridge.kmeans_fit(Xp, init, 15, 0.0)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert a[2] == b[2] and a[3] == b[3]
    # predict from pageable memory (the assignment kernel, direct differences
    # on X as given): the fit's final labels up to near-ties
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).parent))
    from parity import check_labels

    lab = np.empty(X.shape[0], dtype=np.int32)
    _bridge.kmeans_assign(X, a[0], lab, X.shape[0], d, 12)
    check_labels(X, a[0], lab, a[1], "predict vs fit labels")
