"""skmetal_kmeans_update_centers_noalloc against skmetal_kmeans_lloyd_iter.

The no-allocation centroid update keeps its scratch in one static device array
per device. These tests call it through the C ABI on device buffers owned by
the test and compare it with the fit engine's own M-step on consecutive calls,
so a scratch that was not cleared between calls would show up. The file is
named to be collected last: it must pass on its own in a fresh process and
after every other GPU test in the same process.
"""
import ctypes

import numpy as np
import pytest

from skmetal_b200 import _bridge
from skmetal_b200._synthetic import gaussian_mixture

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 2097152  # SKMETAL_NOALLOC_SCRATCH_BYTES


def _torch():
    import torch

    return torch


def _noalloc(X_t, labels_t, k, centers_t, weight_t):
    n, d = X_t.shape
    f = _bridge._fn("skmetal_kmeans_update_centers_noalloc")
    rc = f(ctypes.c_void_p(X_t.data_ptr()), ctypes.c_void_p(labels_t.data_ptr()), n, d, k,
           ctypes.c_void_p(centers_t.data_ptr()),
           ctypes.c_void_p(weight_t.data_ptr()) if weight_t is not None else None, None)
    return rc


def _problem(n, d, k, seed):
    X, _ = gaussian_mixture(n, d, k, seed=seed)
    rng = np.random.default_rng(seed + 100)
    init = np.ascontiguousarray(X[rng.choice(n, k, replace=False)])
    labels, centers_new, weight, _ = _bridge.kmeans_lloyd_iter(X, init)
    assert (weight > 0).all(), "problem must have no empty cluster"
    return X, init, labels, centers_new, weight


def _check_against_lloyd_iter(prob):
    torch = _torch()
    X, init, labels, centers_new, weight = prob
    X_t = torch.from_numpy(X).cuda()
    lab_t = torch.from_numpy(labels.astype(np.int32)).cuda()
    cen_t = torch.from_numpy(init).cuda()
    w_t = torch.full((init.shape[0],), -1.0, dtype=torch.float32, device="cuda")
    rc = _noalloc(X_t, lab_t, init.shape[0], cen_t, w_t)
    assert rc == 0, _bridge._last_error()
    got = cen_t.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), centers_new.view(np.uint32))
    assert np.array_equal(w_t.cpu().numpy(), weight)


def test_noalloc_matches_lloyd_iter_on_consecutive_calls():
    a = _problem(20000, 20, 16, seed=11)
    b = _problem(30000, 13, 40, seed=12)  # d not a multiple of 4, more clusters
    for prob in (a, b, a):
        _check_against_lloyd_iter(prob)


def test_noalloc_leaves_empty_clusters_and_matches_exact_means():
    torch = _torch()
    n, d, k = 5000, 7, 6
    X, _ = gaussian_mixture(n, d, k, seed=21)
    labels = (np.arange(n) % (k - 1)).astype(np.int32)  # cluster k-1 gets no rows
    prev = np.full((k, d), 3.25, dtype=np.float32)
    X_t = torch.from_numpy(X).cuda()
    lab_t = torch.from_numpy(labels).cuda()
    cen_t = torch.from_numpy(prev.copy()).cuda()
    w_t = torch.zeros(k, dtype=torch.float32, device="cuda")
    for _ in range(2):
        assert _noalloc(X_t, lab_t, k, cen_t, w_t) == 0, _bridge._last_error()
        got = cen_t.cpu().numpy()
        w = w_t.cpu().numpy()
        assert np.array_equal(got[k - 1], prev[k - 1])
        assert w[k - 1] == 0.0
        for c in range(k - 1):
            rows = X[labels == c].astype(np.float64)
            assert w[c] == rows.shape[0]
            np.testing.assert_allclose(got[c], rows.mean(axis=0), rtol=1e-6, atol=1e-6)


def test_noalloc_rejects_sizes_beyond_the_scratch():
    torch = _torch()
    k = 4096
    d = SCRATCH_BYTES // 8 // k  # k * (d + 1) > 262143
    X_t = torch.zeros((4, d), dtype=torch.float32, device="cuda")
    lab_t = torch.zeros(4, dtype=torch.int32, device="cuda")
    cen_t = torch.zeros((k, d), dtype=torch.float32, device="cuda")
    rc = _noalloc(X_t, lab_t, k, cen_t, None)
    assert rc == 1
    assert "static scratch" in _bridge._last_error()


def test_noalloc_rejects_labels_out_of_range_without_writing():
    torch = _torch()
    n, d, k = 1000, 8, 4
    X, _ = gaussian_mixture(n, d, k, seed=31)
    labels = (np.arange(n) % k).astype(np.int32)
    labels[17] = k
    X_t = torch.from_numpy(X).cuda()
    lab_t = torch.from_numpy(labels).cuda()
    cen_t = torch.full((k, d), 1.5, dtype=torch.float32, device="cuda")
    assert _noalloc(X_t, lab_t, k, cen_t, None) == 1
    assert "outside" in _bridge._last_error()
    assert bool((cen_t == 1.5).all())
    # the next valid call on the same scratch is unaffected
    labels[17] = 0
    lab_t.copy_(torch.from_numpy(labels))
    assert _noalloc(X_t, lab_t, k, cen_t, None) == 0, _bridge._last_error()
    for c in range(k):
        np.testing.assert_allclose(cen_t[c].cpu().numpy(), X[labels == c].astype(np.float64).mean(axis=0),
                                   rtol=1e-6, atol=1e-6)
