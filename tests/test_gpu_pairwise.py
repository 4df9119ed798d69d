"""skmetal_pairwise_distance on the GPU through the C ABI.

The first two cases are the reference's own kernel tests
(tests/test_kernels.py:26-37: identity and symmetry on 3 x 2 inputs); the
others hold the device result to the same expanded formula evaluated in
float64 on the host, at shapes that cover partial tiles, both store paths
(n a multiple of 4 or not) and more than one 16-column slice of X."""

import numpy as np
import pytest

from skmetal_b200 import _bridge

pytestmark = pytest.mark.gpu


def _expanded_f64(X):
    X64 = X.astype(np.float64)
    nrm = np.einsum("ij,ij->i", X64, X64)
    return np.maximum(nrm[:, None] + nrm[None, :] - 2.0 * (X64 @ X64.T), 0.0), nrm


def test_pairwise_distance_identity():
    X = np.array([[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]], dtype=np.float32)
    D = _bridge.pairwise_distance(X)
    assert D.shape == (3, 3)
    np.testing.assert_allclose(np.diag(D), [0.0, 0.0, 0.0], atol=1e-5)
    np.testing.assert_allclose(D[0, 1], 2.0, rtol=1e-5)
    np.testing.assert_allclose(D[0, 2], 1.0, rtol=1e-5)


def test_pairwise_distance_symmetric():
    X = np.array([[0.0, 0.0], [3.0, 4.0], [1.0, 2.0]], dtype=np.float32)
    D = _bridge.pairwise_distance(X)
    assert np.allclose(D, D.T, rtol=1e-5), "Distance matrix must be symmetric"


@pytest.mark.parametrize("n,d", [(1, 5), (129, 3), (300, 37), (1024, 100), (1001, 130)])
def test_pairwise_matches_float64(n, d):
    rng = np.random.default_rng(n * 1000 + d)
    X = rng.normal(size=(n, d)).astype(np.float32) * rng.uniform(0.5, 4.0, size=(1, d)).astype(np.float32)
    D = _bridge.pairwise_distance(X)
    ref, nrm = _expanded_f64(X)
    # float32 norms and dot products: error below a few ulps of the norms
    tol = 8 * d * np.finfo(np.float32).eps * (nrm[:, None] + nrm[None, :]) + 1e-6
    err = np.abs(D.astype(np.float64) - ref)
    assert np.all(err <= tol), float(np.max(err / tol))
    # every entry of the transposed half is the same float32 value
    assert np.array_equal(D, D.T)
    assert np.all(D >= 0)


def test_pairwise_rejects_bad_input():
    with pytest.raises(TypeError):
        _bridge.pairwise_distance(np.zeros((4, 3), dtype=np.float64))
    with pytest.raises(TypeError):
        _bridge.pairwise_distance(np.zeros((4, 3), dtype=np.float32)[:, :2])
