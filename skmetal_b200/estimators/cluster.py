"""GPU KMeans (the estimator the Lloyd hot path lives behind).

Replaces ``MetalKMeans`` of the reference (``skmetal/estimators/cluster.py:18-146``)
with scikit-learn's ``KMeans.fit`` semantics (``sklearn/cluster/_kmeans.py:1436-1562``)
run on the CUDA library:

* the init is honoured: an explicit array is used as given; ``"k-means++"``
  is seeded on the GPU (scikit-learn's greedy k-means++ on the centred rows,
  drawing from the same random stream in the same order; the cumulative
  sums and potentials are float64 where scikit-learn's are float32, so on
  large inputs a candidate row can differ); ``"random"`` and callables are
  drawn with scikit-learn's own initialisation routine and random stream;
* ``n_init`` restarts keep scikit-learn's best-run rule (lower inertia and
  not the same clustering up to a permutation);
* ``sample_weight`` weights the sums, the cluster weights (a cluster of
  weight zero is empty), the seeding and the inertia, as scikit-learn's
  weighted Lloyd does (one GPU);
* the Lloyd loop, the final E-step, the inertia, ``predict``, ``transform``,
  ``fit_predict``, ``fit_transform`` and ``score`` run on the GPU;
* there is no CPU fallback: without a GPU, or under ``set_device("cpu")``,
  the estimator raises.
"""

from __future__ import annotations

import time
import warnings

import numpy as np
from sklearn.exceptions import ConvergenceWarning
from sklearn.utils import check_random_state
from sklearn.utils.validation import check_array, check_is_fitted

from .. import _bridge
from .._config import _get_device, get_config
from ._base import BaseGPUEstimator

try:  # scikit-learn's helper for the n_init best-run rule
    from sklearn.cluster._k_means_common import _is_same_clustering
except Exception:  # noqa: BLE001
    _is_same_clustering = None


def _gpu_call(fn, *args, **kwargs):
    """A library call; its report of NaN or infinity in the input becomes
    scikit-learn's ValueError."""
    try:
        return fn(*args, **kwargs)
    except RuntimeError as e:
        if "NaN or infinity" in str(e):
            raise ValueError(f"Input X contains NaN or infinity ({e}).") from None
        raise


def _same_clustering(a: np.ndarray, b: np.ndarray, k: int) -> bool:
    if _is_same_clustering is not None:
        return bool(_is_same_clustering(a.astype(np.int32), b.astype(np.int32), k))
    mapping = np.full(k, -1)
    for x, y in zip(a, b):
        if mapping[x] == -1:
            mapping[x] = y
        elif mapping[x] != y:
            return False
    return True


class MetalKMeans(BaseGPUEstimator):
    """KMeans whose Lloyd iterations, assignment and distances run on the GPU."""

    # ------------------------------------------------------------------ helpers
    def _require_gpu(self, X):
        if not self._should_use_gpu(X):
            raise RuntimeError(
                "skmetal_b200 KMeans has no CPU path: device is set to 'cpu' (set_device / "
                "accelerate_context). Use sklearn.cluster.KMeans directly for CPU execution.")
        if not _bridge.GPU_AVAILABLE:
            raise RuntimeError("skmetal_b200 KMeans requires a CUDA GPU (none visible; no CPU fallback)")
        _bridge.set_device(get_config().gpu_index)

    def _check_weights(self, sample_weight, n):
        """float32 weights of the n rows (scikit-learn's _check_sample_weight
        rules: a scalar broadcasts, shape (n,), finite), or None for unit
        weights. The library rejects negative weights and an all-zero set."""
        if sample_weight is None:
            return None
        w = np.asarray(sample_weight, dtype=np.float32)
        if w.ndim == 0:
            w = np.full(n, float(w), dtype=np.float32)
        if w.shape != (n,):
            raise ValueError(f"sample_weight.shape == {w.shape}, expected ({n},)!")
        if not np.all(np.isfinite(w)):
            raise ValueError("Input sample_weight contains NaN or infinity.")
        return np.ascontiguousarray(w)

    # ---------------------------------------------------------------------- fit
    def fit(self, X, y=None, sample_weight=None):
        est = self._estimator
        est._validate_params()
        X = self._validate_data(X)[0]
        self._require_gpu(X)
        n, d = X.shape
        k = int(est.n_clusters)
        if n < k:
            raise ValueError(f"n_samples={n} should be >= n_clusters={k}.")
        sw = self._check_weights(sample_weight, n)

        init = est.init
        init_is_array = hasattr(init, "__array__") or isinstance(init, (list, tuple))
        if est.n_init == "auto":
            n_init = 1 if (init_is_array or (isinstance(init, str) and init == "k-means++")) else 10
        else:
            n_init = int(est.n_init)
        if init_is_array:
            init = check_array(init, dtype=np.float32, order="C", copy=True)
            if init.shape != (k, d):
                raise ValueError(f"The shape of the initial centers {init.shape} does not match "
                                 f"the number of clusters {k} and features {d}.")
            if n_init != 1:
                warnings.warn("Explicit initial center position passed: performing only one init in "
                              f"KMeans instead of n_init={n_init}.", RuntimeWarning, stacklevel=2)
                n_init = 1
        random_state = check_random_state(est.random_state)
        if isinstance(init, str) and init == "k-means++":
            return self._fit_plusplus(X, k, n_init, random_state, sw, t0=time.perf_counter())

        # scikit-learn draws the other non-array inits on the centred data
        Xc = x_sq = mean = None
        if not init_is_array:
            mean = X.mean(axis=0)
            Xc = X - mean
            x_sq = np.einsum("ij,ij->i", Xc, Xc)
        ones = np.ones(n, dtype=np.float32) if sw is None else sw

        t0 = time.perf_counter()
        best = None
        for _ in range(n_init):
            if init_is_array:
                centers_init = init
            else:
                centers_init = est._init_centroids(Xc, x_squared_norms=x_sq, init=init,
                                                   random_state=random_state, sample_weight=ones)
                centers_init = np.ascontiguousarray((centers_init + mean).astype(np.float32))
            centers, labels, inertia, n_iter = _gpu_call(
                _bridge.kmeans_fit, X, centers_init, int(est.max_iter), float(est.tol), center=True, sample_weight=sw)
            if best is None or (inertia < best[2] and not _same_clustering(labels, best[1], k)):
                best = (centers, labels, inertia, n_iter, _bridge.last_fit_distinct())
        self._finish_fit(best, n, d, k, n_init, t0)
        return self

    def _fit_plusplus(self, X, k, n_init, random_state, sw, t0):
        """init="k-means++": every restart seeds on the GPU (scikit-learn's
        greedy k-means++ on the centred rows, drawing from ``random_state`` in
        scikit-learn's order) and fits from there; X is uploaded once."""
        est = self._estimator
        n, d = X.shape
        ds = _gpu_call(_bridge.Dataset, X)
        try:
            best = None
            for _ in range(n_init):
                centers_init, _ = _gpu_call(_bridge.kmeans_plusplus, ds, k, random_state, sample_weight=sw)
                labels = np.empty(n, dtype=np.int32)
                centers, inertia, n_iter = _gpu_call(ds.fit, centers_init, int(est.max_iter), float(est.tol),
                                                     labels_out=labels, sample_weight=sw)
                if best is None or (inertia < best[2] and not _same_clustering(labels, best[1], k)):
                    best = (centers, labels, inertia, n_iter, _bridge.last_fit_distinct())
        finally:
            ds.close()
        self._finish_fit(best, n, d, k, n_init, t0)
        return self

    def _finish_fit(self, best, n, d, k, n_init, t0):
        est = self._estimator
        centers, labels, inertia, n_iter, distinct = best
        if distinct < 0:  # not counted by the library
            distinct = int(np.count_nonzero(np.bincount(labels, minlength=k)))
        if distinct < k:
            warnings.warn(f"Number of distinct clusters ({distinct}) found smaller than "
                          f"n_clusters ({k}). Possibly due to duplicate points in X.", ConvergenceWarning,
                          stacklevel=2)
        est.cluster_centers_ = centers
        est._n_features_out = k
        est.labels_ = labels
        est.inertia_ = float(inertia)
        est.n_iter_ = int(n_iter)
        est.n_features_in_ = d
        est._n_threads = 1
        est._tol = float(est.tol)
        est._n_init = n_init
        est._algorithm = "lloyd"
        self._fitted = True
        if get_config().verbose:
            st = _bridge.last_fit_stats()
            print(f"[skmetal] KMeans: {n}x{d} k={k} n_init={n_init} n_iter={n_iter} "
                  f"wall={time.perf_counter() - t0:.4f}s gpu_loop={st['ms_loop']:.3f}ms "
                  f"({st['ms_loop'] / max(1, st['iterations']):.4f} ms/iter)")

    # ------------------------------------------------------------------ inference
    def _centers(self):
        check_is_fitted(self._estimator, "cluster_centers_")
        return np.ascontiguousarray(self._estimator.cluster_centers_, dtype=np.float32)

    def _check_test(self, X):
        # non-finite values are detected on the device (the library raises)
        X = check_array(X, dtype=np.float32, order="C", ensure_all_finite=False)
        if X.shape[1] != self._estimator.n_features_in_:
            raise ValueError(f"X has {X.shape[1]} features, but KMeans is expecting "
                             f"{self._estimator.n_features_in_} features as input.")
        self._require_gpu(X)
        return X

    def predict(self, X):
        C = self._centers()
        X = self._check_test(X)
        labels = np.empty(X.shape[0], dtype=np.int32)
        _gpu_call(_bridge.kmeans_assign, X, C, labels, X.shape[0], X.shape[1], C.shape[0])
        return labels

    def transform(self, X):
        C = self._centers()
        X = self._check_test(X)
        return _gpu_call(_bridge.kmeans_transform, X, C)

    def fit_predict(self, X, y=None, sample_weight=None):
        return self.fit(X, sample_weight=sample_weight)._estimator.labels_

    def fit_transform(self, X, y=None, sample_weight=None):
        return self.fit(X, sample_weight=sample_weight).transform(X)

    def score(self, X, y=None, sample_weight=None):
        C = self._centers()
        X = self._check_test(X)
        sw = self._check_weights(sample_weight, X.shape[0])
        labels = self.predict(X)
        if sw is not None:
            return -_gpu_call(_bridge.kmeans_inertia_weighted, X, C, labels, sw, X.shape[0], X.shape[1], C.shape[0])
        return -_gpu_call(_bridge.kmeans_inertia, X, C, labels, X.shape[0], X.shape[1], C.shape[0])
