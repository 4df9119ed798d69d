"""The Python surface without a GPU (mirrors the reference's tests/test_accelerate.py
and tests/test_config.py for the KMeans path).

Routing, configuration and the estimator's refusals are host logic; none of
these tests launches a kernel.
"""

import numpy as np
import pytest
from sklearn.cluster import KMeans
from sklearn.linear_model import LinearRegression
from sklearn.pipeline import Pipeline
from sklearn.preprocessing import StandardScaler

import skmetal_b200 as skm
from skmetal_b200 import _bridge
from skmetal_b200._config import _get_device
from skmetal_b200.estimators.cluster import MetalKMeans


def test_accelerate_routes_kmeans_to_the_gpu_estimator():
    km = skm.accelerate(KMeans(n_clusters=4, n_init=1, random_state=0))
    assert isinstance(km, MetalKMeans)
    assert km.n_clusters == 4  # unknown attributes forward to the wrapped estimator


def test_accelerate_leaves_other_estimators_alone():
    lr = LinearRegression()
    assert skm.accelerate(lr) is lr


def test_accelerate_pipeline_factory_and_class():
    pipe = skm.accelerate(Pipeline([("s", StandardScaler()), ("km", KMeans(n_clusters=2))]))
    assert isinstance(pipe.steps[0][1], StandardScaler)
    assert isinstance(pipe.steps[1][1], MetalKMeans)

    @skm.accelerate
    def make():
        return KMeans(n_clusters=3)

    assert isinstance(make(), MetalKMeans)

    with pytest.warns(UserWarning):
        assert skm.accelerate(42) == 42


def test_accelerate_context_is_per_thread_and_restores():
    assert _get_device() == "gpu"
    with skm.accelerate_context(enabled=False):
        assert _get_device() == "cpu"
        with skm.accelerate_context(enabled=True):
            assert _get_device() == "gpu"
        assert _get_device() == "cpu"
    assert _get_device() == "gpu"


def test_config_setters_validate():
    skm.set_verbose(True)
    assert skm.get_config().verbose
    skm.set_threshold(123)
    assert skm.get_config().threshold == 123
    skm.update_threshold("KMeans", 5, 6)
    assert skm.get_config().thresholds["KMeans"] == (5, 6)
    skm.reset_thresholds()
    assert skm.get_config().thresholds["KMeans"] == (1, 1)
    skm.set_gpu(1)
    assert skm.get_config().gpu_index == 1
    with pytest.raises(ValueError):
        skm.set_device("tpu")
    with pytest.raises(ValueError):
        skm.set_dtype("float16")
    with pytest.raises(ValueError):
        skm.set_gpu(-1)


def test_forced_cpu_device_raises_instead_of_falling_back():
    X = np.random.default_rng(0).standard_normal((50, 3)).astype(np.float32)
    km = skm.accelerate(KMeans(n_clusters=2, n_init=1))
    skm.set_device("cpu")
    with pytest.raises(RuntimeError, match="no CPU path"):
        km.fit(X)


@pytest.mark.skipif(_bridge.GPU_AVAILABLE, reason="checks the behaviour without a GPU")
def test_fit_without_gpu_raises():
    X = np.random.default_rng(0).standard_normal((50, 3)).astype(np.float32)
    with pytest.raises(RuntimeError, match="requires a CUDA GPU"):
        skm.accelerate(KMeans(n_clusters=2, n_init=1)).fit(X)


def test_sample_weight_checks():
    """scikit-learn's _check_sample_weight rules on the host: None stays None
    (unit weights), a scalar broadcasts, the shape must be (n,), values must
    be finite; the library itself rejects negative and all-zero weights."""
    km = MetalKMeans(KMeans(n_clusters=2))
    assert km._check_weights(None, 5) is None
    np.testing.assert_array_equal(km._check_weights(2.0, 5), np.full(5, 2.0, np.float32))
    w = km._check_weights(np.arange(5.0), 5)
    assert w.dtype == np.float32 and w.flags["C_CONTIGUOUS"]
    with pytest.raises(ValueError):
        km._check_weights(np.ones(4), 5)
    with pytest.raises(ValueError):
        km._check_weights(np.array([1.0, np.nan, 1.0, 1.0, 1.0]), 5)
