"""Type-exact dispatch from scikit-learn estimators to GPU implementations.

Mirrors ``skmetal/_dispatch.py:9-59`` without the MLX installation hint:
KMeans is always routed to ``MetalKMeans``.
"""

import warnings

from sklearn.pipeline import Pipeline

from ._config import get_config
from .estimators._registry import GPU_REGISTRY


def _is_supported(estimator) -> bool:
    return type(estimator) in GPU_REGISTRY


def _get_gpu_impl(estimator):
    mod_name, cls_name = GPU_REGISTRY[type(estimator)]
    try:
        mod = __import__(mod_name, fromlist=[cls_name])
        return getattr(mod, cls_name)
    except (ImportError, AttributeError) as e:
        raise ImportError(
            f"GPU_REGISTRY entry for {type(estimator).__name__} points to "
            f"'{mod_name}.{cls_name}' but could not import/retrieve it: {e}"
        ) from e


def _wrap_estimator(estimator):
    """Wrap ``estimator`` with its GPU implementation (returned unchanged if none)."""
    if not _is_supported(estimator):
        if get_config().verbose:
            warnings.warn(f"No GPU accelerator for {type(estimator).__name__}. Using CPU.", stacklevel=3)
        return estimator
    return _get_gpu_impl(estimator)(estimator)


def _wrap_pipeline(pipeline):
    steps = [(name, _wrap_estimator(est)) for name, est in pipeline.steps]
    return Pipeline(steps, memory=pipeline.memory, verbose=pipeline.verbose)
