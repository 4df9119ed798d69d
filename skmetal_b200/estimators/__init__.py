"""GPU estimators (KMeans only in this build)."""

from ._base import BaseGPUEstimator  # noqa: F401
from ._registry import GPU_REGISTRY  # noqa: F401
from .cluster import MetalKMeans  # noqa: F401

__all__ = ["BaseGPUEstimator", "GPU_REGISTRY", "MetalKMeans"]
