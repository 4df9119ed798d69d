"""skmetal_b200: B200 (sm_100a) implementation of skmetal's KMeans Lloyd path.

Drop-in for the reference's public surface for this path::

    import skmetal_b200 as skmetal
    from sklearn.cluster import KMeans

    km = skmetal.accelerate(KMeans(n_clusters=50, init=init, n_init=1))
    km.fit(X)           # Lloyd iterations on the GPU
    km.predict(X)       # assignment on the GPU
    km.transform(X)     # distances on the GPU

``accelerate`` wraps estimators, pipelines, classes and factories exactly like
``skmetal.accelerate``; KMeans is routed to the CUDA library
(``libskmetal_cuda.so``), which has no CPU fallback.
"""

from ._about import __version__, __version_info__
from ._bridge import CUDA_AVAILABLE, GPU_AVAILABLE, METAL_AVAILABLE
from ._config import (
    get_config,
    reset_thresholds,
    set_device,
    set_dtype,
    set_gpu,
    set_threshold,
    set_thresholds,
    set_verbose,
    update_threshold,
)
from .accelerate import accelerate, accelerate_context


def device_info() -> dict:
    """Name and memory of the current CUDA device (raises without a GPU)."""
    from ._bridge import device_info as _di

    if not GPU_AVAILABLE:
        raise RuntimeError("skmetal_b200: device_info() requires a CUDA GPU; none is visible.")
    return _di()


__all__ = [
    "__version__",
    "__version_info__",
    "CUDA_AVAILABLE",
    "GPU_AVAILABLE",
    "METAL_AVAILABLE",
    "accelerate",
    "accelerate_context",
    "device_info",
    "get_config",
    "set_device",
    "set_gpu",
    "set_threshold",
    "set_dtype",
    "set_verbose",
    "set_thresholds",
    "update_threshold",
    "reset_thresholds",
]
