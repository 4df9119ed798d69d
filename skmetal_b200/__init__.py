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


def __getattr__(name: str):
    # CUDA_AVAILABLE / GPU_AVAILABLE / METAL_AVAILABLE load the native library
    # on first access (importing the package maps no native code)
    if name in ("CUDA_AVAILABLE", "GPU_AVAILABLE", "METAL_AVAILABLE"):
        from . import _bridge

        return getattr(_bridge, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def device_info() -> dict:
    """Name and memory of the current CUDA device (raises without a GPU)."""
    from . import _bridge

    if not _bridge.GPU_AVAILABLE:
        raise RuntimeError("skmetal_b200: device_info() requires a CUDA GPU; none is visible.")
    return _bridge.device_info()


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
