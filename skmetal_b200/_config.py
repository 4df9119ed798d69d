# Kept from the reference on purpose: the public interface and behaviour
# of skmetal/_config.py of abderahmane-ai/skmetal are the drop-in
# surface of the KMeans path, so its code is reused here, under the
# reference's licence:
#
# MIT License
#
# Copyright (c) 2026 Ainouche Abderahmane
#
# Permission is hereby granted, free of charge, to any person obtaining a copy
# of this software and associated documentation files (the "Software"), to deal
# in the Software without restriction, including without limitation the rights
# to use, copy, modify, merge, publish, distribute, sublicense, and/or sell
# copies of the Software, and to permit persons to whom the Software is
# furnished to do so, subject to the following conditions:
#
# The above copyright notice and this permission notice shall be included in all
# copies or substantial portions of the Software.
#
# THE SOFTWARE IS PROVIDED "AS IS", WITHOUT WARRANTY OF ANY KIND, EXPRESS OR
# IMPLIED, INCLUDING BUT NOT LIMITED TO THE WARRANTIES OF MERCHANTABILITY,
# FITNESS FOR A PARTICULAR PURPOSE AND NONINFRINGEMENT. IN NO EVENT SHALL THE
# AUTHORS OR COPYRIGHT HOLDERS BE LIABLE FOR ANY CLAIM, DAMAGES OR OTHER
# LIABILITY, WHETHER IN AN ACTION OF CONTRACT, TORT OR OTHERWISE, ARISING FROM,
# OUT OF OR IN CONNECTION WITH THE SOFTWARE OR THE USE OR OTHER DEALINGS IN THE
# SOFTWARE.

"""Configuration API (same surface as the reference's ``skmetal/_config.py``).

``Config`` is a lock-protected global with a thread-local device override set
by ``accelerate_context`` (``skmetal/_config.py:35-123``). The per-estimator
thresholds are kept for API compatibility; KMeans ignores them because this
build has no CPU path for it.
"""

import threading

PER_ESTIMATOR_THRESHOLDS: dict[str, tuple[int, int]] = {
    # KMeans always runs on the GPU here (thresholds are informational)
    "KMeans": (1, 1),
}


class Config:
    """Global configuration for GPU dispatch.

    Attributes
    ----------
    device : str
        ``"gpu"``, ``"cpu"`` or ``"auto"``. KMeans raises under ``"cpu"``.
    threshold : int
        Minimum ``n_samples * n_features`` for GPU dispatch (not applied to KMeans).
    dtype : str
        Compute dtype; only ``"float32"``.
    verbose : bool
        Print dispatch decisions and per-fit GPU timings.
    thresholds : dict
        Per-estimator ``(min_rows, min_cols)`` overrides.
    """

    def __init__(self, device: str = "gpu", threshold: int = 1, dtype: str = "float32", verbose: bool = False,
                 thresholds: dict | None = None):
        self._device = device
        self.threshold = threshold
        self.dtype = dtype
        self.verbose = verbose
        self.thresholds = thresholds if thresholds is not None else dict(PER_ESTIMATOR_THRESHOLDS)
        self.gpu_index = 0

    @property
    def device(self) -> str:
        val = getattr(_thread_local, "device", _UNSET)
        return self._device if val is _UNSET else val

    @device.setter
    def device(self, val: str):
        self._device = val

    def __repr__(self):
        return (f"device={self.device}, threshold={self.threshold}, verbose={self.verbose}, "
                f"gpu_index={self.gpu_index}")


_config = Config()
_lock = threading.Lock()
_thread_local = threading.local()
_UNSET = object()


def get_config() -> Config:
    return _config


def _get_device() -> str:
    val = getattr(_thread_local, "device", _UNSET)
    return _config._device if val is _UNSET else val


def _set_thread_device(device: str | None) -> None:
    if device is None:
        if hasattr(_thread_local, "device"):
            del _thread_local.device
    else:
        _thread_local.device = device


def set_device(device: str) -> None:
    """Set the global device preference (``"gpu"``, ``"cpu"`` or ``"auto"``)."""
    with _lock:
        if device not in ("gpu", "cpu", "auto"):
            raise ValueError("device must be 'gpu', 'cpu', or 'auto'")
        _config._device = device
        _thread_local.device = device


def set_threshold(threshold: int) -> None:
    with _lock:
        _config.threshold = int(threshold)


def set_dtype(dtype: str) -> None:
    with _lock:
        if dtype != "float32":
            raise ValueError("Only float32 is supported for GPU operations.")
        _config.dtype = dtype


def set_verbose(verbose: bool) -> None:
    with _lock:
        _config.verbose = bool(verbose)


def set_thresholds(thresholds: dict) -> None:
    with _lock:
        _config.thresholds = dict(thresholds)


def update_threshold(name: str, min_rows: int, min_cols: int) -> None:
    with _lock:
        _config.thresholds[name] = (min_rows, min_cols)


def reset_thresholds() -> None:
    with _lock:
        _config.thresholds = dict(PER_ESTIMATOR_THRESHOLDS)


def set_gpu(index: int) -> None:
    """Select the CUDA device used by estimators in this process."""
    with _lock:
        if int(index) < 0:
            raise ValueError("gpu index must be >= 0")
        _config.gpu_index = int(index)
