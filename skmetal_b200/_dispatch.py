# Kept from the reference on purpose: the public interface and behaviour
# of skmetal/_dispatch.py of abderahmane-ai/skmetal are the drop-in
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
