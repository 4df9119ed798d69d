# Kept from the reference on purpose: the public interface and behaviour
# of skmetal/accelerate.py of abderahmane-ai/skmetal are the drop-in
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

"""``accelerate`` decorator / wrapper and ``accelerate_context``.

Same behaviour as the reference (``skmetal/accelerate.py:17-113``): wraps an
estimator, a Pipeline, an estimator class or a factory function.
"""

from __future__ import annotations

import threading
import warnings
from functools import wraps
from typing import Any

from sklearn.pipeline import Pipeline

from ._config import _get_device, _set_thread_device
from ._dispatch import _wrap_estimator, _wrap_pipeline

_local = threading.local()


def accelerate(obj: Any | None = None) -> Any:
    """Enable GPU acceleration for scikit-learn estimators.

    Decorator or call::

        @accelerate
        def model():
            return KMeans(n_clusters=8)

        model = accelerate(KMeans(n_clusters=8))
    """
    if obj is None:
        return _Accelerator()
    return _Accelerator()(obj)


class _Accelerator:
    @staticmethod
    def _wrap_class(cls: type) -> type:
        orig_new = cls.__new__
        orig_init = cls.__init__

        @wraps(orig_new)
        def new_new(cls2, *args, **kwargs):
            if args and isinstance(args[0], Pipeline):
                return _wrap_pipeline(args[0])
            if args and hasattr(args[0], "fit"):
                return _wrap_estimator(args[0])
            if orig_new is not object.__new__:
                return orig_new(cls2)
            return super(cls, cls2).__new__(cls2)

        @wraps(orig_init)
        def new_init(self, *args, **kwargs):
            if args and hasattr(args[0], "fit"):
                return
            orig_init(self, *args, **kwargs)

        cls.__new__ = new_new
        cls.__init__ = new_init
        return cls

    def __call__(self, obj: Any) -> Any:
        if isinstance(obj, Pipeline):
            return _wrap_pipeline(obj)
        if isinstance(obj, type):
            return self._wrap_class(obj)
        if hasattr(obj, "fit"):
            return _wrap_estimator(obj)
        if callable(obj):

            @wraps(obj)
            def wrapper(*args, **kwargs):
                result = obj(*args, **kwargs)
                if isinstance(result, Pipeline):
                    return _wrap_pipeline(result)
                if hasattr(result, "fit"):
                    return _wrap_estimator(result)
                return result

            return wrapper
        warnings.warn(f"accelerate: {type(obj).__name__} is not a recognized estimator.")
        return obj


class accelerate_context:
    """Temporarily enable/disable acceleration; per-thread device stack."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled

    def __enter__(self):
        if not hasattr(_local, "device_stack"):
            _local.device_stack = []
        _local.device_stack.append(_get_device())
        _set_thread_device("gpu" if self.enabled else "cpu")
        return self

    def __exit__(self, *args):
        if hasattr(_local, "device_stack") and _local.device_stack:
            _set_thread_device(_local.device_stack.pop())
