# Kept from the reference on purpose: the wrapper contract of
# skmetal/estimators/_base.py of abderahmane-ai/skmetal is the drop-in surface
# of the KMeans path, so its code is reused here (without the CPU fallback),
# under the reference's licence:
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

"""Base wrapper for GPU estimators (``skmetal/estimators/_base.py:7-89``).

The wrapper holds the scikit-learn estimator in ``_estimator``, validates
input to C-contiguous float32, and forwards unknown attributes to the wrapped
estimator so fitted attributes read the same as on scikit-learn.
"""

import numpy as np
from sklearn.base import BaseEstimator
from sklearn.utils.validation import check_array

from .._config import _get_device, get_config


class BaseGPUEstimator(BaseEstimator):
    _estimator: BaseEstimator | None

    def __init__(self, _estimator=None):
        self._estimator = _estimator
        self._fitted = False

    def _validate_data(self, X, y=None):
        # NaN / infinity are detected by the library on the device (a fit, an
        # assignment or a transform raises), so X is not scanned on the host
        X = check_array(X, dtype=np.float32, order="C", ensure_min_samples=2, ensure_all_finite=False)
        if y is not None:
            y = check_array(y, dtype=np.float32, order="C", ensure_2d=False)
        return X, y

    def _should_use_gpu(self, X):
        """Routing decision as in the reference (device, sparse input, dtype,
        thresholds); subclasses without a CPU path raise instead of routing away."""
        config = get_config()
        name = type(self).__name__
        if _get_device() == "cpu":
            if config.verbose:
                print(f"[skmetal] {name}: device=cpu (forced by set_device)")
            return False
        if hasattr(X, "nnz"):
            if config.verbose:
                print(f"[skmetal] {name}: device=cpu (sparse matrix)")
            return False
        if config.verbose:
            print(f"[skmetal] {name}: device=gpu ({X.shape[0]}x{X.shape[1]})")
        return True

    def score(self, X, y=None, **kwargs):
        return self._estimator.score(X, y, **kwargs)

    def __sklearn_is_fitted__(self):
        return self._fitted

    def __getattr__(self, name):
        if name in ("_estimator", "_fitted"):
            raise AttributeError(name)
        est = self.__dict__.get("_estimator")
        if est is not None and hasattr(est, name):
            return getattr(est, name)
        raise AttributeError(f"'{type(self).__name__}' has no attribute '{name}'")
