"""ctypes bridge to ``libskmetal_cuda.so`` (the CUDA replacement of the
reference's ``libSkMetalBridge.dylib``).

Mirrors ``skmetal/_bridge.py``: the library is loaded once per process (on
first use rather than at import), ``_bridge_call`` converts numpy arrays / ints / floats / bools the same way
(``skmetal/_bridge.py:78-103``) and raises ``RuntimeError`` on a nonzero
status. Unlike the reference, symbols are bound tolerantly (a missing symbol
disables only its wrapper) and the error text comes from the library.

There is no CPU fallback anywhere in this module: when the library or a GPU
is missing, every compute wrapper raises.
"""

from __future__ import annotations

import ctypes
import os
import warnings
from pathlib import Path

import numpy as np

__all__ = [
    "CUDA_AVAILABLE", "GPU_AVAILABLE", "METAL_AVAILABLE", "LIB_PATH",
    "ensure_warmed_up", "kmeans_assign", "kmeans_batch_fused", "compute_mindists", "kmeans_inertia",
    "kmeans_inertia_weighted",
    "row_norm_sq", "pairwise_distance", "kmeans_plusplus", "kmeans_fit", "kmeans_lloyd_iter", "kmeans_transform", "Dataset", "last_fit_stats",
    "launch_count", "device_info", "device_count", "is_loaded", "set_device", "comm_unique_id", "comm_init",
    "comm_destroy", "kmeans_fit_shard", "debug_inject_failure", "debug_loop_stamps", "FIT_CENTER", "FIT_SIMT", "FIT_PROFILE",
    "FIT_DISTRIBUTED", "FIT_TOL_ABS", "EXPORTED_SYMBOLS",
]

FIT_CENTER = 0x1
FIT_SIMT = 0x2
FIT_PROFILE = 0x4
FIT_DISTRIBUTED = 0x8
FIT_TOL_ABS = 0x10
FIT_BULK_SUMS = 0x20

_c_void_p, _c_size_t, _c_int, _c_float, _c_double = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                                      ctypes.c_float, ctypes.c_double)
_c_i32, _c_u32, _c_u64 = ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64

# (name, restype, argtypes) -- every symbol include/skmetal_cuda.h declares
_SIGNATURES = [
    ("skmetal_init", _c_int, []),
    ("skmetal_warmup", _c_int, []),
    ("skmetal_device_info", _c_int, [ctypes.c_char_p, _c_int, ctypes.POINTER(_c_size_t),
                                     ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(_c_u64)]),
    ("skmetal_device_count", _c_int, [ctypes.POINTER(_c_int)]),
    ("skmetal_set_device", _c_int, [_c_int]),
    ("skmetal_last_error", _c_int, [ctypes.c_char_p, _c_size_t]),
    ("skmetal_launch_count", ctypes.c_ulonglong, []),
    ("skmetal_debug_inject_failure", _c_int, [_c_int, _c_int]),
    ("skmetal_debug_tc_probe", _c_int, [ctypes.POINTER(_c_int), _c_void_p]),
    ("skmetal_debug_tc_probe_wide", _c_int, [ctypes.POINTER(_c_int), _c_void_p]),
    ("skmetal_debug_loop_stamps", _c_int, [_c_void_p, _c_int]),
    ("skmetal_kmeans_assign", _c_int, [_c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_size_t, _c_size_t]),
    ("skmetal_kmeans_batch_fused", _c_int, [_c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_size_t, _c_size_t,
                                            _c_size_t, _c_size_t, _c_float, ctypes.POINTER(_c_i32)]),
    ("skmetal_compute_mindists", _c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_size_t,
                                          _c_size_t]),
    ("skmetal_kmeans_inertia", _c_float, [_c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_size_t, _c_size_t]),
    ("skmetal_row_norm_sq", _c_int, [_c_void_p, _c_void_p, _c_size_t, _c_size_t]),
    ("skmetal_pairwise_distance", _c_int, [_c_void_p, _c_void_p, _c_size_t, _c_size_t]),
    ("skmetal_kmeans_fit", _c_int, [_c_void_p, _c_size_t, _c_size_t, _c_size_t, _c_void_p, _c_i32, _c_double,
                                    _c_u32, _c_void_p, _c_void_p, ctypes.POINTER(_c_double),
                                    ctypes.POINTER(_c_i32)]),
    ("skmetal_kmeans_lloyd_iter", _c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                           _c_size_t, _c_size_t, _c_size_t]),
    ("skmetal_kmeans_transform", _c_int, [_c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_size_t, _c_size_t]),
    ("skmetal_kmeans_fit_weighted", _c_int, [_c_void_p, _c_size_t, _c_size_t, _c_size_t, _c_void_p, _c_i32,
                                             _c_double, _c_u32, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                             _c_void_p]),
    ("skmetal_kmeans_inertia_weighted", _c_float, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size_t,
                                                   _c_size_t, _c_size_t]),
    ("skmetal_dataset_fit_weighted", _c_int, [_c_void_p, _c_void_p, _c_size_t, _c_i32, _c_double, _c_u32,
                                              _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    ("skmetal_kmeans_plusplus", _c_int, [_c_void_p, _c_size_t, _c_size_t, _c_size_t, _c_void_p, ctypes.c_int64,
                                         _c_void_p, _c_size_t, _c_int, _c_void_p, _c_void_p]),
    ("skmetal_dataset_kmeans_plusplus", _c_int, [_c_void_p, _c_size_t, _c_void_p, ctypes.c_int64, _c_void_p,
                                                 _c_size_t, _c_int, _c_void_p, _c_void_p]),
    ("skmetal_dataset_create", _c_int, [_c_void_p, _c_size_t, _c_size_t, ctypes.POINTER(_c_void_p)]),
    ("skmetal_dataset_free", _c_int, [_c_void_p]),
    ("skmetal_kmeans_fit_dataset", _c_int, [_c_void_p, _c_void_p, _c_size_t, _c_i32, _c_double, _c_u32,
                                            _c_void_p, _c_void_p, ctypes.POINTER(_c_double),
                                            ctypes.POINTER(_c_i32)]),
    ("skmetal_kmeans_predict_dataset", _c_int, [_c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    ("skmetal_last_fit_stats", _c_int, [ctypes.POINTER(_c_double)] * 4 + [ctypes.POINTER(_c_i32),
                                        ctypes.POINTER(_c_double), ctypes.POINTER(_c_u64),
                                        ctypes.POINTER(_c_i32)]),
    ("skmetal_last_fit_distinct", _c_int, []),
    ("skmetal_comm_unique_id", _c_int, [_c_void_p]),
    ("skmetal_comm_init", _c_int, [_c_void_p, _c_int, _c_int]),
    ("skmetal_comm_destroy", _c_int, []),
    ("skmetal_kmeans_fit_shard", _c_int, [_c_void_p, _c_size_t, _c_size_t, _c_size_t, _c_void_p, _c_i32,
                                          _c_double, _c_u32, _c_u64, _c_u64, _c_void_p, _c_void_p,
                                          ctypes.POINTER(_c_double), ctypes.POINTER(_c_i32)]),
    ("skmetal_dataset_fit_shard", _c_int, [_c_void_p, _c_void_p, _c_size_t, _c_i32, _c_double, _c_u32, _c_u64,
                                           _c_u64, _c_void_p, _c_void_p, ctypes.POINTER(_c_double),
                                           ctypes.POINTER(_c_i32)]),
    ("skmetal_kmeans_update_centers_noalloc", _c_int, [_c_void_p, _c_void_p, _c_size_t, _c_size_t, _c_size_t,
                                                       _c_void_p, _c_void_p, _c_void_p]),
]
EXPORTED_SYMBOLS = [s[0] for s in _SIGNATURES]


def _find_library() -> Path:
    env = os.environ.get("SKMETAL_CUDA_LIB")
    cands = [Path(env)] if env else []
    cands.append(Path(__file__).resolve().parent / "libskmetal_cuda.so")
    for p in cands:
        if p.exists():
            return p
    raise RuntimeError(
        "libskmetal_cuda.so not found. Build it first: python -m skmetal_b200._build "
        "(or __graft_entry__.build())")


# The library is loaded on first use (any wrapper call, or reading
# CUDA_AVAILABLE / GPU_AVAILABLE / METAL_AVAILABLE / LIB_PATH), not at import:
# importing the package, e.g. only for its workload generators, maps no
# native code and touches no GPU.
_lib = None
_load_error = None
_loaded = False
_funcs: dict = {}
_state: dict = {}


def _load() -> None:
    """Load ``libskmetal_cuda.so`` and bind its symbols (once per process)."""
    global _lib, _load_error, _loaded
    if _loaded:
        return
    _loaded = True
    path = None
    try:
        path = _find_library()
        _lib = ctypes.CDLL(str(path))
    except Exception as e:  # noqa: BLE001
        _load_error = str(e)
        _lib = None
    if _lib is not None:
        for name, res, args in _SIGNATURES:
            try:
                f = getattr(_lib, name)
            except AttributeError:
                continue
            f.restype = res
            f.argtypes = args
            _funcs[name] = f
    cuda = _lib is not None
    gpu = cuda and _device_count_loaded() > 0
    _state.update(LIB_PATH=path, CUDA_AVAILABLE=cuda, GPU_AVAILABLE=gpu,
                  # the reference's public flag name, meaning "GPU path available" here
                  METAL_AVAILABLE=gpu)
    if not cuda:
        warnings.warn(f"skmetal_b200: CUDA library not loaded ({_load_error}); GPU estimators will raise.",
                      stacklevel=3)


def _device_count_loaded() -> int:
    n = _c_int(0)
    if _funcs["skmetal_device_count"](ctypes.byref(n)) != 0:
        return 0
    return int(n.value)


def __getattr__(name: str):
    if name in ("LIB_PATH", "CUDA_AVAILABLE", "GPU_AVAILABLE", "METAL_AVAILABLE"):
        _load()
        return _state[name]
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def is_loaded() -> bool:
    """True once this process has mapped the native library."""
    return _lib is not None


def device_count() -> int:
    _load()
    if _lib is None:
        return 0
    return _device_count_loaded()


def _require():
    _load()
    if not _state["CUDA_AVAILABLE"]:
        raise RuntimeError(f"skmetal_b200: CUDA library not available ({_load_error})")
    if not _state["GPU_AVAILABLE"]:
        raise RuntimeError("skmetal_b200: no CUDA device visible; the KMeans path has no CPU fallback")


def _fn(name: str):
    _require()
    f = _funcs.get(name)
    if f is None:
        raise RuntimeError(f"skmetal_b200: symbol {name} missing from {_state['LIB_PATH']}")
    return f


def _last_error() -> str:
    _load()
    if "skmetal_last_error" not in _funcs:
        return str(_load_error)
    buf = ctypes.create_string_buffer(1024)
    _funcs["skmetal_last_error"](buf, 1024)
    return buf.value.decode("utf-8", "replace")


_WARMUP_DONE = False


def ensure_warmed_up():
    global _WARMUP_DONE
    if not _WARMUP_DONE:
        rc = _fn("skmetal_init")()
        if rc != 0:
            raise RuntimeError(f"skmetal_init failed with code {rc}: {_last_error()}")
        _WARMUP_DONE = True


def set_device(index: int) -> None:
    rc = _fn("skmetal_set_device")(int(index))
    if rc != 0:
        raise RuntimeError(f"skmetal_set_device({index}) failed with code {rc}: {_last_error()}")


def _bridge_call(name: str, *args, context: str = ""):
    """Call ``name`` converting arguments like the reference's ``_bridge_call``."""
    f = _fn(name)
    ensure_warmed_up()
    c_args = []
    for a in args:
        if isinstance(a, np.ndarray):
            c_args.append(a.ctypes.data)
        elif isinstance(a, bool):
            c_args.append(_c_int(int(a)))
        elif isinstance(a, int):
            c_args.append(_c_size_t(a))
        elif isinstance(a, (float, np.floating)):
            c_args.append(_c_float(a))
        else:
            c_args.append(a)
    err = f(*c_args)
    if err != 0:
        msg = f"{name} failed with code {err}: {_last_error()}"
        if context:
            msg += f" ({context})"
        raise RuntimeError(msg)


def _f32c(a, name="array") -> np.ndarray:
    a = np.asarray(a)
    if a.dtype != np.float32 or not a.flags["C_CONTIGUOUS"]:
        raise TypeError(f"{name} must be float32 and C-contiguous")
    return a


def _lab32(a) -> np.ndarray:
    if not isinstance(a, np.ndarray) or a.dtype.itemsize != 4 or a.dtype.kind not in "iu" \
            or not a.flags["C_CONTIGUOUS"]:
        raise TypeError("labels must be a C-contiguous 4-byte integer array")
    return a


# ----------------------------------------------------------------------------
# reference entry points (same Python signatures as skmetal/_bridge.py)
# ----------------------------------------------------------------------------

def kmeans_assign(X, centroids, assignments, n: int, d: int, k: int) -> None:
    """KMeans assignment step (``skmetal/_bridge.py:576-578``)."""
    _f32c(X, "X"), _f32c(centroids, "centroids"), _lab32(assignments)
    _bridge_call("skmetal_kmeans_assign", X, centroids, assignments, int(n), int(d), int(k))


def kmeans_batch_fused(X, centroids, assignments, n: int, d: int, k: int, num_groups: int, max_iter: int,
                       tol: float) -> int:
    """Lloyd iterations on the GPU; ``centroids`` is updated in place (``skmetal/_bridge.py:591-617``)."""
    _f32c(X, "X"), _f32c(centroids, "centroids"), _lab32(assignments)
    n_iter = _c_i32(0)
    _bridge_call("skmetal_kmeans_batch_fused", X, centroids, assignments, int(n), int(d), int(k), int(num_groups),
                 int(max_iter), _c_float(tol), ctypes.byref(n_iter))
    return int(n_iter.value)


def compute_mindists(X, centroids, assignments, dists, n: int, d: int, k: int) -> None:
    """Per-row squared distance to the assigned centre (``skmetal/_bridge.py:620-624``)."""
    _f32c(X, "X"), _f32c(centroids, "centroids"), _lab32(assignments), _f32c(dists, "dists")
    _bridge_call("skmetal_compute_mindists", X, centroids, assignments, dists, int(n), int(d), int(k))


def kmeans_inertia(X, centroids, assignments, n: int, d: int, k: int) -> float:
    """Sum of squared distances to the assigned centres (``skmetal/_bridge.py:627-639``)."""
    _f32c(X, "X"), _f32c(centroids, "centroids"), _lab32(assignments)
    f = _fn("skmetal_kmeans_inertia")
    ensure_warmed_up()
    v = f(X.ctypes.data, centroids.ctypes.data, assignments.ctypes.data, int(n), int(d), int(k))
    if v < 0:
        raise RuntimeError(f"skmetal_kmeans_inertia failed: {_last_error()}")
    return float(v)


def kmeans_inertia_weighted(X, centroids, assignments, sample_weight, n: int, d: int, k: int) -> float:
    """Weighted sum of squared distances to the assigned centres."""
    _f32c(X, "X"), _f32c(centroids, "centroids"), _lab32(assignments), _f32c(sample_weight, "sample_weight")
    f = _fn("skmetal_kmeans_inertia_weighted")
    ensure_warmed_up()
    v = f(X.ctypes.data, centroids.ctypes.data, assignments.ctypes.data, sample_weight.ctypes.data, int(n), int(d),
          int(k))
    if v < 0:
        raise RuntimeError(f"skmetal_kmeans_inertia_weighted failed: {_last_error()}")
    return float(v)


def row_norm_sq(X) -> np.ndarray:
    X = _f32c(X, "X")
    out = np.empty(X.shape[0], dtype=np.float32)
    _bridge_call("skmetal_row_norm_sq", X, out, int(X.shape[0]), int(X.shape[1]))
    return out


def _plusplus_draws(n: int, k: int, random_state, sample_weight, n_local_trials):
    """What scikit-learn's _kmeans_plusplus draws from ``random_state``, in its
    order: the first centre over w / sum(w), then n_local_trials uniforms per
    further centre (one block of (k - 1) x T, the same stream)."""
    w = np.ones(n, dtype=np.float32) if sample_weight is None else np.ascontiguousarray(sample_weight, np.float32)
    if n_local_trials is None:
        n_local_trials = 2 + int(np.log(k))
    first = int(random_state.choice(n, p=w / w.sum()))
    u = np.ascontiguousarray(random_state.uniform(size=(max(k - 1, 0), n_local_trials)), dtype=np.float64)
    return (None if sample_weight is None else w), first, u, int(n_local_trials)


def kmeans_plusplus(X, k: int, random_state, sample_weight=None, n_local_trials=None, center: bool = True):
    """k-means++ seeding on the GPU (scikit-learn's greedy variant and random
    stream). ``X`` is a host array or a :class:`Dataset`. Returns the centres
    (raw rows of X, k x d float32) and their row indices (int64)."""
    k = int(k)
    ds = X if isinstance(X, Dataset) else None
    if ds is None:
        X = _f32c(X, "X")
        n, d = X.shape
    else:
        n, d = ds.n, ds.d
    if not 1 <= k <= n:
        raise ValueError(f"n_samples={n} should be >= n_clusters={k}.")
    w, first, u, T = _plusplus_draws(n, k, random_state, sample_weight, n_local_trials)
    centers = np.empty((k, d), dtype=np.float32)
    idx = np.empty(k, dtype=np.int64)
    if ds is None:
        _bridge_call("skmetal_kmeans_plusplus", X, n, d, k, w, ctypes.c_int64(first), u, T, _c_int(int(bool(center))),
                     centers, idx)
    else:
        _bridge_call("skmetal_dataset_kmeans_plusplus", ds._h, k, w, ctypes.c_int64(first), u, T,
                     _c_int(int(bool(center))), centers, idx)
    return centers, idx


def pairwise_distance(X: np.ndarray) -> np.ndarray:
    """Squared Euclidean pairwise distance matrix (n x n float32).

    Same contract as the reference's ``skmetal/_bridge.py:566-573``: X must be
    float32 and C-contiguous; D[i, j] = max(|x_i|^2 + |x_j|^2 - 2 x_i.x_j, 0).
    """
    if not isinstance(X, np.ndarray) or X.dtype != np.float32 or not X.flags["C_CONTIGUOUS"] or X.ndim != 2:
        raise TypeError("X must be float32 and C-contiguous")
    n, d = X.shape
    D = np.empty((n, n), dtype=np.float32, order="C")
    _bridge_call("skmetal_pairwise_distance", X, D, n, d)
    return D


# ----------------------------------------------------------------------------
# extended entry points
# ----------------------------------------------------------------------------

def kmeans_fit(X, init, max_iter: int, tol: float, *, center: bool = True, tol_abs: bool = False,
               simt: bool = False, profile: bool = False, want_labels: bool = True, bulk_sums: bool = False,
               sample_weight=None):
    """One Lloyd run from ``init`` (KMeans.fit semantics with n_init=1).

    Returns ``(centers, labels, inertia, n_iter)``; ``labels`` is None when
    ``want_labels`` is False.
    """
    X = _f32c(X, "X")
    init = _f32c(init, "init")
    n, d = X.shape
    k = init.shape[0]
    if init.shape[1] != d:
        raise ValueError(f"init has {init.shape[1]} features, X has {d}")
    centers = np.empty((k, d), dtype=np.float32)
    labels = np.empty(n, dtype=np.int32) if want_labels else None
    inertia = _c_double(0.0)
    n_iter = _c_i32(0)
    flags = (FIT_CENTER if center else 0) | (FIT_TOL_ABS if tol_abs else 0) | (FIT_SIMT if simt else 0) \
        | (FIT_PROFILE if profile else 0) | (FIT_BULK_SUMS if bulk_sums else 0)
    if sample_weight is None:
        _bridge_call("skmetal_kmeans_fit", X, int(n), int(d), int(k), init, _c_i32(int(max_iter)), _c_double(tol),
                     _c_u32(flags), centers, labels if labels is not None else None, ctypes.byref(inertia),
                     ctypes.byref(n_iter))
    else:
        w = _f32c(sample_weight, "sample_weight")
        if w.shape != (n,):
            raise ValueError(f"sample_weight has shape {w.shape}, expected ({n},)")
        _bridge_call("skmetal_kmeans_fit_weighted", X, int(n), int(d), int(k), init, _c_i32(int(max_iter)),
                     _c_double(tol), _c_u32(flags), w, centers, labels if labels is not None else None,
                     ctypes.byref(inertia), ctypes.byref(n_iter))
    return centers, labels, float(inertia.value), int(n_iter.value)


def kmeans_lloyd_iter(X, centers_old):
    """One E+M step (``lloyd_iter_chunked_dense``) on X as given.

    Returns ``(labels, centers_new, weight, center_shift)``.
    """
    X = _f32c(X, "X")
    centers_old = _f32c(centers_old, "centers_old")
    n, d = X.shape
    k = centers_old.shape[0]
    labels = np.empty(n, dtype=np.int32)
    centers_new = np.empty((k, d), dtype=np.float32)
    weight = np.empty(k, dtype=np.float32)
    shift = np.empty(k, dtype=np.float32)
    _bridge_call("skmetal_kmeans_lloyd_iter", X, centers_old, centers_new, labels, weight, shift, int(n), int(d),
                 int(k))
    return labels, centers_new, weight, shift


def kmeans_transform(X, centroids) -> np.ndarray:
    X = _f32c(X, "X")
    centroids = _f32c(centroids, "centroids")
    out = np.empty((X.shape[0], centroids.shape[0]), dtype=np.float32)
    _bridge_call("skmetal_kmeans_transform", X, centroids, out, int(X.shape[0]), int(X.shape[1]),
                 int(centroids.shape[0]))
    return out


class Dataset:
    """X resident in device memory (the current CUDA device of this thread)."""

    def __init__(self, X):
        X = _f32c(X, "X")
        self.n, self.d = X.shape
        h = _c_void_p()
        _bridge_call("skmetal_dataset_create", X, int(self.n), int(self.d), ctypes.byref(h))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            _funcs["skmetal_dataset_free"](self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def fit(self, init, max_iter: int, tol: float, *, center: bool = True, tol_abs: bool = False,
            simt: bool = False, profile: bool = False, labels_out=None, shard: tuple | None = None,
            sample_weight=None):
        """Fit on the resident rows; ``shard=(row_base, n_total)`` for a distributed fit."""
        init = _f32c(init, "init")
        k = init.shape[0]
        centers = np.empty((k, self.d), dtype=np.float32)
        inertia = _c_double(0.0)
        n_iter = _c_i32(0)
        flags = (FIT_CENTER if center else 0) | (FIT_TOL_ABS if tol_abs else 0) | (FIT_SIMT if simt else 0) \
            | (FIT_PROFILE if profile else 0)
        if labels_out is not None:
            _lab32(labels_out)
        if sample_weight is not None:
            if shard is not None:
                raise ValueError("sample weights are supported on one GPU only")
            w = _f32c(sample_weight, "sample_weight")
            if w.shape != (self.n,):
                raise ValueError(f"sample_weight has shape {w.shape}, expected ({self.n},)")
            _bridge_call("skmetal_dataset_fit_weighted", self._h, init, int(k), _c_i32(int(max_iter)),
                         _c_double(tol), _c_u32(flags), w, centers, labels_out, ctypes.byref(inertia),
                         ctypes.byref(n_iter))
        elif shard is None:
            _bridge_call("skmetal_kmeans_fit_dataset", self._h, init, int(k), _c_i32(int(max_iter)),
                         _c_double(tol), _c_u32(flags), centers, labels_out, ctypes.byref(inertia),
                         ctypes.byref(n_iter))
        else:
            _bridge_call("skmetal_dataset_fit_shard", self._h, init, int(k), _c_i32(int(max_iter)),
                         _c_double(tol), _c_u32(flags | FIT_DISTRIBUTED), _c_u64(int(shard[0])),
                         _c_u64(int(shard[1])), centers, labels_out, ctypes.byref(inertia), ctypes.byref(n_iter))
        return centers, float(inertia.value), int(n_iter.value)

    def predict(self, centroids, labels_out=None):
        centroids = _f32c(centroids, "centroids")
        if labels_out is not None:
            _lab32(labels_out)
        _bridge_call("skmetal_kmeans_predict_dataset", self._h, centroids, int(centroids.shape[0]), labels_out)
        return labels_out


def last_fit_stats() -> dict:
    v = [_c_double() for _ in range(4)]
    el, ems, la, it = _c_i32(), _c_double(), _c_u64(), _c_i32()
    _fn("skmetal_last_fit_stats")(*[ctypes.byref(x) for x in v], ctypes.byref(el), ctypes.byref(ems),
                                  ctypes.byref(la), ctypes.byref(it))
    return {"ms_total": v[0].value, "ms_prep": v[1].value, "ms_loop": v[2].value, "ms_final": v[3].value,
            "estep_launches": el.value, "estep_ms_sum": ems.value, "launches": int(la.value),
            "iterations": it.value}


def last_fit_distinct() -> int:
    """Distinct labels in the final assignment of this thread's last one-GPU
    fit, counted on the device; -1 when the fit did not count them."""
    return int(_fn("skmetal_last_fit_distinct")())


def launch_count() -> int:
    return int(_fn("skmetal_launch_count")())


def device_info() -> dict:
    ensure_warmed_up()
    name = ctypes.create_string_buffer(256)
    mt, un, ws = _c_size_t(), ctypes.c_uint8(), _c_u64()
    rc = _fn("skmetal_device_info")(name, 256, ctypes.byref(mt), ctypes.byref(un), ctypes.byref(ws))
    if rc != 0:
        raise RuntimeError(f"skmetal: device_info() failed: {_last_error()}")
    return {"name": name.value.decode("utf-8", "replace"), "max_threads_per_threadgroup": mt.value,
            "has_unified_memory": bool(un.value), "recommended_working_set_size_bytes": ws.value}


def debug_tc_probe(raw: bool = False):
    """Tensor-core self-check: (mode, raw) with mode 0 exact, -1 unusable (SIMT E-step).

    ``raw`` (4096 uint32 bit patterns of float32): [0, 2048) the stacked-layout
    products, [2048, 4096) the two-segment-layout products, each 128 x 16.
    """
    mode = _c_int(-3)
    out = np.zeros(4096, dtype=np.uint32) if raw else None
    rc = _fn("skmetal_debug_tc_probe")(ctypes.byref(mode), out.ctypes.data if raw else None)
    if rc != 0:
        raise RuntimeError(f"skmetal_debug_tc_probe failed with code {rc}: {_last_error()}")
    return int(mode.value), out


def debug_tc_probe_wide():
    """Self-check of the k > 256 E-step's blocked centre image and MMA
    sequence: (mode, raw) with raw the 128 x 32 products (uint32 bit patterns
    of float32); mode 0 exact, -1 unusable (SIMT E-step for k > 256)."""
    mode = _c_int(-3)
    out = np.zeros(4096, dtype=np.uint32)
    rc = _fn("skmetal_debug_tc_probe_wide")(ctypes.byref(mode), out.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"skmetal_debug_tc_probe_wide failed with code {rc}: {_last_error()}")
    return int(mode.value), out


def debug_loop_stamps() -> np.ndarray:
    """Device timestamps (ns) of the last profiled persistent-loop fit on this
    thread: per iteration [start, E-step done, sums and empties done, centres
    done], then the end stamp; empty when that fit used the multi-launch loop."""
    n = int(_fn("skmetal_debug_loop_stamps")(None, 0))
    out = np.zeros(max(n, 0), dtype=np.uint64)
    if n > 0:
        _fn("skmetal_debug_loop_stamps")(out.ctypes.data, n)
    return out


def debug_inject_failure(code: int, after_calls: int = 0) -> None:
    """Make the ``after_calls``-th next guarded library call fail with ``code`` (tests)."""
    _fn("skmetal_debug_inject_failure")(int(code), int(after_calls))


# ----------------------------------------------------------------------------
# multi-GPU
# ----------------------------------------------------------------------------

def _point_at_torch_nccl():
    if os.environ.get("SKMETAL_NCCL_LIB"):
        return
    try:
        import nvidia.nccl  # noqa: F401  (the NCCL PyTorch ships)
        base = Path(list(nvidia.nccl.__path__)[0]) / "lib" / "libnccl.so.2"
        if base.exists():
            os.environ["SKMETAL_NCCL_LIB"] = str(base)
    except Exception:  # noqa: BLE001
        pass


def comm_unique_id() -> bytes:
    _point_at_torch_nccl()
    buf = (ctypes.c_uint8 * 128)()
    rc = _fn("skmetal_comm_unique_id")(ctypes.cast(buf, _c_void_p))
    if rc != 0:
        raise RuntimeError(f"skmetal_comm_unique_id failed with code {rc}: {_last_error()}")
    return bytes(buf)


def comm_init(uid: bytes, nranks: int, rank: int) -> None:
    _point_at_torch_nccl()
    if len(uid) != 128:
        raise ValueError("unique id must be 128 bytes")
    buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
    rc = _fn("skmetal_comm_init")(ctypes.cast(buf, _c_void_p), int(nranks), int(rank))
    if rc != 0:
        raise RuntimeError(f"skmetal_comm_init failed with code {rc}: {_last_error()}")


def comm_destroy() -> None:
    if is_loaded() and "skmetal_comm_destroy" in _funcs:
        _funcs["skmetal_comm_destroy"]()


def kmeans_fit_shard(X, init, max_iter: int, tol: float, row_base: int, n_total: int, *, center: bool = True,
                     tol_abs: bool = False, simt: bool = False, want_labels: bool = True):
    X = _f32c(X, "X")
    init = _f32c(init, "init")
    n, d = X.shape
    k = init.shape[0]
    centers = np.empty((k, d), dtype=np.float32)
    labels = np.empty(n, dtype=np.int32) if want_labels else None
    inertia = _c_double(0.0)
    n_iter = _c_i32(0)
    flags = FIT_DISTRIBUTED | (FIT_CENTER if center else 0) | (FIT_TOL_ABS if tol_abs else 0) \
        | (FIT_SIMT if simt else 0)
    _bridge_call("skmetal_kmeans_fit_shard", X, int(n), int(d), int(k), init, _c_i32(int(max_iter)),
                 _c_double(tol), _c_u32(flags), _c_u64(int(row_base)), _c_u64(int(n_total)), centers, labels,
                 ctypes.byref(inertia), ctypes.byref(n_iter))
    return centers, labels, float(inertia.value), int(n_iter.value)
