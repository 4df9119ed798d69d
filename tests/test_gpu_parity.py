"""GPU parity tests: the CUDA path through the C ABI against the oracle.

Protocol (scikit-learn's Lloyd is chaotic in float32, so end-to-end label
agreement between two correct implementations with different summation
orders drifts; parity is therefore judged in lockstep):

* lockstep: each GPU Lloyd step starts from the oracle's centres of that
  iteration and is compared with the oracle's step (labels, counts, centres,
  shift);
* end to end: full fits compared with scikit-learn on well-separated data
  where both converge to the same clustering.
"""

import numpy as np
import pytest

from oracle import lloyd as ora
from skmetal_b200 import _bridge
from skmetal_b200._synthetic import gaussian_mixture, make_workload, scaled

from parity import CENTER_RTOL, INERTIA_RTOL, check_counts, check_labels, lockstep, probe_c as _probe_c, probe_x as _probe_x

pytestmark = pytest.mark.gpu


def _fp64_centres(X, labels, k, init):
    C = np.zeros((k, X.shape[1]))
    cnt = np.bincount(labels, minlength=k)
    np.add.at(C, labels, X.astype(np.float64))
    nz = cnt > 0
    C[nz] /= cnt[nz, None]
    return C, cnt


# ---------------------------------------------------------------------------
# reference golden vector (skmetal tests/test_kernels.py:94-98)
# ---------------------------------------------------------------------------

def test_kmeans_assign_golden():
    X = np.array([[0.0, 0.0], [1.0, 1.0], [10.0, 10.0], [9.0, 9.0]], dtype=np.float32)
    centroids = np.array([[0.0, 0.0], [10.0, 10.0]], dtype=np.float32)
    assignments = np.empty(4, dtype=np.int32)
    _bridge.kmeans_assign(X, centroids, assignments, 4, 2, 2)
    np.testing.assert_array_equal(assignments, [0, 0, 1, 1])


def test_compute_mindists_and_inertia_golden():
    X = np.array([[0.0, 0.0], [1.0, 1.0], [10.0, 10.0], [9.0, 9.0]], dtype=np.float32)
    C = np.array([[0.0, 0.0], [10.0, 10.0]], dtype=np.float32)
    lab = np.array([0, 0, 1, 1], dtype=np.uint32)
    dists = np.empty(4, dtype=np.float32)
    _bridge.compute_mindists(X, C, lab, dists, 4, 2, 2)
    np.testing.assert_allclose(dists, [0.0, 2.0, 0.0, 2.0], rtol=1e-6)
    assert _bridge.kmeans_inertia(X, C, lab, 4, 2, 2) == pytest.approx(4.0, rel=1e-6)
    np.testing.assert_allclose(_bridge.row_norm_sq(X), [0, 2, 200, 162], rtol=1e-6)


def test_tensor_core_probe():
    """The fp16 split of X, the centre image and both MMA sequences give the
    exact x_hi.c_hi + x_lo.c_hi + x_hi.c_lo on exactly representable operands."""
    mode, raw = _bridge.debug_tc_probe(raw=True)
    assert mode == 0, mode
    j = np.arange(16)
    x = _probe_x(np.arange(128)[:, None], j[None, :])          # 128 x 16, exact in float32
    c = _probe_c(np.arange(16)[:, None], j[None, :])           # 16 x 16
    xh, ch = np.round(x), np.round(c)
    want = (xh @ ch.T + (x - xh) @ ch.T + xh @ (c - ch).T).astype(np.float32)
    got = raw.view(np.float32)
    np.testing.assert_array_equal(got[:2048].reshape(128, 16), want)
    np.testing.assert_array_equal(got[2048:].reshape(128, 16), want)


# ---------------------------------------------------------------------------
# assignment
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("n,d,k", [(5000, 32, 8), (3000, 8, 16), (2000, 100, 50), (1000, 7, 3), (777, 1, 5)])
def test_assign_matches_fp64_argmin(n, d, k):
    rng = np.random.default_rng(n + d + k)
    X = rng.standard_normal((n, d)).astype(np.float32) * 3
    C = rng.standard_normal((k, d)).astype(np.float32) * 3
    lab = np.empty(n, dtype=np.int32)
    _bridge.kmeans_assign(X, C, lab, n, d, k)
    want, _ = ora.assign(X, C, "fp64")
    check_labels(X, C, lab, want, "assign")


def test_transform_matches_fp64():
    rng = np.random.default_rng(7)
    X = rng.standard_normal((1500, 13)).astype(np.float32)
    C = rng.standard_normal((9, 13)).astype(np.float32)
    D = _bridge.kmeans_transform(X, C)
    ref = np.sqrt(((X[:, None, :].astype(np.float64) - C[None].astype(np.float64)) ** 2).sum(-1))
    np.testing.assert_allclose(D, ref, rtol=1e-5, atol=1e-6)


# ---------------------------------------------------------------------------
# golden fixtures produced by the reference's own API (tests/golden)
# ---------------------------------------------------------------------------

def _golden_case(name):
    import importlib.util
    import json
    from pathlib import Path

    g = Path(__file__).resolve().parent / "golden"
    spec = importlib.util.spec_from_file_location("make_golden", g / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    z = np.load(g / "golden_kmeans.npz")
    c = json.loads(str(z["meta"]))["cases"][name]
    X, init = mg.case_inputs(c["gen"])
    assert mg.digest(X, init) == c["sha256"]
    return X, init, c, z


@pytest.mark.parametrize("name", ["c1_small", "c2_small", "c3_small", "c3_k1024", "c4_small", "k300_odd",
                                  "tol_rel", "relocation", "odd_shape"])
def test_fit_matches_reference_golden(name):
    """Full fits against the reference's outputs on the same inputs (the
    BASELINE recipes with near-ties by the relative-gap rule only)."""
    X, init, c, z = _golden_case(name)
    centers, labels, inertia, n_iter = _bridge.kmeans_fit(X, init, c["max_iter"], c["tol"])
    mean, Xc, _ = ora.center_data(X)
    check_labels(Xc, centers - mean, labels, z[f"{name}/full/labels"], f"{name} labels",
                 strict=name.startswith(("c1", "c2", "c3", "c4")))
    scale = float(np.abs(X).max())
    np.testing.assert_allclose(centers, z[f"{name}/full/centers"], rtol=CENTER_RTOL, atol=1e-5 * scale)
    assert inertia == pytest.approx(float(z[f"{name}/full/inertia"]), rel=INERTIA_RTOL)
    assert n_iter == int(z[f"{name}/full/n_iter"])


# ---------------------------------------------------------------------------
# lockstep Lloyd steps
# ---------------------------------------------------------------------------

def _lockstep(X, init, iters, strict=False):
    return lockstep(X, init, iters, strict=strict)


@pytest.mark.parametrize("name,n", [("c1", 20000), ("c2", 25000)])
def test_lloyd_step_lockstep(name, n):
    w = scaled(name, n)
    X, init = make_workload(w)
    reps = _lockstep(X, init, 8, strict=True)  # BASELINE recipes: relative-gap near-ties only
    assert sum(r["mismatches"] for r in reps) <= 8 * max(1, n // 10000)


def test_lloyd_step_relocation_lockstep():
    # k=20 on 5 blobs with duplicate-heavy init: empty clusters every step
    X, _ = gaussian_mixture(4000, 10, 5, seed=11)
    init = np.ascontiguousarray(np.repeat(X[:4], 5, axis=0))
    init[::5] += 0  # duplicates on purpose
    _lockstep(X, init, 5)


def test_fit_single_empty_cluster_matches_oracle():
    """A duplicated initial centre leaves exactly one cluster empty in the
    first iteration (ties go to the lower index), so the relocation picks one
    farthest row, through the selection's one-row path: the fit must match the
    oracle's (_k_means_common.pyx:160-196); the oracle relocates one row in
    each of the first two iterations."""
    X, init = _golden_gen("reloc1")  # centre 6 duplicates centre 0
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, 30, 0.0)
    res = ora.kmeans_lloyd(X, init, 30, 0.0, relocation_order="sorted")
    assert n_iter == res.n_iter
    assert np.mean(lab == res.labels) >= 0.9999
    np.testing.assert_allclose(c, res.centers, rtol=CENTER_RTOL, atol=1e-5)
    assert inertia == pytest.approx(res.inertia, rel=INERTIA_RTOL)


@pytest.mark.parametrize("n,d,k", [(300_000, 36, 24), (200_000, 100, 50), (150_000, 64, 256), (120_000, 40, 200),
                                   (100_000, 24, 137)])
def test_estep_many_tiles_per_cta(n, d, k):
    """Sizes at which every CTA of the persistent tensor-core E-step runs many
    tiles, so its shared-memory stages, accumulators and both MMA issuers wrap
    around many times: one Lloyd step against the oracle's E-step. With
    k = 200 and k = 137 the four epilogue groups that share each tile scan
    unequal column ranges (64, 64, 64, 16 and 48, 48, 48, none)."""
    X, init = gaussian_mixture(n, d, k, seed=n + d + k)
    lab, cnew, weight, shift = _bridge.kmeans_lloyd_iter(X, init)
    want, _ = ora.assign(X, init, "fp32")
    check_labels(X, init, lab, want, "many-tile E-step")
    np.testing.assert_array_equal(weight.astype(np.int64), np.bincount(lab, minlength=k))


@pytest.mark.parametrize("ratio,k", [(1e-3, 16), (1e-5, 16), (1e-3, 200)])
def test_wide_dynamic_range_columns(ratio, k):
    """One column spans the whole range of X (uniform noise, the same for
    every centre) while the clusters live in columns `ratio` times smaller.
    The tensor-core E-step scales each operand by one power of two, so the
    small columns sit far down fp16's range. One E-step from the true centres
    must give the float64 argmin of ||c||^2 - 2 x.c for every row whose two
    best float64 values are further apart than 2^-20 of the magnitudes that
    enter them (2 sum|x||c| + ||c||^2 of both centres); here every row is, by
    a factor of about 250 at ratio 1e-5."""
    rng = np.random.default_rng(int(round(1 / ratio)) + k)
    n, d = 60000, 24
    centres = rng.uniform(-10, 10, size=(k, d)) * ratio
    centres[:, 0] = 0.0
    lab = rng.integers(0, k, n)
    X = centres[lab] + ratio * rng.normal(size=(n, d))
    X[:, 0] = rng.uniform(-1, 1, size=n)
    X = X.astype(np.float32)
    mean, Xc, C = ora.center_data(X, centres.astype(np.float32))
    got, _, weight, _ = _bridge.kmeans_lloyd_iter(Xc, C)
    np.testing.assert_array_equal(weight.astype(np.int64), np.bincount(got, minlength=k))
    Xd, Cd = Xc.astype(np.float64), C.astype(np.float64)
    cn = (Cd ** 2).sum(axis=1)
    E = cn[None, :] - 2.0 * (Xd @ Cd.T)
    want = np.argmin(E, axis=1)
    mism = np.nonzero(got != want)[0]
    if mism.size:
        A = np.abs(Xd[mism]) @ np.abs(Cd).T
        a, b = got[mism], want[mism]
        gap = np.abs(E[mism, a] - E[mism, b])
        bound = 2.0 ** -20 * (2 * A[np.arange(mism.size), a] + 2 * A[np.arange(mism.size), b] + cn[a] + cn[b])
        assert np.all(gap <= bound), (f"{int((gap > bound).sum())} of {n} labels differ from the float64 argmin "
                                      f"beyond the split's precision (gap/bound {np.sort(gap / bound)[-5:]})")


# ---------------------------------------------------------------------------
# tensor-core vs SIMT E-step, full fits
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name,n", [("c1", 30000), ("c2", 30000)])
def test_tc_fit_matches_simt_fit(name, n):
    """Tensor-core and SIMT E-steps agree (one Lloyd iteration plus the final
    E-step, so that the comparison is not amplified by later iterations)."""
    w = scaled(name, n)
    X, init = make_workload(w)
    c_tc, l_tc, i_tc, n_tc = _bridge.kmeans_fit(X, init, 1, 0.0)
    c_si, l_si, i_si, n_si = _bridge.kmeans_fit(X, init, 1, 0.0, simt=True)
    mean, Xc, _ = ora.center_data(X)
    check_labels(Xc, c_si - mean, l_tc, l_si, "tc vs simt")
    np.testing.assert_allclose(c_tc, c_si, rtol=CENTER_RTOL, atol=1e-4)
    assert i_tc == pytest.approx(i_si, rel=1e-5)


@pytest.mark.parametrize("name,n,max_iter", [("c1", 20000, 50), ("c2", 20000, 30)])
def test_fit_end_to_end_vs_sklearn(name, n, max_iter):
    from sklearn.cluster import KMeans

    w = scaled(name, n)
    X, init = make_workload(w)
    km = KMeans(w.k, init=init, n_init=1, max_iter=max_iter, tol=0, algorithm="lloyd").fit(X)
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, max_iter, 0.0)
    res = ora.kmeans_lloyd(X, init, max_iter, 0.0)
    # End to end, float32 Lloyd is chaotic: a single near-tie decided
    # differently in an early iteration moves a few hundred rows later (the
    # oracle and scikit-learn themselves differ by machine and thread count).
    # Parity proper is the lockstep test; here the fits must land on the same
    # clustering up to that drift.
    floor = np.mean(res.labels == km.labels_)
    agree = np.mean(lab == km.labels_)
    assert agree >= min(floor, 0.99) - 0.005, (agree, floor)
    assert inertia == pytest.approx(km.inertia_, rel=1e-3)
    if agree == 1.0:
        np.testing.assert_allclose(c, km.cluster_centers_, rtol=CENTER_RTOL, atol=1e-4)


def test_tolerance_decision_lockstep():
    """The scaled-tolerance stop (_kmeans.py:285-294,731-738) decided in lockstep.

    End to end the iteration at which sum(shift^2) <= tol first holds depends
    on float32 summation order (a few tie rows change the tiny late shifts), so
    the decision is checked step by step from the oracle's centres.
    """
    from sklearn.cluster import KMeans

    X, init = gaussian_mixture(20000, 16, 6, seed=5)
    res = ora.kmeans_lloyd(X, init, 300, 1e-4, keep_centers=True)
    km = KMeans(6, init=init, n_init=1, max_iter=300, tol=1e-4, algorithm="lloyd").fit(X)
    # the oracle's loop is scikit-learn's, but when the relative tolerance stops
    # it depends on float32 summation order, which depends on the host's thread
    # count: the exact pinning is test_oracle.py's, on fixed fixtures
    assert abs(res.n_iter - km.n_iter_) <= 5
    tol_abs = ora.tolerance(X, 1e-4)
    mean, Xc, _ = ora.center_data(X)
    for i, h in enumerate(res.history):
        lab, cnew, weight, shift = _bridge.kmeans_lloyd_iter(Xc, h["centers_in"])
        if np.array_equal(lab, h["labels"]):
            stop_gpu = float((shift.astype(np.float64) ** 2).sum()) <= tol_abs
            stop_ref = h["shift_tot"] <= tol_abs
            if abs(h["shift_tot"] - tol_abs) > 1e-3 * tol_abs:
                assert stop_gpu == stop_ref, (i, h["shift_tot"], tol_abs)
    # end to end: same clustering, iteration count within the float32 noise
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, 300, 1e-4)
    assert abs(n_iter - km.n_iter_) <= 5
    assert np.mean(lab == km.labels_) >= 0.99
    assert inertia == pytest.approx(km.inertia_, rel=1e-3)


def test_batch_fused_reference_abi():
    X, init = gaussian_mixture(5000, 12, 4, seed=2)
    C = init.copy()
    lab = np.empty(X.shape[0], dtype=np.uint32)
    n_iter = _bridge.kmeans_batch_fused(X, C, lab, X.shape[0], 12, 4, (X.shape[0] + 255) // 256, 100, 0.0)
    res = ora.kmeans_lloyd(X, init, 100, 0.0)  # same loop, but centred
    assert 1 <= n_iter <= 100
    assert np.mean(lab.astype(np.int32) == res.labels) >= 0.999


# ---------------------------------------------------------------------------
# edge cases
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("n,d,k", [(5, 3, 2), (130, 1, 1), (257, 9, 7), (1000, 33, 32), (64, 4, 64),
                                   (300, 129, 5), (2000, 16, 257)])
def test_fit_odd_shapes(n, d, k):
    """Every E-step variant by shape (tensor core k <= 256, blocked tensor
    core k > 256, SIMT d > 128) against the oracle: lockstep steps, the final
    labels as the assignment of the returned centres, and the end-to-end fit.
    End to end the fit must equal the oracle's wherever the oracle's float32
    and float64 runs reach the same clustering; where they do not (the k = 257
    case is chaotic), it must reproduce one of those two runs."""
    rng = np.random.default_rng(n * 7 + d + k)
    X = (rng.standard_normal((n, d)) * 2 + 5).astype(np.float32)
    init = np.ascontiguousarray(X[rng.choice(n, k, replace=False)])
    lockstep(X, init, 2)
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, 20, 0.0)
    res = ora.kmeans_lloyd(X, init, 20, 0.0, relocation_order="sorted")
    res64 = ora.kmeans_lloyd(X, init, 20, 0.0, mode="fp64", relocation_order="sorted")
    assert c.shape == (k, d) and lab.shape == (n,)
    assert lab.min() >= 0 and lab.max() < k
    # the returned labels are the final E-step's assignment of the returned centres
    mean, Xc, _ = ora.center_data(X)
    want, _ = ora.assign(Xc, c - mean, "fp64")
    check_labels(Xc, c - mean, lab, want, "final labels vs returned centres")
    # inertia is consistent with the returned labels and centres
    assert inertia == pytest.approx(ora.inertia(X, c, lab), rel=1e-5, abs=1e-6)
    floor = float(np.mean(res64.labels == res.labels))
    if floor == 1.0 and res64.n_iter == res.n_iter:
        np.testing.assert_array_equal(lab, res.labels)
        assert n_iter == res.n_iter
        np.testing.assert_allclose(c, res.centers, rtol=CENTER_RTOL, atol=1e-5 * float(np.abs(X).max()))
        assert inertia == pytest.approx(res.inertia, rel=INERTIA_RTOL)
    else:
        # chaotic: the oracle's float32 and float64 runs end in different
        # clusterings; the fit must reproduce one of the two trajectories
        ref = max((res, res64), key=lambda r: float(np.mean(lab == r.labels)))
        assert np.mean(lab == ref.labels) >= 0.9999, (np.mean(lab == res.labels), np.mean(lab == res64.labels))
        assert n_iter == ref.n_iter
        assert inertia == pytest.approx(ref.inertia, rel=INERTIA_RTOL)


def test_last_fit_distinct_counts_final_labels():
    """The library counts the distinct final labels on the device (for
    scikit-learn's fewer-distinct-clusters warning): equal to the host count on
    a regular fit, below k when X has fewer distinct rows than k, and the
    estimator warns as scikit-learn does."""
    import warnings

    from sklearn.cluster import KMeans
    from sklearn.exceptions import ConvergenceWarning

    import skmetal_b200 as skmetal

    X, init = make_workload(scaled("c1", 20000))
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, 20, 0.0)
    assert _bridge.last_fit_distinct() == len(np.unique(lab))
    Xd = np.repeat(X[:3], 200, axis=0)  # three distinct rows, eight clusters
    init_d = np.ascontiguousarray(Xd[::75][:8])
    c, lab, inertia, n_iter = _bridge.kmeans_fit(Xd, init_d, 10, 0.0)
    assert _bridge.last_fit_distinct() == len(np.unique(lab)) <= 3
    with warnings.catch_warnings(record=True) as rec:
        warnings.simplefilter("always")
        skmetal.accelerate(KMeans(8, init=init_d, n_init=1, max_iter=10, tol=0)).fit(Xd)
    assert any(issubclass(r.category, ConvergenceWarning) for r in rec)


def test_fit_all_rows_identical():
    X = np.ones((500, 6), dtype=np.float32) * 3.5
    init = np.ascontiguousarray(X[:4])
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, init, 10, 0.0)
    from sklearn.cluster import KMeans
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        km = KMeans(4, init=init, n_init=1, max_iter=10, tol=0).fit(X)
    np.testing.assert_array_equal(lab, km.labels_)
    np.testing.assert_allclose(c, km.cluster_centers_)
    assert n_iter == km.n_iter_
    assert inertia == pytest.approx(0.0, abs=1e-6)


def test_fit_rejects_bad_input():
    X = np.ones((10, 3), dtype=np.float32)
    with pytest.raises(RuntimeError):
        _bridge.kmeans_fit(X, np.ones((11, 3), dtype=np.float32), 5, 0.0)  # k > n
    Xn = X.copy()
    Xn[3, 1] = np.nan
    with pytest.raises(RuntimeError):
        _bridge.kmeans_fit(Xn, Xn[:2].copy(), 5, 0.0)


@pytest.mark.parametrize("simt,name,n", [(False, "c1", 20000), (True, "c1", 20000), (False, "c4", 60000),
                                          (False, "c3", 40000)])
def test_incremental_sums_equal_bulk_sums(simt, name, n):
    """Fixed-point sums are exact: updating them with the rows that changed
    label must give bit-identical fits to recomputing them every iteration.
    c4 (k = 256) takes the persistent loop's atomic bulk pass and the
    epilogue's deltas; c3 (k = 1024) the wide E-step, whose deltas go through
    the deferred-delta ring, and the M-step kernel's global bulk sums."""
    X, init = make_workload(scaled(name, n))
    a = _bridge.kmeans_fit(X, init, 30, 0.0, simt=simt)
    b = _bridge.kmeans_fit(X, init, 30, 0.0, simt=simt, bulk_sums=True)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert a[2] == b[2] and a[3] == b[3]


def test_fit_prefix_consistency():
    """Centres after m iterations are the exact means of the labels after m-1
    (the final E-step labels of an (m-1)-iteration fit)."""
    X, init = make_workload(scaled("c1", 20000))
    mean, Xc, _ = ora.center_data(X)
    prev = _bridge.kmeans_fit(X, init, 1, 0.0)
    for m in range(2, 10):
        cur = _bridge.kmeans_fit(X, init, m, 0.0)
        ref, cnt = _fp64_centres(Xc, prev[1], init.shape[0], None)
        ok = cnt > 0
        np.testing.assert_allclose((cur[0] - mean)[ok], ref[ok], rtol=1e-5, atol=1e-5, err_msg=f"m={m}")
        prev = cur


def test_fit_is_deterministic():
    X, init = make_workload(scaled("c2", 20000))
    a = _bridge.kmeans_fit(X, init, 10, 0.0)
    b = _bridge.kmeans_fit(X, init, 10, 0.0)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert a[2] == b[2] and a[3] == b[3]


def _golden_gen(gen):
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location("make_golden", Path(__file__).parent / "golden" / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.case_inputs(gen)


@pytest.mark.parametrize("gen,max_iter,tol,bulk_sums", [
    ("reloc", 10, 0.0, False),                      # empty clusters relocated in the loop
    ("mixture:60000:100:50:1", 30, 0.0, False),     # C2 recipe: bulk iterations, relocation, deltas
    ("mixture:40000:32:8:0", 100, 1e-4, False),     # relative tolerance stop
    ("mixture:30000:100:50:1", 12, 0.0, True),      # bulk sums in every iteration
    ("mixture:20000:64:256:2", 15, 0.0, False),     # k = 256: two-segment centre image
    ("dirichlet:40000:64:128:3", 20, 0.0, False),   # C4 recipe, two accumulators
])
def test_persistent_loop_matches_launch_loop(monkeypatch, gen, max_iter, tol, bulk_sums):
    """The persistent loop kernel (one launch per fit) and the multi-launch
    loop (E-step and M-step kernels per iteration) run the same arithmetic in
    the same order: their fits are bit-identical."""
    X, init = _golden_gen(gen)
    a = _bridge.kmeans_fit(X, init, max_iter, tol, bulk_sums=bulk_sums)
    la = _bridge.last_fit_stats()["launches"]
    monkeypatch.setenv("SKMETAL_LOOP", "launches")
    b = _bridge.kmeans_fit(X, init, max_iter, tol, bulk_sums=bulk_sums)
    lb = _bridge.last_fit_stats()["launches"]
    assert a[3] == b[3]
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert a[2] == b[2]
    # the persistent loop really ran: a fixed number of launches, not ~2 per iteration
    assert la < 20 and lb >= 2 * b[3], (la, lb)


def test_dataset_fit_matches_host_fit():
    X, init = make_workload(scaled("c1", 10000))
    a = _bridge.kmeans_fit(X, init, 15, 0.0)
    ds = _bridge.Dataset(X)
    lab = np.empty(X.shape[0], dtype=np.int32)
    c, inertia, n_iter = ds.fit(init, 15, 0.0, labels_out=lab)
    np.testing.assert_array_equal(c, a[0])
    np.testing.assert_array_equal(lab, a[1])
    assert inertia == a[2] and n_iter == a[3]
    p = np.empty(X.shape[0], dtype=np.int32)
    ds.predict(c, p)
    q = np.empty(X.shape[0], dtype=np.int32)
    _bridge.kmeans_assign(X, c, q, X.shape[0], X.shape[1], c.shape[0])
    np.testing.assert_array_equal(p, q)
    ds.close()


def test_injected_failure_raises():
    X = np.ones((10, 3), dtype=np.float32)
    _bridge.debug_inject_failure(8, 0)
    with pytest.raises(RuntimeError, match="injected"):
        _bridge.kmeans_fit(X, X[:2].copy(), 5, 0.0)
    # the next call works again
    c, lab, inertia, n_iter = _bridge.kmeans_fit(X, X[:2].copy(), 5, 0.0)
    assert c.shape == (2, 3)


# ---------------------------------------------------------------------------
# predict: the small-d kernel with the centres in its parameter block
# ---------------------------------------------------------------------------

def test_predict_c5_recipe():
    """The C5 recipe (U[0,1)^8, 16 fixed centres) at 4M rows through the
    reference's assign entry point: labels against the float64 argmin,
    near-ties by the relative-gap rule only; a resident dataset's predict
    gives the same labels."""
    X, C = make_workload(scaled("c5", 4_000_000))
    lab = np.empty(X.shape[0], dtype=np.int32)
    _bridge.kmeans_assign(X, C, lab, X.shape[0], X.shape[1], C.shape[0])
    want, _ = ora.assign(X, C, "fp64")
    check_labels(X, C, lab, want, "predict c5", strict=True)
    ds = _bridge.Dataset(X)
    p = np.empty_like(lab)
    ds.predict(C, p)
    np.testing.assert_array_equal(p, lab)
    ds.close()


@pytest.mark.parametrize("d,k", [(8, 16), (8, 27), (4, 9), (16, 16)])
def test_predict_exact_ties_take_lowest_index(d, k):
    """Rows exactly halfway between two centres (dyadic values: every sum,
    difference and square is exact) tie in any arithmetic; the kernel must
    see that its expansion cannot decide them and fall back to direct
    differences with strict '<', i.e. the lower index (np.argmin's rule)."""
    rng = np.random.default_rng(d * 100 + k)
    C = (rng.integers(0, 64, (k, d)) / 64.0).astype(np.float32)
    pairs = [(a, b) for a in range(k) for b in range(a + 1, k)]
    X = np.concatenate([(C[[a for a, _ in pairs]] + C[[b for _, b in pairs]]) / 2,
                        (rng.integers(0, 64, (5000, d)) / 64.0)]).astype(np.float32)
    lab = np.empty(X.shape[0], dtype=np.int32)
    _bridge.kmeans_assign(X, C, lab, X.shape[0], d, k)
    D = ((X[:, None, :].astype(np.float64) - C[None].astype(np.float64)) ** 2).sum(-1)
    np.testing.assert_array_equal(lab, np.argmin(D, axis=1))


# ---------------------------------------------------------------------------
# full-size BASELINE workloads, one step each
# ---------------------------------------------------------------------------

def test_lloyd_step_full_size_c2():
    """The metric workload itself (C2: 500k x 100, k = 50): one Lloyd step
    from its explicit init in lockstep with the oracle."""
    X, init = make_workload("c2")
    reps = lockstep(X, init, 1, strict=True)
    assert reps[0]["agreement"] >= 0.9999


def test_estep_full_size_c3():
    """C3 at full size (2M x 128, k = 1024, the k > 256 tensor-core E-step):
    one step's labels against the oracle's float32 E-step, counts exact."""
    X, init = make_workload("c3")
    lab, cnew, weight, shift = _bridge.kmeans_lloyd_iter(X, init)
    want, _ = ora.assign(X, init, "fp32")
    check_labels(X, init, lab, want, "C3 full-size E-step", strict=True)
    np.testing.assert_array_equal(weight.astype(np.int64), np.bincount(lab, minlength=init.shape[0]))


def test_lloyd_step_c4_5m_rows():
    """The C4 recipe (Dirichlet-sized mixture, k = 256) at 5M rows: one Lloyd
    step in lockstep with the oracle."""
    X, init = make_workload(scaled("c4", 5_000_000))
    reps = lockstep(X, init, 1, strict=True)
    assert reps[0]["agreement"] >= 0.9999
