"""The tensor-core E-step for more than 256 clusters (the C3 codebook shape,
k = 1024, d = 128) through the C ABI, against the oracle.

The clusters are processed in blocks of at most 256 (one MMA's N) whose
centre units stream through shared memory; these tests cover the blocked
centre image bit for bit (probe), whole Lloyd steps in lockstep with the
oracle at k = 1024 and at an uneven k = 300 with d not a multiple of 8, a
step over enough rows that every CTA wraps its X stages and centre ring many
times, exact incremental sums, and full fits against the reference's own
outputs (golden fixtures)."""

import numpy as np
import pytest

from oracle import lloyd as ora
from skmetal_b200 import _bridge
from skmetal_b200._synthetic import gaussian_mixture, make_workload, scaled

from parity import CENTER_RTOL, INERTIA_RTOL, check_labels, lockstep, probe_c, probe_x

pytestmark = pytest.mark.gpu


def test_tensor_core_probe_wide():
    """The fp16 split of X, the blocked centre image (two blocks of 16) and the
    three-MMA sequence give the exact x_hi.c_hi + x_lo.c_hi + x_hi.c_lo."""
    mode, raw = _bridge.debug_tc_probe_wide()
    assert mode == 0, mode
    j = np.arange(16)
    x = probe_x(np.arange(128)[:, None], j[None, :])
    c = probe_c(np.arange(32)[:, None], j[None, :])
    xh, ch = np.round(x), np.round(c)
    want = (xh @ ch.T + (x - xh) @ ch.T + xh @ (c - ch).T).astype(np.float32)
    np.testing.assert_array_equal(raw.view(np.float32).reshape(128, 32), want)


def test_lloyd_step_lockstep_k1024():
    """C3 recipe (unit rows, k = 1024): four Lloyd steps from the oracle's
    centres, labels near-ties only by the relative-gap rule."""
    X, init = make_workload(scaled("c3", 20000))
    reps = lockstep(X, init, 4, strict=True)
    assert sum(r["mismatches"] for r in reps) <= 8


def test_lloyd_step_lockstep_k300_odd_d():
    """k = 300 (two blocks of 160, the last 10 clusters padding), d = 37
    (an odd number of 8-column chunks): empty clusters are relocated."""
    X, init = gaussian_mixture(9000, 37, 300, seed=4)
    lockstep(X, init, 4)


def test_wide_estep_many_tiles():
    """300k rows: every CTA runs ~16 tiles x 4 blocks x 8 column pairs, so its
    X stages, centre-unit ring and both accumulators wrap many times; one
    step's labels and counts against the oracle's E-step."""
    X, init = make_workload(scaled("c3", 300_000))
    lab, cnew, weight, shift = _bridge.kmeans_lloyd_iter(X, init)
    want, _ = ora.assign(X, init, "fp32")
    check_labels(X, init, lab, want, "k=1024 E-step", strict=True)
    np.testing.assert_array_equal(weight.astype(np.int64), np.bincount(lab, minlength=1024))


def test_wide_fit_uses_tensor_cores_and_matches_simt():
    """A k = 1024 fit runs the tensor-core E-step (few launches per
    iteration, no SIMT assignment) and agrees with the SIMT E-step fit after
    one iteration (later iterations amplify rounding differences)."""
    X, init = make_workload(scaled("c3", 40000))
    a = _bridge.kmeans_fit(X, init, 1, 0.0)
    b = _bridge.kmeans_fit(X, init, 1, 0.0, simt=True)
    mean, Xc, _ = ora.center_data(X)
    check_labels(Xc, b[0] - mean, a[1], b[1], "tc vs simt (k=1024)")
    np.testing.assert_allclose(a[0], b[0], rtol=CENTER_RTOL, atol=1e-5)
    assert a[2] == pytest.approx(b[2], rel=1e-5)


def test_wide_incremental_sums_equal_bulk_sums():
    """Fixed-point sums are exact at k = 1024 too: updating them with the rows
    that changed label gives the same bits as rebuilding them every iteration."""
    X, init = make_workload(scaled("c3", 30000))
    a = _bridge.kmeans_fit(X, init, 8, 0.0)
    b = _bridge.kmeans_fit(X, init, 8, 0.0, bulk_sums=True)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert a[2] == b[2] and a[3] == b[3]
