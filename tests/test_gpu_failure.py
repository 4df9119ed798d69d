"""Failure detection without a GPU fault: a wait on another rank runs out.

A sharded fit's persistent loop waits on its peers (the inbox polls of the
owners, the cross-rank barrier), every wait bounded by the peer-wait limit
(``SKMETAL_PEER_WAIT_MS``, 5 s by default). Here a one-GPU fit runs its loop
as rank 0 of two ranks whose rank 1 never starts
(``SKMETAL_DEBUG_ORPHAN_PEER=1``): its pushes land in a local stand-in region
and nothing ever writes the inbox words it polls. The poll runs out after the
limit, the kernel records error 1005, every CTA leaves the loop at the next
grid barrier (bounded too), the kernel exits normally and the call fails with
that code. The CUDA context stays usable: the next fit on the same thread
succeeds and equals a fit made before the failure."""

import time

import numpy as np
import pytest

from skmetal_b200 import _bridge
from skmetal_b200._synthetic import make_workload, scaled

pytestmark = pytest.mark.gpu


def test_peer_that_never_starts_times_out(monkeypatch):
    X, init = make_workload(scaled("c1", 20000))
    before = _bridge.kmeans_fit(X, init, 10, 0.0)
    monkeypatch.setenv("SKMETAL_DEBUG_ORPHAN_PEER", "1")
    monkeypatch.setenv("SKMETAL_PEER_WAIT_MS", "300")
    t0 = time.perf_counter()
    with pytest.raises(RuntimeError, match="code 1005"):
        _bridge.kmeans_fit(X, init, 10, 0.0)
    assert time.perf_counter() - t0 < 10.0
    monkeypatch.delenv("SKMETAL_DEBUG_ORPHAN_PEER")
    monkeypatch.delenv("SKMETAL_PEER_WAIT_MS")
    after = _bridge.kmeans_fit(X, init, 10, 0.0)
    np.testing.assert_array_equal(after[0], before[0])
    np.testing.assert_array_equal(after[1], before[1])
    assert after[2] == before[2] and after[3] == before[3]
