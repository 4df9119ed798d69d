"""Sharded fits on two GPUs against the single-GPU fit (skipped with fewer GPUs).

Two processes, one per GPU, each fit their row shard through
``skmetal_kmeans_fit_shard``, with either loop:
- persistent: one loop kernel per rank; the ranks read each other's
  fixed-point deltas and relocation candidates over NVLink from their peer
  regions, synchronised by cross-rank arrival words;
- launches: kernels per iteration and an NCCL all-reduce of the sums and
  candidates.
The sums are exact integers, so both ranks must return the single-GPU fit's
centres and n_iter bit for bit, and the single-GPU labels on their rows;
inertia is a float64 sum in another order (rtol 1e-12).

Rendezvous (the NCCL unique id) goes over a gloo group on 127.0.0.1 with a
short timeout; NVLS is off.
"""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = {
    # k = 20 on 5 blobs with a duplicate-heavy init: empty clusters to relocate
    "relocation": dict(gen="reloc", max_iter=10, tol=0.0),
    # the C2 recipe at 60k rows: 4 empty clusters in iteration 2, then 30 iterations
    "c2_60k": dict(gen="mixture:60000:100:50:1", max_iter=30, tol=0.0),
    # relative tolerance: the stop decision must agree on both ranks
    "tol": dict(gen="mixture:40000:32:8:0", max_iter=100, tol=1e-4),
    # one empty cluster: each rank offers its single farthest row
    "one_empty": dict(gen="reloc1", max_iter=30, tol=0.0),
}


def _gpu_count():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:  # noqa: BLE001
        return 0


def _inputs(gen):
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location("make_golden", Path(__file__).parent / "golden" / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.case_inputs(gen)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, case, loop, out):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      SKMETAL_COMM_TIMEOUT_S="60", SKMETAL_LOOP=loop)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from skmetal_b200 import _bridge
    from skmetal_b200.distributed import init_library_comm, shard_range

    try:
        _bridge.set_device(rank)
        init_library_comm(_bridge, dist, rank, world)
        X, init = _inputs(case["gen"])
        lo, hi = shard_range(X.shape[0], rank, world)
        c, lab, inertia, n_iter = _bridge.kmeans_fit_shard(X[lo:hi], init, case["max_iter"], case["tol"], lo,
                                                           X.shape[0])
        launches = _bridge.last_fit_stats()["launches"]
        out.put((rank, "ok", c, lab, inertia, n_iter, lo, hi, launches))
    except Exception as e:  # noqa: BLE001
        out.put((rank, f"error: {e}", None, None, None, None, None, None, None))
    finally:
        _bridge.comm_destroy()
        dist.destroy_process_group()


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("loop", ["persistent", "launches"])
def test_two_gpu_shards_match_one_gpu(name, loop):
    import torch.multiprocessing as mp

    from skmetal_b200 import _bridge

    case = CASES[name]
    X, init = _inputs(case["gen"])
    c1, l1, i1, n1 = _bridge.kmeans_fit(X, init, case["max_iter"], case["tol"])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, case, loop, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for rank, status, c, lab, inertia, n_iter, lo, hi, launches in res:
        assert status == "ok", f"rank {rank}: {status}"
        # the loop asked for ran: one loop kernel, or kernels per iteration
        assert (launches < 20) if loop == "persistent" else (launches >= 2 * n_iter), (loop, launches)
        assert n_iter == n1
        np.testing.assert_array_equal(c, c1)
        np.testing.assert_array_equal(lab, l1[lo:hi])
        assert inertia == pytest.approx(i1, rel=1e-12)
    assert all(p.exitcode == 0 for p in procs)
