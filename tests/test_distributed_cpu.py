"""Multi-GPU host logic on CPU: two gloo ranks (no GPU).

* row sharding: contiguous, disjoint shards covering every row;
* communicator set-up: every rank joins with the unique id made by rank 0
  (the library is replaced by a recording stand-in);
* max-over-ranks timing reduction;
* the reason the sharded fit is deterministic: the per-iteration cluster sums
  are exact fixed-point integers (scale 2^F with F = 62 - E - L, as the
  library's fixed_scale), so their all-reduce over shards equals the sums of
  the whole dataset bit for bit, whatever the number of ranks.
"""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from skmetal_b200.distributed import init_library_comm, max_over_ranks, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _RecordingBridge:
    def __init__(self, rank):
        self.rank = rank
        self.joined = None

    def comm_unique_id(self):
        assert self.rank == 0, "only rank 0 makes the unique id"
        return bytes(range(128))

    def comm_init(self, uid, world, rank):
        self.joined = (uid, world, rank)


def _fixed_sums(X, labels, k, n_total, maxabs):
    """Exact per-cluster fixed-point sums and counts (the library's scheme)."""
    E = np.frexp(np.float64(maxabs))[1] if maxabs > 0 else -60
    L = np.frexp(np.float64(max(n_total, 1)))[1]
    scale = np.ldexp(1.0, 62 - E - L)
    fx = np.rint(X.astype(np.float64) * scale).astype(np.int64)
    S = np.zeros((k, X.shape[1]), dtype=np.int64)
    np.add.at(S, labels, fx)
    return S, np.bincount(labels, minlength=k).astype(np.int64)


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        br = _RecordingBridge(rank)
        uid = init_library_comm(br, dist, rank, world)
        rng = np.random.default_rng(5)
        n, d, k = 1001, 7, 5
        X = (rng.standard_normal((n, d)) * 4).astype(np.float32)
        labels = rng.integers(0, k, n)
        lo, hi = shard_range(n, rank, world)
        S, c = _fixed_sums(X[lo:hi], labels[lo:hi], k, n, float(np.abs(X).max()))
        ts, tc = torch.from_numpy(S), torch.from_numpy(c)
        dist.all_reduce(ts)
        dist.all_reduce(tc)
        t = max_over_ranks(dist, [1.0 + rank, 5.0 - rank])
        out.put((rank, br.joined, uid, (lo, hi), ts.numpy(), tc.numpy(), t))
    finally:
        dist.destroy_process_group()


def test_shard_range_covers_rows():
    for n in (0, 1, 7, 1000, 500_001):
        for w in (1, 2, 3, 8):
            rngs = [shard_range(n, r, w) for r in range(w)]
            assert rngs[0][0] == 0 and rngs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rngs, rngs[1:]))
            assert max(h - l for l, h in rngs) - min(h - l for l, h in rngs) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    uid0 = res[0][2]
    for rank, joined, uid, _, _, _, t in res:
        assert joined == (uid0, world, rank)
        assert t == [2.0, 5.0]
    assert res[0][3] == (0, 500) and res[1][3] == (500, 1001)
    # sharded exact sums == whole-dataset sums, bit for bit
    rng = np.random.default_rng(5)
    X = (rng.standard_normal((1001, 7)) * 4).astype(np.float32)
    labels = rng.integers(0, 5, 1001)
    S, c = _fixed_sums(X, labels, 5, 1001, float(np.abs(X).max()))
    for r in res:
        np.testing.assert_array_equal(r[4], S)
        np.testing.assert_array_equal(r[5], c)
