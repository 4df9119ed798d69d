"""Benchmark: Lloyd rows x iterations / s on the KMeans metric workload.

Default workload (BASELINE.json ``configs[1]``): X 500,000 x 100 fp32 from a
50-component Gaussian mixture (seed 1), k = 50, explicit init = 50 seeded rows,
n_init = 1, max_iter = 100, tol = 0. One *step* is one full fit (all its Lloyd
iterations, the final E-step and the inertia).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]

* ``value``: whole-job rows x iterations / s with X already resident in HBM
  (device time of the fit, CUDA events on the library's stream; max over ranks).
* ``e2e``: the same metric through the public C-ABI call with host buffers
  (pinned X in, labels/centres out, host<->device copies inside the timed region).
* ``roofline``: the dominant kernel against the measured HBM copy bandwidth;
  algorithmic bytes = 4 n d per Lloyd iteration (X read once). On one GPU it
  is the persistent loop kernel (one launch runs every iteration of a fit),
  timed with CUDA events around its launch; ``e_phase`` splits out the E-step
  part of an iteration from the kernel's device timestamps. With N > 1 GPUs
  (multi-launch loop) it is the E-step kernel, timed with CUDA events on the
  E-step launches of every 10th iteration. ``traffic`` = DRAM bytes per launch
  from the committed ncu summary (profiles/), scaled to this run's rows and
  iterations.
* ``cpu_baseline`` (rank 0, N = 1): scikit-learn's Lloyd (the reference's CPU
  path) on a bounded sample of the same workload.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): weak scaling.
Every GPU holds as many rows as the N = 1 workload (500,000 for C2) of one
dataset of N times that size drawn with the same recipe; rank r fits its
contiguous shard and the library all-reduces the per-iteration k x d sums and
k counts with NCCL. ``value`` counts the rows of all GPUs.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Lloyd rows x iters/s (500k x 100, k=50)"
UNIT = "rows*iters/s"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, read through NVML
    every 5 ms on a background thread while the timed region runs."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.sm: list[float] = []
        self.reasons: set[str] = set()
        self.sm_max = None
        self.error = None
        self._stop = threading.Event()
        self.t = None

    def _handle(self, nv):
        import torch

        props = torch.cuda.get_device_properties(self.cuda_index)
        try:
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # noqa: BLE001
            return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def start(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            self.nv = nv
            self.h = self._handle(nv)
            self.sm_max = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # noqa: BLE001
            self.error = f"nvml unavailable: {e}"

    def _sample(self):
        nv = self.nv
        self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
        bits = int(self.get_reasons(self.h))
        for name, const in self.REASONS:
            if bits & int(getattr(nv, const, 0)):
                self.reasons.add(name)

    def _run(self):
        while not self._stop.wait(self.period):
            try:
                self._sample()
            except Exception:  # noqa: BLE001
                return

    def stop(self) -> dict:
        if self.error:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error], "samples": 0}
        self._stop.set()
        if self.t is not None:
            self.t.join(timeout=5)
        try:
            self._sample()
        except Exception:  # noqa: BLE001
            pass
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.sm_max,
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml, 5 ms"}


def _traffic_for(kernel: str, config: str, rows: int, iters: float = 1.0):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu
    summary profiles/<kernel>_<config>.md, scaled by rows (and by Lloyd
    iterations for the loop kernel, whose launch runs all of them) when this
    run differs from the captured one; None without a summary."""
    import re

    p = ROOT / "profiles" / f"{kernel}_{config}.md"
    if not p.exists():
        return None
    text = p.read_text()
    m = re.search(r"traffic_bytes_per_launch = (\d+)", text)
    n = re.search(r"\((\d[\d,]*) x \d+, k = \d+\)", text)
    if not m or not n:
        return None
    scale = rows / int(n.group(1).replace(",", ""))
    it = re.search(r"iterations_per_launch = (\d+)", text)
    if it:
        scale *= iters / int(it.group(1))
    return float(m.group(1)) * scale


def cpu_baseline(X, init, k, sample_iters: int):
    """scikit-learn's Lloyd (the reference's CPU path) on a bounded sample."""
    from sklearn.cluster import KMeans
    from threadpoolctl import threadpool_info
    from sklearn.utils._openmp_helpers import _openmp_effective_n_threads

    times, iters = [], []
    for _ in range(2):
        t0 = time.perf_counter()
        km = KMeans(k, init=init, n_init=1, max_iter=sample_iters, tol=0, algorithm="lloyd").fit(X)
        times.append(time.perf_counter() - t0)
        iters.append(km.n_iter_)
    t = statistics.median(times)
    cores = _openmp_effective_n_threads()
    blas = [f"{i.get('internal_api')}:{i.get('num_threads')}" for i in threadpool_info()]
    return {"value": X.shape[0] * iters[0] / t, "unit": UNIT, "cores": int(cores), "kind": "reference",
            "sample": (f"sklearn {__import__('sklearn').__version__} KMeans(lloyd, n_init=1, tol=0) on the full "
                       f"{X.shape[0]}x{X.shape[1]} k={k} workload, max_iter={sample_iters} "
                       f"(median of 2 fits, {t:.2f}s each); threads {blas}")}


def run_reference(args, w, X, init):
    """--impl reference: the reference's own CPU implementation of the path."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from sklearn.cluster import KMeans
    from sklearn.utils._openmp_helpers import _openmp_effective_n_threads

    # a bounded sample per step: about 20 x 500k row-iterations whatever N is
    world = int(os.environ.get("WORLD_SIZE", "1"))
    sample_iters = max(2, round(20 / world))
    for _ in range(args.warmup):
        KMeans(w.k, init=init, n_init=1, max_iter=sample_iters, tol=0, algorithm="lloyd").fit(X)
    rows_iters, t_total = 0, 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        km = KMeans(w.k, init=init, n_init=1, max_iter=sample_iters, tol=0, algorithm="lloyd").fit(X)
        t_total += time.perf_counter() - t0
        rows_iters += X.shape[0] * km.n_iter_
    v = rows_iters / t_total
    cores = _openmp_effective_n_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture, BASELINE configs[1])",
        "config": {"workload": w.name, "n": w.n, "d": w.d, "k": w.k, "max_iter": sample_iters, "tol": 0,
                   "parallelism": "cpu threads"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": int(cores), "kind": "reference",
                         "sample": f"scikit-learn {__import__('sklearn').__version__} Lloyd, max_iter={sample_iters} "
                                   f"per step on the full {w.n}x{w.d} k={w.k} workload"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2")
    ap.add_argument("--rows", type=int, default=0, help="override n (testing)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()

    from skmetal_b200._synthetic import WORKLOADS, make_workload, scaled

    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    rows_per_gpu = args.rows or WORKLOADS[args.config].n
    # Weak scaling: every GPU holds rows_per_gpu rows of the same recipe; at
    # N = 1 the workload is exactly the metric's configuration.
    w = scaled(args.config, rows_per_gpu * world_env) if (args.rows or world_env > 1) else WORKLOADS[args.config]
    X, init = make_workload(w)
    if args.impl == "reference":
        run_reference(args, w, X, init)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from skmetal_b200 import _bridge

    _bridge.set_device(local)
    _bridge.ensure_warmed_up()
    from skmetal_b200.distributed import init_library_comm, max_over_ranks, shard_range

    if world > 1:
        init_library_comm(_bridge, dist, rank, world)

    n = X.shape[0]
    lo, hi = shard_range(n, rank, world)
    Xs = np.ascontiguousarray(X[lo:hi])
    shard = (lo, n) if world > 1 else None
    ds = _bridge.Dataset(Xs)
    labels = np.empty(Xs.shape[0], dtype=np.int32)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        ds.fit(init, w.max_iter, 0.0, shard=shard)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    l0 = _bridge.launch_count()
    ms_total, ms_loop, est_ms, est_n, iters = 0.0, 0.0, 0.0, 0, 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _, _, n_iter = ds.fit(init, w.max_iter, 0.0, profile=True, shard=shard)
        st = _bridge.last_fit_stats()
        ms_total += st["ms_total"]
        ms_loop += st["ms_loop"]
        est_ms += st["estep_ms_sum"]
        est_n += st["estep_launches"]
        iters += n_iter
    wall = time.perf_counter() - t0
    launches = _bridge.launch_count() - l0
    persistent = len(_bridge.debug_loop_stamps()) > 0  # the profiled fits ran the loop kernel
    barrier()
    clk = clocks.stop()
    t_dev = ms_total / 1e3
    if dist is not None:
        t_dev, wall = max_over_ranks(dist, [t_dev, wall], device="cuda")
    rows_iters = n * iters  # every rank ran the same iterations over its shard of n rows
    value = rows_iters / t_dev

    # end to end through the host-buffer C-ABI call (pinned X in, labels + centres out)
    Xp = torch.empty(Xs.shape, dtype=torch.float32, pin_memory=True).numpy()
    Xp[...] = Xs
    lab_p = torch.empty(Xs.shape[0], dtype=torch.int32, pin_memory=True).numpy()
    e2e_steps = max(1, min(args.steps, 3))

    def e2e_fit():
        if world > 1:
            return _bridge.kmeans_fit_shard(Xp, init, w.max_iter, 0.0, lo, n)[3]
        return _bridge.kmeans_fit(Xp, init, w.max_iter, 0.0)[3]

    e2e_fit()  # untimed warm-up of the host-buffer path (its first call sets up staging)
    barrier()
    t0 = time.perf_counter()
    e2e_iters = 0
    for _ in range(e2e_steps):
        e2e_iters += e2e_fit()
    e2e_t = time.perf_counter() - t0
    if dist is not None:
        (e2e_t,) = max_over_ranks(dist, [e2e_t], device="cuda")
    e2e_value = n * e2e_iters / e2e_t

    hbm, bf16, src = _peaks()
    alg_bytes = 4.0 * Xs.shape[0] * w.d  # X read once per Lloyd iteration
    est_avg_s = est_ms / max(1, est_n) / 1e3
    e_achieved = alg_bytes / est_avg_s / 1e9 if est_avg_s > 0 else None
    if persistent:
        per_launch = alg_bytes * iters / args.steps  # one launch per fit, all its iterations
        dur_s = ms_loop / 1e3 / args.steps
        achieved = per_launch / dur_s / 1e9 if dur_s > 0 else None
        traffic = _traffic_for("lloyd_loop", w.name, Xs.shape[0], iters / args.steps)
        kernel = "lloyd_loop_kernel (persistent: every Lloyd iteration of a fit in one launch)"
        e_timing = "device globaltimer stamps of every iteration (E-step through the grid barrier)"
    else:
        per_launch = alg_bytes
        achieved = e_achieved
        traffic = _traffic_for("estep_tc", w.name, Xs.shape[0])
        kernel = "E-step (estep_tc_kernel)"
        e_timing = "CUDA events on the E-step launches of every 10th iteration"
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": (achieved / hbm) if achieved else None, "traffic": traffic, "kernel": kernel,
                "peak_source": src, "algorithmic_bytes_per_launch": per_launch,
                "e_phase": {"achieved": e_achieved, "frac": (e_achieved / hbm) if e_achieved else None,
                            "timing": e_timing},
                "loop_frac": (alg_bytes * iters / (ms_loop / 1e3)) / 1e9 / hbm if ms_loop > 0 else None}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_dev / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture, BASELINE configs[1]); X resident in HBM",
        "config": {"workload": w.name, "n": n, "n_per_gpu": n // world, "d": w.d, "k": w.k,
                   "max_iter": w.max_iter, "tol": 0, "iters_per_step": iters / args.steps,
                   "parallelism": f"rows sharded x{world} (weak scaling: {n // world} rows per GPU)",
                   "l2": "X (%.0f MB per GPU) > L2 (126 MB) between iterations" % (alg_bytes / 1e6)},
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": int(Xs.nbytes + init.nbytes),
                "d2h_bytes_per_step": int(Xs.shape[0] * 4 + init.nbytes + 12)},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "clocks": clk,
        "wall_s": wall,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(X, init, w.k, sample_iters=20)
    if world > 1:
        _bridge.comm_destroy()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
