"""Benchmark: Lloyd rows x iterations / s on the KMeans workloads.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config c1|c2|c3|c4|c5] [--scaling weak|strong]

Default (no flags): ``configs[1]`` of BASELINE.json on one GPU -- X 500,000 x
100 fp32 from a 50-component Gaussian mixture (seed 1), k = 50, explicit init =
50 seeded rows, n_init = 1, max_iter = 100, tol = 0. One *step* is one full fit
(all its Lloyd iterations, the final E-step and the inertia). ``c5`` is the
predict workload (400M x 8, 16 fixed centres): a step is one assignment pass.

* ``value``: whole-job rows x iterations / s (rows / s for c5) with X already
  resident in HBM: device time of the fit (CUDA events on the library's
  stream), max over ranks.
* ``e2e``: the same metric through the public API a user calls --
  ``skmetal_b200.accelerate(KMeans(...)).fit(X)`` (``.predict`` for c5) on one
  GPU, the sharded C-ABI fit on several -- with X in ordinary (pageable)
  host memory, its upload and the labels' / centres' download inside the
  timed region. ``e2e_pinned`` repeats it from page-locked host memory.
* ``roofline``: the dominant kernel against ``MEASURED_PEAKS.json``. A Lloyd
  iteration reads X once (4 n d bytes) and runs 3 (2 n k d) tensor flops; its
  roofline is the slower of the two at the measured copy bandwidth and bf16
  burst peak (the MMAs are kind::f16), so c1 and c2 are HBM-bound and c3 and
  c4 tensor-bound. Fits with k <= 256 (c1, c2, c4): the persistent loop
  kernel, one launch per fit; the k > 256 codebook fit (c3): the tensor-core
  E-step launches. Predict (c5): the assignment kernel, 4 n d + 4 n bytes per
  pass.
  ``traffic`` = DRAM bytes per launch from the committed ncu summary
  (profiles/), scaled to this run's rows and iterations.
* ``cpu_baseline`` (rank 0, N = 1): the reference's CPU path on a bounded
  sample of the same workload, with every host core.

``--impl reference`` times the reference's own CPU implementation of the path
-- ``skmetal.accelerate(KMeans(...)).fit`` of the reference package installed
in ``baseline/_ref``, which on a machine without Apple Metal is scikit-learn's
Lloyd -- on rank 0 with every host core; the other ranks exit.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``), one process per
GPU. ``weak`` (default for c1, c2): every GPU holds as many rows as the N = 1
workload, of one dataset of N times that size drawn with the same recipe.
``strong`` (default for c3, c4, c5): the N = 1 workload's rows split over the
N GPUs. Rank r fits its contiguous shard; the library exchanges the
per-iteration k x d sums and k counts between the GPUs over NVLink. Predict
needs no exchange: every rank labels its own rows.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
REF_SITE = ROOT / "baseline" / "_ref"

UNIT_FIT = "rows*iters/s"
UNIT_PREDICT = "rows/s"
DEFAULT_SCALING = {"c1": "weak", "c2": "weak", "c3": "strong", "c4": "strong", "c5": "strong"}
# the reference arm's per-step sample on workloads whose full fit takes the
# host minutes: (rows, Lloyd iterations) per step
REF_SAMPLE = {"c3": (2_000_000, 2), "c4": (4_000_000, 2), "c5": (50_000_000, 1)}


def _metric(w) -> str:
    if w.kind == "predict":
        return f"KMeans.predict rows/s ({w.n // 1_000_000}M x {w.d}, k={w.k})"
    n = f"{w.n // 1000}k" if w.n < 1_000_000 else f"{w.n // 1_000_000}M"
    return f"Lloyd rows x iters/s ({n} x {w.d}, k={w.k})"


def _config(w, n_total: int, world: int, scaling: str) -> dict:
    """The workload as both arms name it (identical dicts for the same run)."""
    per_gpu = n_total // world
    c = {"workload": w.name, "n": n_total, "n_per_gpu": per_gpu, "d": w.d, "k": w.k,
         "scaling": scaling,
         "l2": "X (%.0f MB per GPU) %s L2 (126 MB) between passes" % (
             4.0 * per_gpu * w.d / 1e6, ">" if 4.0 * per_gpu * w.d > 126e6 else "<")}
    if w.kind == "fit":
        c.update({"max_iter": w.max_iter, "tol": 0, "init": "explicit array of k seeded rows", "n_init": 1})
    return c


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)),
                float(d.get("bf16_tflops_sustained", 1400.0)), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def _host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


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
    iterations for a launch that runs several) when this run differs from the
    captured one; None without a summary."""
    import re

    p = ROOT / "profiles" / f"{kernel}_{config}.md"
    if not p.exists():
        return None
    text = p.read_text()
    m = re.search(r"traffic_bytes_per_launch = (\d+)", text)
    n = re.search(r"rows_per_launch = (\d+)", text) or re.search(r"\((\d[\d,]*) x \d+, k = \d+\)", text)
    if not m or not n:
        return None
    scale = rows / int(n.group(1).replace(",", ""))
    it = re.search(r"iterations_per_launch = (\d+)", text)
    if it:
        scale *= iters / int(it.group(1))
    return float(m.group(1)) * scale


# ---------------------------------------------------------------------------
# the reference's CPU path
# ---------------------------------------------------------------------------

def _reference_kmeans():
    """``skmetal.accelerate`` and scikit-learn's ``KMeans`` from the reference
    package installed in baseline/_ref (its stock public API)."""
    if str(REF_SITE) not in sys.path:
        sys.path.insert(0, str(REF_SITE))
    import warnings

    with warnings.catch_warnings():
        warnings.simplefilter("ignore")  # "Metal GPU not available": the reference's CPU path
        import skmetal
        from sklearn.cluster import KMeans
    if not Path(skmetal.__file__).resolve().is_relative_to(REF_SITE.resolve()):
        raise RuntimeError(f"reference package not loaded from {REF_SITE} ({skmetal.__file__})")
    return skmetal.accelerate, KMeans


def _ref_fit(accelerate, KMeans, X, init, max_iter):
    est = accelerate(KMeans(n_clusters=init.shape[0], init=init, n_init=1, max_iter=max_iter, tol=0,
                            algorithm="lloyd"))
    t0 = time.perf_counter()
    est.fit(X)
    return time.perf_counter() - t0, int(est.n_iter_)


def _ref_predict(accelerate, KMeans, X, centers):
    est = accelerate(KMeans(n_clusters=centers.shape[0], init=centers, n_init=1, max_iter=1))
    est.fit(X[:max(centers.shape[0], 1000)])
    est.cluster_centers_ = centers.copy()
    t0 = time.perf_counter()
    est.predict(X)
    return time.perf_counter() - t0


def _ref_sample(w, n_total: int, world: int):
    """(rows, iterations) of one reference step: the full workload at N = 1
    for c1 / c2; a bounded sample otherwise (the metric is per row-iteration)."""
    if w.name in REF_SAMPLE:
        r, it = REF_SAMPLE[w.name]
        return min(r, n_total), it
    if world == 1:
        return n_total, w.max_iter
    return n_total, max(2, round(w.max_iter / world))


def _ref_threads_info():
    from threadpoolctl import threadpool_info

    return [f"{i.get('internal_api')}:{i.get('num_threads')}" for i in threadpool_info()]


def cpu_baseline(w, X, init) -> dict:
    """The reference's CPU path on a bounded sample (about 10-30 s of work)."""
    from threadpoolctl import threadpool_limits

    accelerate, KMeans = _reference_kmeans()
    cores = _host_cores()
    with threadpool_limits(cores):
        if w.kind == "predict":
            m = min(X.shape[0], 50_000_000)
            ts = [_ref_predict(accelerate, KMeans, X[:m], init) for _ in range(2)]
            t = statistics.median(ts)
            return {"value": m / t, "unit": UNIT_PREDICT, "cores": cores, "kind": "reference",
                    "sample": f"skmetal.accelerate(KMeans).predict (reference, baseline/_ref: scikit-learn "
                              f"{__import__('sklearn').__version__}) on the first {m} rows, median of 2 "
                              f"({t:.2f} s each); threads {_ref_threads_info()}"}
        rows, iters = _ref_sample(w, X.shape[0], 1)
        rows = min(rows, X.shape[0])
        runs = [_ref_fit(accelerate, KMeans, X[:rows], init, iters) for _ in range(2)]
        t = statistics.median(r[0] for r in runs)
        return {"value": rows * runs[0][1] / t, "unit": UNIT_FIT, "cores": cores, "kind": "reference",
                "sample": f"skmetal.accelerate(KMeans(lloyd, n_init=1, tol=0)).fit (reference, baseline/_ref: "
                          f"scikit-learn {__import__('sklearn').__version__}) on {rows}x{w.d} k={w.k}, "
                          f"max_iter={iters}, median of 2 fits ({t:.2f} s each); threads {_ref_threads_info()}"}


def run_reference(args, w, n_total, world, scaling):
    """--impl reference: the reference's own CPU implementation of the path."""
    from threadpoolctl import threadpool_limits

    from skmetal_b200._synthetic import make_rows

    cores = _host_cores()
    accelerate, KMeans = _reference_kmeans()
    rows, iters = _ref_sample(w, n_total, world)
    X, init = make_rows(w.__class__(w.name, n_total, w.d, w.k, w.max_iter, w.seed, w.kind, w.description), 0, rows)
    total_units, t_total = 0, 0.0
    with threadpool_limits(cores):
        for _ in range(args.warmup):
            if w.kind == "predict":
                _ref_predict(accelerate, KMeans, X, init)
            else:
                _ref_fit(accelerate, KMeans, X, init, iters)
        for _ in range(args.steps):
            if w.kind == "predict":
                t_total += _ref_predict(accelerate, KMeans, X, init)
                total_units += X.shape[0]
            else:
                t, n_iter = _ref_fit(accelerate, KMeans, X, init, iters)
                t_total += t
                total_units += X.shape[0] * n_iter
        threads = _ref_threads_info()
    v = total_units / t_total
    unit = UNIT_PREDICT if w.kind == "predict" else UNIT_FIT
    sample = (f"skmetal.accelerate(KMeans).{'predict' if w.kind == 'predict' else 'fit'} of the reference package "
              f"(baseline/_ref; scikit-learn {__import__('sklearn').__version__} Lloyd on this host) per step on "
              f"{rows} of the workload's {n_total} rows" + ("" if w.kind == "predict" else f", max_iter={iters}")
              + f"; {cores} host threads {threads}")
    line = {
        "impl": "reference", "metric": _metric(w), "value": v, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_total / args.steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded, BASELINE {w.name} recipe)",
        "config": _config(w, n_total, world, scaling),
        "parallelism": f"{cores} host threads",
        "cpu_baseline": {"value": v, "unit": unit, "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# this library
# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"])
    ap.add_argument("--rows", type=int, default=0, help="override the N = 1 row count (testing)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end legs (profiling runs)")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    scaling = args.scaling or DEFAULT_SCALING[args.config]

    if args.impl == "reference":
        if rank != 0:
            return
        # torchrun sets OMP_NUM_THREADS=1; the reference's CPU path gets every host core
        for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
            os.environ[v] = str(_host_cores())

    from skmetal_b200._synthetic import WORKLOADS, Workload, make_rows

    w = WORKLOADS[args.config]
    base_rows = args.rows or w.n
    n_total = base_rows * world if scaling == "weak" else base_rows
    wt = Workload(w.name, n_total, w.d, w.k, w.max_iter, w.seed, w.kind, w.description)
    if args.impl == "reference":
        run_reference(args, wt, n_total, world, scaling)
        return

    import numpy as np
    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from skmetal_b200 import _bridge
    from skmetal_b200.distributed import init_library_comm, max_over_ranks, shard_range

    lo, hi = shard_range(n_total, rank, world)
    Xs, init = make_rows(wt, lo, hi)
    _bridge.set_device(local)
    _bridge.ensure_warmed_up()
    fit = w.kind == "fit"
    if world > 1 and fit:
        init_library_comm(_bridge, dist, rank, world)
    shard = (lo, n_total) if (world > 1 and fit) else None
    ds = _bridge.Dataset(Xs)
    labels = np.empty(Xs.shape[0], dtype=np.int32)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    last_fit = {}

    def step(profile):
        if fit:
            c, _, n_it = ds.fit(init, w.max_iter, 0.0, profile=profile, shard=shard)
            last_fit["c"], last_fit["n_iter"] = c, n_it
            return n_it
        ds.predict(init, labels)
        return 1

    for _ in range(args.warmup):
        step(False)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    l0 = _bridge.launch_count()
    ms_total, ms_loop, est_ms, est_n, iters = 0.0, 0.0, 0.0, 0, 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        iters += step(True)
        st = _bridge.last_fit_stats()
        ms_total += st["ms_total"]
        ms_loop += st["ms_loop"]
        est_ms += st["estep_ms_sum"]
        est_n += st["estep_launches"]
    wall = time.perf_counter() - t0
    launches = _bridge.launch_count() - l0
    stamps = _bridge.debug_loop_stamps() if fit else []
    persistent = len(stamps) > 0  # the profiled fits ran the loop kernel
    phases = None
    if persistent:
        # device timestamps of the last fit: per iteration [start, E-step done,
        # owners done, M-step done]; bulk / relocation iterations show a long M-step
        T = (len(stamps) - 1) // 4
        st4 = np.asarray(stamps[:4 * T], dtype=np.float64).reshape(T, 4) / 1e3  # us
        e_us = st4[:, 1] - st4[:, 0]
        m_us = np.concatenate([st4[1:, 0] - st4[:-1, 1], [stamps[4 * T] / 1e3 - st4[-1, 1]]])
        phases = {"iterations": int(T), "estep_us_median": float(np.median(e_us)), "estep_us_sum": float(e_us.sum()),
                  "mstep_us_median": float(np.median(m_us)), "mstep_us_sum": float(m_us.sum()),
                  "mstep_over_2x_median": int((m_us > 2 * np.median(m_us)).sum()),
                  "timing": "globaltimer stamps of the loop kernel (last timed fit)"}
    barrier()
    clk = clocks.stop()
    t_dev = ms_total / 1e3
    if dist is not None:
        t_dev, wall = max_over_ranks(dist, [t_dev, wall], device="cuda")
    ranks_agree = None
    if dist is not None and fit:
        # a sharded fit returns the same centres and n_iter on every rank (the
        # sums are exact integers): compare a hash of them across ranks
        import hashlib

        h = hashlib.sha256(last_fit["c"].tobytes() + int(last_fit["n_iter"]).to_bytes(4, "little")).digest()
        hv = torch.tensor([int.from_bytes(h[:7], "little")], dtype=torch.int64, device="cuda")
        hmin, hmax = hv.clone(), hv.clone()
        dist.all_reduce(hmin, op=dist.ReduceOp.MIN)
        dist.all_reduce(hmax, op=dist.ReduceOp.MAX)
        ranks_agree = bool(hmin.item() == hmax.item())
    units = n_total * iters  # every rank ran the same iterations over its shard
    value = units / t_dev
    unit = UNIT_FIT if fit else UNIT_PREDICT

    # ---- end to end through the public API, pageable host X (and pinned)
    e2e, e2e_pinned, e2e_calls, e2e_pinned_calls = None, None, None, None
    h2d = int(Xs.nbytes + init.nbytes)
    d2h = int(Xs.shape[0] * 4 + (init.nbytes + 12 if fit else 0))
    if not args.no_e2e:
        from sklearn.cluster import KMeans

        import skmetal_b200

        def e2e_call(X):
            if not fit:
                est = skmetal_b200.accelerate(KMeans(n_clusters=w.k, init=init, n_init=1, max_iter=1))
                est.fit(X[:max(w.k, 1000)])
                est._estimator.cluster_centers_ = init.copy()
                t_0 = time.perf_counter()
                est.predict(X)
                return time.perf_counter() - t_0, 1
            if world > 1:
                t_0 = time.perf_counter()
                n_it = _bridge.kmeans_fit_shard(X, init, w.max_iter, 0.0, lo, n_total)[3]
                return time.perf_counter() - t_0, n_it
            est = skmetal_b200.accelerate(KMeans(n_clusters=w.k, init=init, n_init=1, max_iter=w.max_iter, tol=0,
                                                 algorithm="lloyd"))
            t_0 = time.perf_counter()
            est.fit(X)
            return time.perf_counter() - t_0, est.n_iter_

        def e2e_time(X, steps):
            e2e_call(X)  # untimed warm-up of the host-buffer path
            barrier()
            t_sum, it_sum, calls = 0.0, 0, []
            for _ in range(steps):
                t_i, n_i = e2e_call(X)
                t_sum += t_i
                it_sum += n_i
                calls.append(round(t_i * 1e3, 3))
            if dist is not None:
                (t_sum,) = max_over_ranks(dist, [t_sum], device="cuda")
            return n_total * it_sum / t_sum, calls

        e2e_steps = max(1, min(args.steps, 5))
        e2e, e2e_calls = e2e_time(Xs, e2e_steps)
        Xp = torch.empty(Xs.shape, dtype=torch.float32, pin_memory=True).numpy()
        Xp[...] = Xs
        e2e_pinned, e2e_pinned_calls = e2e_time(Xp, e2e_steps)
        del Xp

    hbm, bf16, bf16_sus, src = _peaks()
    rows_here = Xs.shape[0]
    if fit:
        # per Lloyd iteration: X read once (4 n d bytes) and 3 (2 n k d) tensor
        # flops (the split product); the roofline is the slower of the two at
        # the measured peaks (the MMAs are kind::f16, the bf16 burst peak)
        alg_bytes = 4.0 * rows_here * w.d
        flops = 6.0 * rows_here * w.k * w.d
        t_hbm, t_tc = alg_bytes / (hbm * 1e9), flops / (bf16 * 1e12)
        tensor = t_tc > t_hbm
        work, peak, scale, unit_r = (flops, bf16, 1e12, "TFLOP/s") if tensor else (alg_bytes, hbm, 1e9, "GB/s")
        est_avg_s = est_ms / max(1, est_n) / 1e3
        e_achieved = work / est_avg_s / scale if est_avg_s > 0 else None
        if persistent:
            per_launch = work * iters / args.steps  # one launch per fit, all its iterations
            dur_s = ms_loop / 1e3 / args.steps
            achieved = per_launch / dur_s / scale if dur_s > 0 else None
            traffic = _traffic_for("lloyd_loop", w.name, rows_here, iters / args.steps)
            kernel = "lloyd_loop_kernel (persistent: every Lloyd iteration of a fit in one launch)"
            e_timing = "device globaltimer stamps of every iteration (E-step through the grid barrier)"
        else:
            per_launch = work
            achieved = e_achieved
            wide = w.k > 256
            traffic = _traffic_for("estep_wide" if wide else "estep_tc", w.name, rows_here)
            kernel = "estep_wide_kernel (tcgen05 E-step, k > 256)" if wide else "E-step (estep_tc_kernel)"
            e_timing = "CUDA events on the E-step launches of every 10th iteration"
        roofline = {"bound": "tensor" if tensor else "hbm", "achieved": achieved, "peak": peak, "unit": unit_r,
                    "frac": (achieved / peak) if achieved else None, "traffic": traffic, "kernel": kernel,
                    "peak_source": f"{src} bf16 burst" if tensor else src,
                    ("algorithmic_flops_per_launch" if tensor else "algorithmic_bytes_per_launch"): per_launch,
                    "iteration_roofline_us": {"hbm": t_hbm * 1e6, "tensor": t_tc * 1e6},
                    "e_phase": {"achieved": e_achieved, "frac": (e_achieved / peak) if e_achieved else None,
                                "timing": e_timing}}
        if tensor:
            roofline["frac_of_sustained"] = (achieved / bf16_sus) if achieved else None
        if persistent and ms_loop > 0:
            roofline["loop_frac"] = (work * iters / (ms_loop / 1e3)) / scale / peak
    else:
        per_launch = 4.0 * rows_here * (w.d + 1)  # X read once, int32 labels written
        dur_s = ms_loop / 1e3 / args.steps
        achieved = per_launch / dur_s / 1e9 if dur_s > 0 else None
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                    "frac": (achieved / hbm) if achieved else None,
                    "traffic": _traffic_for("assign_predict", w.name, rows_here),
                    "kernel": "predict assignment kernel", "peak_source": src,
                    "algorithmic_bytes_per_launch": per_launch,
                    "timing": "CUDA events around the assignment launch of every step"}
    line = {
        "metric": _metric(wt), "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_dev / args.steps, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded, BASELINE {w.name} recipe); X resident in HBM",
        "config": _config(w, n_total, world, scaling),
        "parallelism": f"rows sharded x{world} ({scaling} scaling: {n_total // world} rows per GPU)",
        "iters_per_step": iters / args.steps,
        "e2e": {"value": e2e, "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "host_memory": "pageable numpy (as a user passes it)",
                "path": ("skmetal_b200.accelerate(KMeans).fit" if fit else "skmetal_b200.accelerate(KMeans).predict")
                if world == 1 or not fit else "skmetal_kmeans_fit_shard (C ABI, per rank)",
                "calls_ms": e2e_calls},
        "e2e_pinned": {"value": e2e_pinned, "unit": unit, "host_memory": "page-locked", "calls_ms": e2e_pinned_calls},
        "gpu_launches": int(launches),
        "ranks_agree": ranks_agree,
        "roofline": roofline,
        "phases": phases,
        "clocks": clk,
        "wall_s": wall,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w, Xs, init)
    ds.close()
    if world > 1:
        if fit:
            _bridge.comm_destroy()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
