"""bench.py's roofline inputs (CPU): the DRAM traffic it reports for each
workload's dominant kernel comes from the committed ncu summaries under
profiles/, scaled to the bench's rows and iterations. Each summary must parse,
and the traffic cannot fall much below the kernel's algorithmic bytes."""

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# kernel, config, rows, Lloyd iterations per launch, algorithmic bytes per launch
CASES = [
    ("lloyd_loop", "c2", 500_000, 100, 4 * 500_000 * 100 * 100),
    ("lloyd_loop", "c4", 50_000_000, 20, 4 * 50_000_000 * 64 * 20),
    ("estep_wide", "c3", 2_000_000, 1, 4 * 2_000_000 * 128),
    ("assign_predict", "c5", 400_000_000, 1, 400_000_000 * (4 * 8 + 4)),
]


@pytest.mark.parametrize("kernel,config,rows,iters,algo", CASES)
def test_profile_traffic_parses(kernel, config, rows, iters, algo):
    t = _bench()._traffic_for(kernel, config, rows, iters)
    assert t is not None, f"profiles/{kernel}_{config}.md gives no traffic"
    assert 0.95 * algo <= t <= 2.0 * algo, (t, algo)
