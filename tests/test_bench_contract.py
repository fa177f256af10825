"""The JSON line contract of bench.py's reference arm, on the CPU at small
sizes: one line with the metric, unit, timing, config and the cpu_baseline /
e2e objects the driver reads; ranks other than 0 print nothing."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                       capture_output=True, text=True, env=e, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stdout.splitlines() if l.startswith("{")]


def check_line(line, workload_prefix):
    d = json.loads(line)
    assert d["impl"] == "reference"
    assert d["metric"] == "queries_per_sec" and d["unit"] == "queries/s"
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["p50_us"] > 0
    assert d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["vs_baseline"] is None
    assert d["config"]["workload"].startswith(workload_prefix)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    return d


def test_reference_arm_flat_line():
    lines = run_bench(["--impl", "reference", "--n", "4096", "--dim", "64", "--steps", "2",
                       "--warmup", "1"])
    assert len(lines) == 1
    d = check_line(lines[0], "exact_flat_4096x64_cosine_top10_nq1")
    assert d["steps"] == 2 and d["warmup"] == 1


def test_reference_arm_batch_takes_the_bounded_route():
    """Batches over n >= 16384 take the reference's CPU batch route
    (BoundedExactScan per query, queries in parallel)."""
    lines = run_bench(["--impl", "reference", "--n", "20000", "--dim", "32", "--nq", "8",
                       "--steps", "1", "--warmup", "0"])
    assert len(lines) == 1
    d = check_line(lines[0], "exact_flat_20000x32_cosine_top10_nq8")
    assert "BoundedExactScan" in d["cpu_baseline"]["sample"]


@pytest.mark.parametrize("workload,extra", [
    ("ivf", []),
    ("ivfpq", ["--pq-m", "8"]),
])
def test_reference_arm_index_lines(workload, extra):
    lines = run_bench(["--impl", "reference", "--workload", workload, "--n", "5000", "--dim",
                       "32", "--nlist", "16", "--components", "16", "--nq", "4", "--steps", "1",
                       "--warmup", "0", *extra])
    assert len(lines) == 1
    check_line(lines[0], "ivf_flat_" if workload == "ivf" else "ivfpq_")


def test_reference_arm_other_ranks_print_nothing():
    assert run_bench(["--impl", "reference", "--n", "4096", "--dim", "64", "--steps", "1",
                      "--warmup", "0"], env={"RANK": "1"}) == []
