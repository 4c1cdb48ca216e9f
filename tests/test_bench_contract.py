"""bench.py's reference arm runs on the host (the reference's own torch Viterbi from baseline/_ref when installed, else
the C restatement of it, all host threads) and prints one JSON line with the keys the driver reads; checked on CPU with
one timed step.  A warm-up below 3 steps is refused, not silently raised."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_json_line():
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3 and d["value"] > 0
    assert d["metric"] == d["unit"] == d["e2e"]["unit"] and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert "workload" in d["config"]


def test_short_warmup_refused():
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert p.returncode != 0 and "--warmup must be at least 3" in p.stderr


def test_cpu_baseline_names_reference_and_port():
    """cpu_baseline: the reference's own torch viterbi_ub when its install is present (kind "reference"), with the
    oracle's C port timed beside it as a second, labelled number; the port alone otherwise."""
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle.refroot import reference_root
    cb = bench.cpu_baseline_sample(1.0, port_seconds=1.0)
    assert cb["value"] > 0 and cb["cores"] >= 1 and cb["unit"] == bench.METRIC
    if reference_root() is not None:
        assert cb["kind"] == "reference" and "viterbi_ub" in cb["sample"]
        assert cb["port"]["kind"] == "port" and cb["port"]["value"] > 0 and "tcq_oracle.c" in cb["port"]["sample"]
    else:
        assert cb["kind"] == "port" and "port" not in cb
