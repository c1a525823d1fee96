"""bench.py's contract on the host: the reference arm (the reference's own CPU code on the host
cores) prints one JSON line with the fields the driver reads, for an attention and a projection
workload, and the workload table names every configuration."""
from __future__ import annotations

import json
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]


def run_reference(workload):
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload,
                           "--also", "none", "--steps", "1", "--warmup", "1"],
                          capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, proc.stdout
    return json.loads(lines[0])


def check_line(d, unit):
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_projection_workloads():
    check_line(run_reference("proj_decode"), "GB/s")
    d = run_reference("proj_prefill")
    check_line(d, "TFLOP/s")
    assert d["config"]["tokens"] == 4096 and d["config"]["activations"] == "bf16"


def test_reference_arm_decode_workload():
    d = run_reference("c1_decode")
    check_line(d, "GB/s")
    assert d["config"]["workload"] == "c1_decode"


def test_default_workloads_cover_every_configuration():
    sys.path.insert(0, str(ROOT))
    import bench
    from apex_b200.configs import CONFIGS
    assert set((bench.PRIMARY,) + tuple(bench.ALSO)) == set(CONFIGS)
    for cfg in CONFIGS.values():
        metric, unit, _ = bench.metric_of(cfg)
        assert unit in ("GB/s", "TFLOP/s") and metric
        assert bench.config_of(cfg)["workload"] == cfg.name
