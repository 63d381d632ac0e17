"""The benchmark's reference arm on the CPU: ``bench.py --impl reference``
prints one JSON line with the driver's keys (the reference's CPU path, a
bounded sample), and the argument parser knows every mode."""
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_the_contract_line():
    cmd = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
           "--ctx", "32", "--nodes", "8", "--depth", "3", "--branch", "2"]
    res = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    line = [l for l in res.stdout.splitlines() if l.startswith("{")][-1]
    out = json.loads(line)
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in out, key
    assert out["impl"] == "reference" and out["n_gpus"] == 1 and out["steps"] == 1
    assert out["value"] > 0 and out["higher_is_better"] is True
    assert "workload" in out["config"]
    cb = out["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == out["value"] and cb["sample"]
    assert out["e2e"] == {"value": out["value"], "unit": out["unit"], "h2d_bytes_per_step": 0,
                          "d2h_bytes_per_step": 0}


def test_parser_accepts_every_mode():
    sys.path.insert(0, str(REPO))
    import bench

    for mode in ("auto", "verify", "ep", "decode", "block", "graph", "sweep", "kernels"):
        args = bench.parse_args(["--mode", mode])
        assert args.mode == mode and args.gpus == 1 and args.warmup >= 3
    args = bench.parse_args(["--mode", "kernels", "--kernel", "router,combine", "--fused-gather"])
    assert args.kernel == "router,combine" and args.fused_gather
