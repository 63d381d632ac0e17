"""The benchmark's reference arm on the CPU: ``bench.py --impl reference``
prints one JSON line with the driver's keys (the reference's CPU path, a
bounded sample), and the argument parser knows every mode."""
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


ARGS = ["--impl", "reference", "--steps", "1", "--warmup", "0", "--layers", "2", "--ctx", "32",
        "--nodes", "8", "--depth", "3", "--branch", "2"]
# Runs the reference arm in a fresh interpreter, then lists every module of
# this package that the run imported (there must be none).
WRAPPER = """
import runpy, sys
sys.argv = ["bench.py"] + sys.argv[1:]
runpy.run_path("bench.py", run_name="__main__")
print("PACKAGE_MODULES", sorted(m for m in sys.modules if m.split(".")[0] == "specfit_b200"))
"""


def test_reference_arm_prints_the_contract_line():
    cmd = [sys.executable, "-c", WRAPPER, *ARGS]
    res = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    loaded = [l for l in res.stdout.splitlines() if l.startswith("PACKAGE_MODULES")]
    assert loaded == ["PACKAGE_MODULES []"], loaded
    line = [l for l in res.stdout.splitlines() if l.startswith("{")][-1]
    out = json.loads(line)
    sys.path.insert(0, str(REPO))
    import bench

    assert out["config"] == bench.headline_config(bench.parse_args(ARGS))
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


def test_workload_tree_and_config_match_the_package():
    """The bench's package-free tree and config equal the package's."""
    sys.path.insert(0, str(REPO))
    import bench
    from specfit_b200 import synthetic
    from specfit_b200.runtime.qwen3_verifier import qwen3_moe_config

    for nodes, depth, branch, seed in ((64, 6, 4, 2), (128, 8, 4, 2), (8, 3, 2, 5)):
        assert bench.workload_tree(nodes, depth, branch, seed, 151936) == synthetic.random_tree(
            nodes, max_depth=depth, max_branch=branch, seed=seed, vocab=151936)
    mine, theirs = bench.reference_config(48).to_dict(), qwen3_moe_config(48).to_dict()
    for d in (mine, theirs):
        d.pop("_attn_implementation_internal", None)
    assert mine == theirs
    assert bench.reference_model_bytes(48) / 1e9 > 60
