"""bench.py's output contract, checked where it can run without a GPU: the
reference arm (the reference's PyTorch layer on the host cores) prints one
JSON line with the keys the driver reads."""

import json
import subprocess
import sys

from tests.conftest import ROOT


def _run(*args):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                       timeout=600, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_json_line():
    d = _run("--impl", "reference", "--config", "cfg1", "--steps", "2", "--warmup", "1")
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["warmup"] >= 3                       # the contract's minimum
    assert d["value"] > 0 and d["unit"] == "tokens/s"
    assert d["config"]["workload"] == "cfg1"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_cfg5_times_the_streamed_formulation():
    """cfg5: the reference layer itself is infeasible ([B,H,S,S] scores), so
    the arm times the reference's streamed formulation and says so."""
    d = _run("--impl", "reference", "--config", "cfg5", "--steps", "1", "--warmup", "1")
    assert d["impl"] == "reference" and d["value"] > 0
    assert "infeasible" in d["reference_layer"]
    assert "reference_chunked" in d["cpu_baseline"]["sample"]
    assert d["config"]["workload"] == "cfg5"


def test_default_workload_is_cfg5():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m.DEFAULT_CONFIG == "cfg5"
    assert m.shard_pieces(4, 100000, 1024) == 16
    assert m.shard_pieces(1250, 128, 128) == 4
