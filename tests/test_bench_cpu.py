"""bench.py's reference arm (the reference's own CPU forward from the offline
install in baseline/_ref, or the CPU oracle port of it when the reference is
not installed, timed on this host's cores) prints one JSON line with the
benchmark contract's keys; it needs no GPU."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "3", "--cpu-seconds", "1"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [x for x in out.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, out.stdout
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["unit"] == "decisions/s" and line["higher_is_better"] is True
    assert 1 <= line["steps"] <= 2 and line["warmup"] >= 1
    assert line["value"] > 0 and abs(line["e2e"]["value"] - line["value"]) < 1e-9
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    base = line["cpu_baseline"]
    sys.path.insert(0, str(ROOT))
    from baseline import laya_net
    want = "reference" if laya_net.reference_src() is not None else "port"
    assert base["kind"] == want and base["cores"] >= 1 and base["value"] == line["value"]
    assert line["config"]["workload"].startswith("C1")


def test_fp32_restatement_is_labelled_and_bounded():
    """BASELINE config 0's "CPU fp32" figure, reported inside cpu_baseline as a
    labelled restatement (the oracle with fp32 Linears), within its time bound."""
    import time
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "laya-inference-engine_b200"))
    import bench
    from laya_b200.config import TINY
    from laya_b200.weights import seeded_weights
    t0 = time.perf_counter()
    out = bench.cpu_fp32_restatement(TINY, 0.5, seeded_weights(TINY, seed=0))
    assert time.perf_counter() - t0 < 30
    assert out["kind"] == "port" and out["value"] > 0 and out["cores"] >= 1
    assert "restatement" in out["sample"] and "fp32" in out["sample"]
