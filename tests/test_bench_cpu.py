"""The benchmark's reference arm (`bench.py --impl reference`: the reference's CPU path on the host cores) runs here
and prints the one JSON line of the bench contract, with the keys the driver reads. CPU only."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_the_contract_line():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup",
                           "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 3
    assert line["metric"] and line["config"]["workload"] and line["vs_baseline"] is None
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"] and cpu["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # each step is a bounded sample (one layer) that the line names, so steps x ms_per_step is the time it ran
    assert line["config"]["sample_layers_per_step"] == 1 and "block scales" in line["config"]["format"]
    assert abs(line["value"] - 16 / (48 * line["ms_per_step"] * 1e-3)) <= 1e-6 * line["value"]
