"""bench.py's reference arm: the reference's own CPU path for the step (the oracle
port of its torch compositions) timed on the host cores with bounded samples.  It
needs no GPU, so its JSON line is checked here against the driver's contract."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "DiT s/step (40 blocks, 18432 tok)" and d["unit"] == "s/step"
    assert d["higher_is_better"] is False and d["steps"] == 1 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["value"] > 0 and abs(d["ms_per_step"] - d["value"] * 1e3) <= 1e-3 * d["ms_per_step"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1
    assert cb["cpu_model"] and "256 of 18944 tokens" in cb["sample"]
    assert d["config"]["seq_len"] == 18944 and d["config"]["blocks"] == 40
