"""bench.py's reference arm on the CPU: the JSON line the driver parses, with
a reduced sample (one row, two layers) so it runs in seconds."""
import json
import subprocess
import sys

from conftest import REPO


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run(
        [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "2",
         "--warmup", "1", "--cpu-seqs", "1", "--layers", "2"],
        capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "paged decode-attn HBM GB/s"
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 2, 1)
    assert d["ms_per_step"] > 0 and d["vs_baseline"] is None
    assert d["config"]["layers"] == 2 and "2 layers" in d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == "GB/s"
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == "GB/s"
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
