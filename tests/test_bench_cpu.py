"""bench.py's reference arm (the CPU oracle timed on the host) keeps the
one-line JSON contract the measurement driver parses; it runs here without a
GPU on the small fp32 configuration."""

import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _run(*args):
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_json_line():
    d = _run("--impl", "reference", "--config", "c1_fp32_toy", "--steps", "2", "--warmup", "3")
    assert d["impl"] == "reference"
    assert d["metric"] == "moe_ffn_block tokens/s" and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert d["config"]["workload"] == "c1_fp32_toy"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_warmup_floor():
    """W >= 3 warm-up steps whatever is asked."""
    d = _run("--impl", "reference", "--config", "c1_fp32_toy", "--steps", "1", "--warmup", "0")
    assert d["warmup"] >= 3
