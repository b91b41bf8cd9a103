"""bench.py's reference arm runs on the CPU and prints the contract's line."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT


@pytest.mark.parametrize("config", ["mlp-8x128x128x64", "lm-t64-d64-f64-l2-h4"])
def test_reference_arm_prints_one_contract_line(config):
    from oracle.oracle import reference_available
    if not reference_available():
        pytest.skip("reference CPU build (oracle/_ref) not present")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", config,
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["value"] == line["value"] and line["e2e"]["h2d_bytes_per_step"] == 0
    # the reference arm never loads the product library
    assert "libhexatrain_b200" not in r.stderr
