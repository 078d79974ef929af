"""bench.py's command-line contract on CPU: the reference arm answers with an
``unavailable`` JSON line for configurations whose reference path is not
run here, and the flags the driver passes parse."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(*args):
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, timeout=300,
                       cwd=ROOT)
    return p.returncode, p.stdout.strip().splitlines()


def test_reference_arm_reports_unavailable_with_a_reason():
    rc, out = _run("--impl", "reference", "--gpus", "1", "--steps", "2", "--warmup", "3")
    assert rc == 0 and len(out) == 1
    line = json.loads(out[0])
    assert line["impl"] == "reference" and line["unavailable"]


def test_flags_parse():
    rc, out = _run("--help")
    assert rc == 0
    text = "\n".join(out)
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--config", "--exposed-comm"):
        assert flag in text
