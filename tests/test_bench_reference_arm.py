"""bench.py's reference arm (the reference's own CPU code from oracle/_ref)
prints one JSON line with the fields the driver reads, for a decode and the
encode workload; on CPU only (it never touches a GPU)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "liboracle_ref.so")


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="the reference library is not built here")
@pytest.mark.parametrize("workload,metric", [("c2", "decoded audio-sec/sec (emitted)"),
                                             ("e1", "encoded audio-sec/sec")])
def test_reference_arm_prints_one_json_line(workload, metric):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                        workload, "--steps", "2"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == metric and d["unit"] == "audio-s/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
