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
@pytest.mark.parametrize("workload,metric", [("c4", "decoded audio-sec/sec"), ("c2", "decoded audio-sec/sec"),
                                             ("e1", "encoded audio-sec/sec")])
def test_reference_arm_prints_one_json_line(workload, metric):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                        workload, "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == metric and d["unit"] == "audio-s/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    # the driver divides the two arms' values only when metric, steps and warmup match
    assert d["steps"] == 2 and d["warmup"] == 3


def test_both_arms_share_one_metric_string_per_family():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    src = open(os.path.join(ROOT, "bench.py")).read()
    # every "metric" key of either arm is one of the two module constants
    assert src.count('"metric": METRIC_DECODE') == 2 and src.count('"metric": METRIC_ENCODE') == 2
    assert '"metric": "' not in src
    assert b.DEFAULT_WORKLOAD == "c4" and b.WORKLOADS["c4"][1] == 256
