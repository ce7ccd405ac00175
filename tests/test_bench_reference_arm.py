"""`bench.py --impl reference` on the CPU: the reference build times its own
conv + BN + ReLU on the full workload and prints one JSON line with the
benchmark's metric, unit and config, a cpu_baseline describing the run and an
e2e object without host-device bytes. Skipped where the reference build
(oracle/_ref/libnpl_ref.so) is absent."""
import json
import subprocess
import sys

import pytest

import support as S


def test_reference_arm_json_line():
    if not (S.REPO / "oracle" / "_ref" / "libnpl_ref.so").exists():
        pytest.skip("reference build absent")
    out = subprocess.run([sys.executable, str(S.REPO / "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "3"], capture_output=True, text=True,
                         timeout=300, cwd=S.REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and "unavailable" not in d
    assert d["metric"].startswith("fused conv2d+BN+ReLU TFLOP/s")
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["value"] > 0
    assert d["config"]["workload"].startswith("npl_conv2d_bn_activation")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
