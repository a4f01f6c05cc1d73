"""bench.py's reference arm on the CPU (`--impl reference`: the reference's own imi_seoul from oracle/_ref on this
host's cores) prints the same JSON line as the GPU arm, and the workloads' synthetic inputs are the ones the
configurations name."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def ref_built() -> bool:
    import oracle
    return oracle.reference_available()


@pytest.mark.skipif(not ref_built(), reason="oracle/_ref is not built")
def test_reference_arm_prefill_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "prefill",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "positions/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "positions/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"].startswith("configs[2]") and line["steps"] == 1 and line["warmup"] == 3


def test_workload_inputs():
    import numpy as np
    import bench
    a, b = bench.multi_contexts(0), bench.multi_contexts(1)
    assert len(a) == bench.MULTI_N == 64 and a == bench.multi_contexts(0) and a != b
    assert all(256 <= x <= 2048 for x in a + b)
    vecs, ids = bench.prefill_inputs(64, 1000)
    assert vecs.shape == (400, 64) and vecs.dtype == np.float32 and abs(float(vecs.std()) - 0.5) < 0.02
    assert len(ids) == 16 and all(0 <= int(t) < 1000 for t in ids)


def test_default_steps_per_workload(monkeypatch):
    import bench
    for wl, k in (("ride2", 128), ("b1", 128), ("prefill", 5), ("multi64", 256)):
        monkeypatch.setattr(sys, "argv", ["bench.py", "--workload", wl])
        assert bench.parse().steps == k
    monkeypatch.setattr(sys, "argv", ["bench.py", "--workload", "multi64", "--steps", "7"])
    assert bench.parse().steps == 7
