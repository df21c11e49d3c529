"""bench.py pieces that need no GPU: the reference arm's JSON line (the CPU
restatement of Prana's decode on a tiny seeded model), the per-step launch
count it claims, and the seeded KV rows both arms start from."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402
from prana_b200 import synth  # noqa: E402


def test_reference_arm_line(tmp_path):
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "stories15m_q8_0",
           "--ctx", "64", "--steps", "2", "--warmup", "3", "--model-dir", str(tmp_path)]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": bench.UNIT, "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"] == "stories15m_q8_0"


def test_launches_per_step_counts():
    spec = synth.PRESETS["llama3_8b_q4_0"]
    # embed + 32 x (Q|K|V, attention, wo, gate|up, down) + LM head + advance
    assert bench.launches_per_step(spec) == 1 + 32 * 5 + 1 + 1
    # tensor parallel: + the argmax merge; with the peer exchange + 2 exchanges per layer + the argmax gather
    assert bench.launches_per_step(spec, 2) == 164
    assert bench.launches_per_step(spec, 2, True) == 164 + 2 * 32 + 1


def test_seeded_kv_rows_deterministic():
    a = bench.seeded_kv_rows(3, True, 16, 64)
    b = bench.seeded_kv_rows(3, True, 16, 64)
    c = bench.seeded_kv_rows(3, False, 16, 64)
    assert a.dtype == np.uint16 and a.shape == (16, 64)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
