"""bench.py --impl reference: the reference's CPU path (the oracle's C port of
kernel/rans.py:101-123 + kernel/bench.py:54 on one full layer of the config's
shapes, encoded by the oracle's C restatement of the reference encoder) must
never load this repository's library or torch, and must print the same config
dict as the repository's own arm."""
import json
import os
import subprocess
import sys

from conftest import ROOT

CODE = r"""
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--config", "2", "--steps", "1", "--warmup", "1"]
sys.path.insert(0, ROOT)
import bench
bench.main()
loaded = sorted(m for m in sys.modules if m in ("rans_b200", "rans_dist", "rans_model", "torch"))
print("LOADED " + json.dumps(loaded))
"""


def test_reference_arm_uses_only_the_oracle():
    out = subprocess.run([sys.executable, "-c", f"ROOT = {ROOT!r}\n" + CODE], capture_output=True, text=True,
                         cwd=ROOT, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.splitlines()
    line = json.loads([l for l in lines if l.startswith("{")][-1])
    loaded = json.loads([l for l in lines if l.startswith("LOADED ")][-1][len("LOADED "):])
    assert loaded == [], loaded
    assert line["impl"] == "reference" and line["value"] > 0
    import bench
    shapes, nl, _, _, _ = bench.CONFIGS["2"]
    weights = nl * sum(r * c for _, r, c in shapes)
    assert line["config"] == bench.config_dict("2", nl, 8, 1, weights)
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
