"""The trace build (instantllm_b200.trace): one traced config-2 pass in a fresh process, whose
stamps come back in stage order."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_trace_build_stamps_the_stages_in_order():
    code = ("import json; from instantllm_b200 import trace; "
            "t = trace.run(layers=6, passes=2); print(json.dumps(t))")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=900,
                       env=dict(os.environ, PYTHONPATH=str(ROOT)))
    assert r.returncode == 0, r.stderr[-2000:]
    t = json.loads(r.stdout.strip().splitlines()[-1])
    L = t["layer"]
    # within layer 5: QKV epilogue, attention combine, O epilogue, gate/up epilogue, the barrier and
    # the down epilogue follow one another (medians over each stage's CTAs)
    seq = [L["QKV"]["epilogue"][0], L["attention"]["combined"][0], L["O"]["epilogue"][0],
           L["gate/up"]["epilogue"][0], L["barriers"]["0"][1], L["down"]["epilogue"][0]]
    assert all(a < b for a, b in zip(seq, seq[1:])), seq
    rounds = t["lm_head"]["rounds"]
    assert rounds and all(r["compute_mean"] > 0 and r["wait_mean"] >= 0 for r in rounds)
    assert sum(r["jobs"] for r in rounds) == 151936 // 16  # every row-block of the vocabulary once
    assert all(x > 0 for x in t["pass_us"])
