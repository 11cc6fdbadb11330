"""Host-side logic: algorithmic byte counts, tree buffers, seeded trees and prompts."""
import numpy as np
import pytest

from instantllm_b200 import synth
from oracle import accept as A


def test_weight_bytes_match_reference_figures():
    # README.md:30 "278 MB" per q4 pass; exact figure derived from the formats
    assert synth.weight_bytes("q4") == 278_139_392
    assert synth.weight_bytes("q8") == 509_683_712
    assert synth.weight_bytes("f16") == 988_208_640


def test_tree_buffer_layout():
    tree = {"n": 4, "depth": [0, 1, 1, 2], "parent": [-1, 0, 0, 2], "tok": [0, 7, 8, 9]}
    b = synth.tree_to_buffer(tree)
    assert b.shape == (65,) and b.dtype == np.int32
    assert b[0] == 4
    assert list(b[1:5]) == [0, 1, 1, 2]
    assert list(b[17:21]) == [-1, 0, 0, 2]
    assert list(b[33:37]) == [0, 7, 8, 9]
    assert list(b[49:53]) == [0b1, 0b11, 0b101, 0b1101]  # ancestor masks incl. self


def test_seeded_tree_shape_and_acceptance_rate():
    rng = np.random.default_rng(1)
    acc = []
    for _ in range(400):
        y = list(rng.integers(0, 1000, size=9))
        t = synth.seeded_tree(rng, y, n=16)
        assert t["n"] == 16 and t["depth"][0] == 0
        for i in range(1, 16):
            assert 0 <= t["parent"][i] < i
            assert t["depth"][i] == t["depth"][t["parent"][i]] + 1 <= 8
        parents, tokens = A.to_python_numbering(t)
        acc.append(A.accept_tree(parents, tokens, y, 0))
    # p = 0.6 matching drafts: the root alone has ~6 children, so the first draft is accepted
    # almost always and the mean accepted path is around 2
    assert 1.0 < np.mean(acc) < 4.0


def test_prompts_are_seeded_and_in_range():
    a, b = synth.make_prompt(256, 3), synth.make_prompt(256, 3)
    assert (a == b).all() and a.min() >= 0 and a.max() < synth.PROMPT_VOCAB
    assert not (a == synth.make_prompt(256, 4)).all()


def test_synthetic_distributions():
    rng = np.random.default_rng(0)
    q4 = synth.make_matrix("q4", 64, 128, rng)
    s, mn = q4["scales"][..., 0].astype(np.float32), q4["scales"][..., 1].astype(np.float32)
    assert (s >= 0).all() and np.allclose(mn, -7.5 * s, rtol=1e-3, atol=1e-7)
    q8 = synth.make_matrix("q8", 64, 128, rng)
    assert q8["codes"].min() >= -127 and q8["codes"].max() <= 127


def test_adaptive_pass_shape_follows_the_reference_rule():
    """PassShape mirrors Engine.nextPassShape (Engine.swift:887-898): the configured tree until at
    least 3 samples of (passes, accepted) span 2 or more passes, then the tree while the accepted
    drafts per pass over the oldest of the last 4 samples reach adaptHi (1.5), else an 8-row chain
    (7 drafts, one child per expansion)."""
    from instantllm_b200.engine import PassShape

    TREE, CHAIN = (15, 8), (7, 1)
    s = PassShape()
    assert s.next(1, 0) == TREE and s.next(1, 0) == TREE  # the same sample is recorded once
    assert s.hist == [(1, 0)]
    assert s.next(2, 0) == TREE                            # 2 samples
    assert s.next(3, 0) == CHAIN                           # 3 samples over 2 passes, rate 0
    assert s.next(4, 6) == TREE                            # (6 - 0) / (4 - 1) = 2.0
    assert s.next(5, 6) == TREE                            # window (2, 0): 6 / 3 = 2.0
    assert s.next(6, 6) == TREE                            # window (3, 0): 6 / 3 = 2.0
    assert s.next(7, 6) == CHAIN                           # window (4, 6): 0 / 3
    s = PassShape()
    for p, a in [(1, 0), (2, 2), (3, 3)]:
        s.next(p, a)
    assert s.next(4, 4) == CHAIN                           # window (1, 0): 4 / 3 = 1.33 < 1.5
    assert s.next(5, 7) == TREE                            # window (2, 2): 5 / 3 = 1.67
    s = PassShape(adaptive=False)
    assert all(s.next(p, 0) == TREE for p in range(1, 10))
    s = PassShape(tree_b=9, chain_rows=4, adapt_hi=0.5)
    assert [s.next(p, 0) for p in (1, 2, 3)] == [(9, 8), (9, 8), (3, 1)]
    s.reset()
    assert s.hist == [] and s.next(7, 0) == (9, 8)


def test_config5_summary_takes_the_max_over_ranks_in_each_mode():
    import bench

    # per mode of bench.C5_MODES (1, 2, 4): [ms, tokens, request passes, launches, ok, GB/s, differ]
    r0 = [100.0, 500.0, 200.0, 200.0, 1.0, 300.0, 0.0] + [70.0, 501.0, 200.0, 110.0, 1.0, 430.0, 1.0] \
        + [50.0, 500.0, 200.0, 60.0, 1.0, 600.0, 0.0]
    r1 = [120.0, 520.0, 210.0, 210.0, 1.0, 290.0, 0.0] + [80.0, 520.0, 210.0, 115.0, 1.0, 435.0, 0.0] \
        + [55.0, 520.0, 210.0, 62.0, 1.0, 610.0, 2.0]
    s = bench.config5_summary([r0, r1], 16)
    assert bench.C5_MODES == (1, 2, 4) and bench.C5_HEADLINE == 4
    assert s["value"] == 1020 / 0.055 and s["requests_per_launch"] == 4 and s["tokens"] == 1020
    m = s["modes"]
    assert m["1"]["value"] == 1020 / 0.120 and m["1"]["launches"] == 410
    assert m["2"]["value"] == 1021 / 0.080 and m["2"]["truth_differs_from_whole_gpu"] == 1
    assert m["4"]["ms_per_rank"] == [50.0, 55.0] and m["4"]["truth_differs_from_whole_gpu"] == 2
    assert s["tree_equals_sequential"]
    r1[4 + 7] = 0.0  # one rank's two-per-launch run failed its check
    assert not bench.config5_summary([r0, r1], 16)["tree_equals_sequential"]


def test_trace_timeline_reads_the_stamp_layout():
    from instantllm_b200 import trace as T

    G = 4
    buf = np.zeros(T.TRACE_LEN, dtype=np.int64)

    def put(ev, cta, ns):
        buf[T.TRACE_BASE + 256 * ev + cta] = ns

    for c in range(G):
        put(56, c, 10_000 + 100 * c)                      # layer start
        put(T.stage_event(0, 0), c, 11_000 + 100 * c)     # QKV entry
        put(T.stage_event(4, 0), c, 100_000 + 500 * c)    # lm_head entry
        for w in range(16):
            put(T.lm_job_event(w, 0, 0), c, 101_000)
            put(T.lm_job_event(w, 0, 1), c, 102_000)
            put(T.lm_job_event(w, 0, 2), c, 106_000)
    put(48, 2, 30_000)
    put(49, 2, 31_000)
    t = T.timeline(buf, G)
    assert t["layer"]["QKV"]["entry"] == pytest.approx((1.15, 1.3))  # median, max over the stamping CTAs
    assert "inputs" not in t["layer"]["QKV"]                # no CTA stamped it
    assert t["layer"]["barriers"][0] == (20.0, 21.0)
    (r,) = t["lm_head"]["rounds"]
    assert r["jobs"] == 16 * G and r["wait_mean"] == 1.0 and r["compute_mean"] == 4.0 and r["done_max"] == 6.0
    t["pass_us"] = [580.0]
    text = T.report(t)
    assert "round 0: 64 jobs" in text and "grid barrier 0: last arrival 20.00" in text


def test_batched_loop_rejects_bad_arguments_before_touching_a_device():
    from types import SimpleNamespace

    from instantllm_b200.engine import VerifyEngine

    dev = SimpleNamespace()
    e = [SimpleNamespace(device=dev) for _ in range(5)]
    d = [SimpleNamespace(device=dev) for _ in range(5)]
    p = [[1, 2, 3]] * 5
    gen = VerifyEngine.generate_drafted_batch
    with pytest.raises(ValueError):
        gen(e[:5], p[:5], 8, d[:5])                 # five requests: at most four shares
    with pytest.raises(ValueError):
        gen(e[:3], p[:3], 8, d[:3], shares=2)       # more requests than shares
    with pytest.raises(ValueError):
        gen(e[:2], p[:1], 8, d[:2])                 # one prompt per engine
    with pytest.raises(ValueError):
        gen([e[0], e[0]], p[:2], 8, d[:2])          # the same engine twice
    with pytest.raises(ValueError):
        gen(e[:2], p[:2], 8, [d[0], SimpleNamespace(device=object())])  # drafters on another device
    with pytest.raises(ValueError):
        gen(e[:2], p[:2], 8, d[:2], depth=-1)


def test_bench_parses_every_workload():
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, str(root / "bench.py"), "--help"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    for w in ("config2", "batch2", "batch3", "batch4", "config3", "config4", "config5", "sketch_head", "decode_loop"):
        assert w in r.stdout
