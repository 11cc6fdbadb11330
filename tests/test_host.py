"""Host-side logic: algorithmic byte counts, tree buffers, seeded trees and prompts."""
import numpy as np

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
