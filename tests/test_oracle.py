"""The CPU oracle against fixtures produced by the reference's own code (tests/golden/make_golden.py
imports tools/reference/qwen_ref.py and tools/draft/ildraft.py), plus the oracle's tree semantics
against its own causal path."""
import json

import numpy as np
import pytest

from instantllm_b200 import synth
from oracle import accept as A
from oracle import qwen_oracle as Q


@pytest.mark.parametrize("fmt", ["f32", "q4"])
def test_small_model_matches_reference(golden_dir, fmt):
    g = np.load(golden_dir / f"qwen_small_{fmt}.npz")
    w = synth.make_weights(fmt, n_layers=2, vocab=2048, seed=11)
    m = Q.model_from_weights(w)
    prompt = list(g["prompt"])
    cache = Q.KVCache(2, 64)
    pre = Q.forward_causal(m, cache, prompt, 0, all_logits=True)
    assert np.abs(pre - g["prefill_logits"]).max() < 2e-5
    ids, _, steps = Q.greedy(m, prompt, 8, stop_ids=())
    assert ids == g["output_ids"].tolist()
    # steps[0] is the prefill's last row; steps[1+j] the logits after feeding output j
    assert np.abs(steps[1:] - g["decode_logits"][: len(steps) - 1]).max() < 2e-5


def test_full_model_config1_matches_reference(golden_dir):
    """BASELINE config 1 at full size: 24 layers, vocab 151936, fp32, 64-token prompt, 32 tokens."""
    g = json.loads((golden_dir / "qwen_full_f32.json").read_text())
    w = synth.make_weights("f32", n_layers=24, seed=0)
    m = Q.model_from_weights(w)
    ids, _, steps = Q.greedy(m, g["prompt"], 32)
    ref = g["output_ids"] + ([g["stop_token"]] if g["stop_token"] is not None else [])
    assert ids == ref
    for s, top in zip(steps, g["step_top5"]):
        for tid, val in top:
            assert abs(float(s[tid]) - val) < 1e-4


def test_dequant_matches_scalar_restatement():
    """Shaders.swift:120-126 embed_at: q = (i & 1) ? b >> 4 : b & 15; w = s * q + min."""
    rng = np.random.default_rng(0)
    m = synth.make_matrix("q4", 16, 128, rng)
    d = Q.dequant(m)
    for r in range(0, 16, 5):
        for i in range(0, 128, 7):
            b = int(m["codes"][r, i >> 1])
            q = (b >> 4) if (i & 1) else (b & 15)
            s, mn = m["scales"][r, i >> 6].astype(np.float32)
            assert d[r, i] == np.float32(s * np.float32(q)) + mn
    m8 = synth.make_matrix("q8", 16, 128, rng)
    d8 = Q.dequant(m8)
    assert d8[3, 70] == np.float32(m8["scales"][3, 1]) * np.float32(m8["codes"][3, 70])
    # the reference's q8 (quantizeQ8, Convert.swift:254-282): one scale per 32 columns
    m32 = synth.make_matrix("q8g32", 16, 128, rng)
    d32 = Q.dequant(m32)
    assert m32["scales"].shape == (16, 4)
    for r, i in ((3, 70), (15, 31), (0, 32), (9, 127)):
        assert d32[r, i] == np.float32(m32["scales"][r, i // 32]) * np.float32(m32["codes"][r, i])


def test_accept_tree_matches_reference(golden_dir):
    for c in json.loads((golden_dir / "accept_tree.json").read_text()):
        assert A.accept_tree(c["parents"], c["tokens"], c["y"], c["p"]) == c["a"]


def _gpu_tree(parents, tokens):
    n = len(parents) + 1
    depth = [0]
    par = [-1] + [p + 1 for p in parents]
    for i in range(1, n):
        depth.append(depth[par[i]] + 1)
    return {"n": n, "depth": depth, "parent": par, "tok": [0] + list(tokens)}


def test_walk_tree_equals_accept_tree(golden_dir):
    """The GPU-numbered walk (Shaders.swift:311-320) accepts what accept_tree accepts when each
    on-path row's argmax is the next target token."""
    for c in json.loads((golden_dir / "accept_tree.json").read_text()):
        parents, tokens, y, p = c["parents"], c["tokens"], c["y"], c["p"]
        if len(parents) > 15:
            continue
        tree = _gpu_tree(parents, tokens)
        # argmax of a row = target token at its depth if the row is on the matched path
        g = []
        for i in range(tree["n"]):
            d = tree["depth"][i]
            g.append(y[p + d] if p + d < len(y) else -1)
        path = A.walk_tree(tree, g)
        assert len(path) == c["a"]


def test_chain_acceptance():
    assert A.accept_chain([5, 6, 7], [5, 6, 9], 0) == 2
    assert A.accept_chain([], [1], 0) == 0
    tree = synth.chain_tree([5, 6, 7])
    assert A.walk_tree(tree, [5, 6, 9, 1]) == [1, 2]


def test_commit_moves_and_stop():
    tree = {"n": 5, "depth": [0, 1, 1, 2, 2], "parent": [-1, 0, 0, 2, 2], "tok": [0, 9, 4, 8, 5]}
    g = [4, 0, 5, 0, 7]
    r = A.commit(tree, g, pos=100, step=3, maxsteps=50)
    assert r["path"] == [2, 4] and r["tokens"] == [4, 5, 7] and r["pos"] == 103
    assert r["moves"] == [(102, 101), (104, 102)]
    r = A.commit(tree, g, pos=100, step=3, maxsteps=5)
    assert r["tokens"] == [4, 5] and r["done"]
    r = A.commit(tree, [4, 0, 151645, 0, 7], pos=100, step=0, maxsteps=50)
    assert r["tokens"] == [4, 151645] and r["done"]


def test_tree_pass_equals_sequential_oracle():
    """A tree row's logits equal those of the same path decoded one token at a time
    (the reference's speculation-is-exact criterion, README.md:90-93), up to BLAS rounding."""
    w = synth.make_weights("f32", n_layers=2, vocab=1024, seed=3)
    m = Q.model_from_weights(w)
    prompt = [5, 9, 300, 17, 800, 2]
    cache = Q.KVCache(2, 64)
    lg = Q.forward_causal(m, cache, prompt, 0)
    root = int(np.argmax(lg))
    tree = {"n": 6, "depth": [0, 1, 1, 2, 3, 2], "parent": [-1, 0, 0, 2, 3, 1], "tok": [0, 11, 12, 13, 14, 15]}
    tl = Q.tree_pass(m, cache.copy(), len(prompt), root, tree)
    for row, path_toks in [(3, [12, 13]), (4, [12, 13, 14]), (5, [11, 15]), (0, [])]:
        c = cache.copy()
        seq = [root] + path_toks
        sl = Q.forward_causal(m, c, seq, len(prompt), all_logits=True)[-1]
        assert np.abs(sl - tl[row]).max() < 1e-5
