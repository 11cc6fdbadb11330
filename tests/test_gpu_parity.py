"""Parity of the CUDA verification pass with the CPU oracle, through the C ABI (VerifyEngine).

Criteria:
  * committed tokens of tree / chain passes are bit-identical to the same kernels run one token at a
    time (1-row passes),
  * accept/commit is bit-exact against the reference's acceptance logic (oracle/accept.py, pinned
    to tools/draft/ildraft.py:accept_tree by tests/test_oracle.py),
  * logits agree with the fp32 CPU oracle within LOGIT_TOL (fp16 activations, fp32 accumulation:
    the reference's own guidance is max|d| ~0.03-0.04 with --max-abs-tol 0.1,
    tools/reference/README.md:270-272), with argmax agreement reported.
"""
import numpy as np
import pytest
import torch

from instantllm_b200 import synth
from oracle import accept as A
from oracle import qwen_oracle as Q

pytestmark = pytest.mark.gpu

LOGIT_TOL = 0.05   # max |gpu - fp32 oracle| on logits of scale ~2-3
VOCAB_SMALL = 4096


def _engine(w, **kw):
    from instantllm_b200.engine import VerifyEngine
    return VerifyEngine(w, **kw)


@pytest.fixture(scope="module", params=["q4", "q8", "q8g32", "f16"])
def small(request):
    fmt = request.param
    w = synth.make_weights(fmt, n_layers=2, vocab=VOCAB_SMALL, seed=21)
    eng = _engine(w, max_ctx=512, max_steps=128)
    yield fmt, w, Q.model_from_weights(w), eng
    eng.close()


def test_prefill_and_tree_logits_match_oracle(small):
    fmt, w, m, eng = small
    prompt = (synth.make_prompt(37, seed=8) % VOCAB_SMALL).tolist()
    eng.begin(0, 32)
    eng.prefill(prompt)
    gl = eng.logits().cpu().numpy()
    cache = Q.KVCache(2, 512)
    ref = Q.forward_causal(m, cache, prompt, 0, all_logits=True)
    last = len(prompt) - 32  # rows of the last 16-row chunk
    d = np.abs(gl[:last] - ref[32:]).max()
    assert d < LOGIT_TOL, d
    first = eng.tokens(1)[0]
    assert first == int(np.argmax(ref[-1]))
    rng = np.random.default_rng(3)
    tree = synth.seeded_tree(rng, [first] * 9, n=16, vocab=VOCAB_SMALL)
    eng.verify(tree)
    gl = eng.logits().cpu().numpy()
    rl = Q.tree_pass(m, cache.copy(), len(prompt), first, tree)
    d = np.abs(gl - rl).max()
    agree = int((gl.argmax(1) == rl.argmax(1)).sum())
    assert d < LOGIT_TOL, d
    assert agree >= 15, agree


def test_commit_kernel_matches_commit_oracle(small):
    """Tree walk, token commit, pos update and KV compaction against oracle.commit with crafted
    argmax partials (including ties, which must resolve to the lowest id)."""
    fmt, w, m, eng = small
    if fmt != "q4":
        pytest.skip("format independent")
    rng = np.random.default_rng(17)
    for case in range(25):
        prompt = (synth.make_prompt(20 + case, seed=case) % VOCAB_SMALL).tolist()
        eng.begin(0, 40)
        eng.prefill(prompt)
        st0 = eng.state()
        n = int(rng.integers(1, 17))
        y = list(rng.integers(0, 8, size=9))
        tree = synth.seeded_tree(rng, y, n=n, vocab=8)
        eng.verify(tree)
        torch.cuda.synchronize()
        # crafted argmaxes: on-path rows follow y, others random in a small alphabet
        g = [int(v) for v in rng.integers(0, 8, size=n)]
        path = A.walk_tree(tree, [y[tree["depth"][i]] for i in range(n)])
        for k, row in enumerate([0] + path):
            g[row] = int(y[k])
        pval, pidx = eng.argmax_partials()
        parts = pval.shape[1]
        pval.fill_(-1.0)
        pidx.copy_(torch.arange(parts, device=pval.device, dtype=torch.int32).mul(16).expand(16, parts))
        for t in range(n):
            # two tied maxima: the lower id must win
            pval[t, (g[t] + 30) % parts] = 5.0
            pidx[t, (g[t] + 30) % parts] = g[t]
            pval[t, (g[t] + 31) % parts] = 5.0
            pidx[t, (g[t] + 31) % parts] = g[t] + 1000
        k_before, v_before = [b.clone() for b in eng.kv()]
        eng.commit()
        st = eng.state()
        exp = A.commit(tree, g, st0["pos"], st0["step"], 40)
        got = eng.tokens(st["step"])[st0["step"]:]
        assert got == exp["tokens"], (case, got, exp)
        assert st["pos"] == exp["pos"] and st["step"] == exp["step"]
        assert st["accepted"] - st0["accepted"] == exp["m"]
        k_after, v_after = eng.kv()
        kx, vx = k_before.clone(), v_before.clone()
        for src, dst in exp["moves"]:
            kx[:, :, dst] = kx[:, :, src]
            vx[:, :, dst] = vx[:, :, src]
        assert torch.equal(kx, k_after) and torch.equal(vx, v_after)


def test_device_errors_set_flags_without_hanging(small):
    fmt, w, m, eng = small
    if fmt != "q4":
        pytest.skip("format independent")
    eng.begin(0, 8)
    eng.prefill([1, 2, 3])
    bad = synth.seeded_tree(np.random.default_rng(0), [1] * 9, n=4)
    bad["parent"][3] = 3  # a row cannot be its own parent
    eng.verify(bad)
    st = eng.state()
    assert st["err"] & 1 and st["done"] == 1
    eng.commit()  # later kernels of the request return at once
    assert eng.state()["step"] == st["step"]
    # context overflow detected on the device
    eng2 = _engine(w, max_ctx=64, max_steps=16)
    eng2.begin(0, 4)
    eng2.prefill(list(range(70)))
    st = eng2.state()
    assert st["err"] & 2 and st["done"] == 1
    eng2.close()


def test_write_state_replays_a_pass(small):
    """vp_write_state: a state snapshot written back (from device and from host memory) replays the
    same pass over the same cached prefix: same committed tokens, same state, same KV rows."""
    fmt, w, m, eng = small
    if fmt != "q4":
        pytest.skip("format independent")
    prompt = (synth.make_prompt(21, seed=5) % VOCAB_SMALL).tolist()
    eng.begin(0, 40)
    eng.prefill(prompt)
    snap = eng.snapshot()
    first = eng.tokens(1)[0]
    tree = synth.seeded_tree(np.random.default_rng(9), [first] * 9, n=12, vocab=VOCAB_SMALL)
    eng.pass_(tree)
    st1, tok1 = eng.state(), eng.tokens()
    k1, v1 = (x.clone() for x in eng.kv())
    for on_device in (True, False):
        eng.restore(snap, on_device=on_device)
        assert eng.state()["step"] == 1
        eng.pass_(tree)
        assert eng.state() == st1 and eng.tokens() == tok1
        k2, v2 = eng.kv()
        assert torch.equal(k1, k2) and torch.equal(v1, v2)


def test_prefix_file_skips_prefill(small, tmp_path):
    """Engine.savePrefix / loadPrefix: a fresh engine that loads a saved 32-token prefix and
    prefills only the rest of the prompt decodes exactly the tokens of a full prefill."""
    fmt, w, m, eng = small
    if fmt != "q4":
        pytest.skip("format independent")
    prompt = (synth.make_prompt(40, seed=12) % VOCAB_SMALL).tolist()
    full = eng.generate(prompt, 20)
    path = str(tmp_path / "prefix.bin")
    eng.save_prefix(path, prompt[:32])
    other = _engine(w, max_ctx=512, max_steps=128)
    assert other.load_prefix(path) == prompt[:32]
    got = other.generate(prompt, 20, cached=32)
    assert got["tokens"] == full["tokens"]
    other.close()
    # a file made for another context size (or model) is refused
    third = _engine(w, max_ctx=256, max_steps=128)
    assert third.load_prefix(path) is None
    third.close()


# ---------------------------------------------------------------------------------------------
# full-size model


@pytest.fixture(scope="module")
def full_q4():
    w = synth.make_weights("q4", seed=0)
    eng = _engine(w, max_ctx=4096, max_steps=512)
    yield w, eng
    eng.close()


def _check_head_partials(eng, rows):
    """The pass's lm_head stage (per CTA: the largest logit of its vocabulary rows and the lowest
    id holding it, per token) against the stand-alone head's full logits on the same rows: equal
    bit for bit. The two are separate kernels with their own work split; the tokens the commit
    takes, the no-alloc head and the sketch head all rely on their arithmetic being the same."""
    pval, pidx = (a.cpu().numpy() for a in eng.argmax_partials())
    gl = eng.logits().cpu().numpy()
    G = pval.shape[1]
    nrb = gl.shape[1] // 16
    for cta in range(G):
        rb0, rb1 = cta * nrb // G, (cta + 1) * nrb // G
        seg = gl[:rows, 16 * rb0:16 * rb1]
        best = seg.max(axis=1)
        ids = seg.argmax(axis=1) + 16 * rb0  # first maximum = lowest id
        assert np.array_equal(best.view(np.uint32), pval[:rows, cta].view(np.uint32)), (cta, best, pval[:rows, cta])
        assert np.array_equal(ids, pidx[:rows, cta]), (cta, ids, pidx[:rows, cta])


def test_pass_lm_head_equals_standalone_head(small):
    fmt, w, m, eng = small
    prompt = (synth.make_prompt(29, seed=11) % VOCAB_SMALL).tolist()
    eng.begin(0, 32)
    eng.prefill(prompt)
    first = eng.tokens(1)[0]
    eng.verify(synth.seeded_tree(np.random.default_rng(5), [first] * 9, n=16, vocab=VOCAB_SMALL))
    _check_head_partials(eng, 16)


def test_pass_lm_head_equals_standalone_head_full_vocab(full_q4):
    w, eng = full_q4
    prompt = synth.make_prompt(64, seed=77).tolist()
    eng.begin(0, 32)
    eng.prefill(prompt)
    first = eng.tokens(1)[0]
    eng.verify(synth.seeded_tree(np.random.default_rng(6), [first] * 9, n=16))
    _check_head_partials(eng, 16)


def _tree_fn(y_seq, rng, n=16, p=0.6):
    def fn(out):
        y = list(y_seq[len(out):len(out) + 9])
        y += [0] * (9 - len(y))
        return synth.seeded_tree(rng, y, n=n, p_match=p)
    return fn


def test_tree_equals_sequential_200_prompts(full_q4):
    """token-for-token bit-identical tree vs sequential output on 200 seeded
    prompts (q4, full model, 16-row trees as in config 2)."""
    w, eng = full_q4
    passes_seq = passes_tree = 0
    for i in range(200):
        prompt = synth.make_prompt(8 + (i * 37) % 120, seed=500 + i).tolist()
        seq = eng.generate(prompt, 24)
        rng = np.random.default_rng(i)
        tr = eng.generate(prompt, 24, tree_fn=_tree_fn(seq["tokens"], rng))
        assert tr["tokens"] == seq["tokens"], i
        passes_seq += seq["passes"]
        passes_tree += tr["passes"]
    # the seeded trees must actually speculate: fewer passes than tokens
    assert passes_tree < 0.7 * passes_seq


def test_fused_pass_equals_separate_launches(full_q4):
    """vp_pass (verify + commit in one launch) and vp_verify + vp_commit give the same tokens."""
    w, eng = full_q4
    prompt = synth.make_prompt(40, seed=77).tolist()
    seq = eng.generate(prompt, 20)
    a = eng.generate(prompt, 20, tree_fn=_tree_fn(seq["tokens"], np.random.default_rng(1)))
    b = eng.generate(prompt, 20, tree_fn=_tree_fn(seq["tokens"], np.random.default_rng(1)),
                     fused=False)
    assert a["tokens"] == b["tokens"] == seq["tokens"]
    assert a["passes"] == b["passes"]


def test_pass_graph_replays_the_pass(full_q4):
    """vp_pass_graph: the fused pass captured once as a CUDA graph over the context's own tree
    buffer and replayed per pass (the tree written into that buffer before each replay) commits
    the tokens the library call does."""
    w, eng = full_q4
    prompt = synth.make_prompt(48, seed=78).tolist()
    seq = eng.generate(prompt, 24)
    tree_buf = eng.buffer(7, (synth.TREE_INTS,), "<i4")
    g = eng.pass_graph(tree_buf)
    try:
        fn = _tree_fn(seq["tokens"], np.random.default_rng(5))
        eng.begin(0, 24)
        eng.prefill(prompt)
        out = eng.tokens(1)
        while not eng.state()["done"]:
            tree_buf.copy_(torch.from_numpy(synth.tree_to_buffer(fn(out))).to(eng.device))
            g.launch(eng._s)
            out = eng.tokens()
        assert out == seq["tokens"]
    finally:
        g.close()


def test_config2_logits_match_oracle_full_size(full_q4):
    """Config 2 shape at full size: 256-token prefix, one 16-row tree pass."""
    w, eng = full_q4
    m = Q.model_from_weights(w)
    prompt = synth.make_prompt(256, seed=1000).tolist()
    eng.begin(0, 32)
    eng.prefill(prompt)
    first = eng.tokens(1)[0]
    cache = Q.KVCache(24, 300)
    ref = Q.forward_causal(m, cache, prompt, 0)
    assert first == int(np.argmax(ref))
    seq_cache = cache.copy()
    y, pos = [first], 256
    for _ in range(9):
        lg = Q.forward_causal(m, seq_cache, [y[-1]], pos)
        y.append(int(np.argmax(lg)))
        pos += 1
    tree = synth.seeded_tree(np.random.default_rng(2), y[1:], n=16)
    eng.verify(tree)
    gl = eng.logits().cpu().numpy()
    rl = Q.tree_pass(m, cache.copy(), 256, first, tree)
    d = np.abs(gl - rl).max()
    agree = int((gl.argmax(1) == rl.argmax(1)).sum())
    print(f"config2 tree logits: max|d|={d:.4g} argmax agree {agree}/16")
    assert d < LOGIT_TOL and agree >= 15
    eng.commit()
    st = eng.state()
    exp = A.commit(tree, gl.argmax(1), 256, 1, 32)
    assert eng.tokens(st["step"])[1:] == exp["tokens"]


@pytest.mark.parametrize("fmt", ["q8", "q8g32"])
def test_config3_q8_chains_equal_sequential(fmt):
    """Config 3: q8 (group 64 as BASELINE, and the reference's own group 32), 1024-token prefix,
    8-row chains with p=0.5 matching drafts, 64 tokens, against 1-row sequential decode through
    the same kernels."""
    w = synth.make_weights(fmt, seed=3)
    eng = _engine(w, max_ctx=2048, max_steps=128)
    prompt = synth.make_prompt(1024, seed=33).tolist()
    seq = eng.generate(prompt, 64)
    rng = np.random.default_rng(9)

    def chain(out):
        y = list(seq["tokens"][len(out):len(out) + 8]) + [0] * 8
        d = [int(y[i]) if rng.random() < 0.5 else int(rng.integers(0, 151643)) for i in range(7)]
        return synth.chain_tree(d)

    tr = eng.generate(prompt, 64, tree_fn=chain)
    assert tr["tokens"] == seq["tokens"]
    assert tr["passes"] < seq["passes"]
    eng.close()


def test_config4_f16_teacher_forced_logits():
    """Config 4: f16, 512-token prompt prefilled in 16-row chunks, 16-row tree decode to 64 tokens;
    logits of every decoded position against the fp32 oracle fed the same tokens."""
    w = synth.make_weights("f16", seed=4)
    m = Q.model_from_weights(w)
    eng = _engine(w, max_ctx=1024, max_steps=128)
    prompt = synth.make_prompt(512, seed=44).tolist()
    seq = eng.generate(prompt, 64)
    rng = np.random.default_rng(4)
    tr = eng.generate(prompt, 64, tree_fn=_tree_fn(seq["tokens"], rng))
    assert tr["tokens"] == seq["tokens"]
    toks = seq["tokens"]
    cache = Q.KVCache(24, 600)
    ref = Q.forward_causal(m, cache, prompt + toks[:-1], 0, all_logits=True)[511:]
    agree = int((ref.argmax(1) == np.asarray(toks)).sum())
    print(f"config4 teacher-forced argmax agreement {agree}/{len(toks)}")
    assert agree >= len(toks) - 2
    # logits of the first tree pass against the oracle
    eng.begin(0, 64)
    eng.prefill(prompt)
    tree = synth.seeded_tree(np.random.default_rng(5), toks[1:10], n=16)
    eng.verify(tree)
    gl = eng.logits().cpu().numpy()
    c2 = Q.KVCache(24, 600)
    Q.forward_causal(m, c2, prompt, 0)
    rl = Q.tree_pass(m, c2, 512, toks[0], tree)
    d = np.abs(gl - rl)
    rel = d.max() / np.abs(rl).max()
    print(f"config4 tree logits max|d|={d.max():.4g} max rel {rel:.3g}")
    assert d.max() < LOGIT_TOL
    eng.close()
