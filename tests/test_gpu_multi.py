"""vp_pass_multi: two requests' verify passes in one launch, each on half of the SMs.

Every request gets the same share of the SMs whatever the number of requests in the launch, so a
request decoded with 16-row trees through vp_pass_multi commits exactly the tokens that 1-row passes
through vp_pass_multi commit (tree == sequential), whether its partner request runs beside it or
not; its logits match the fp32 oracle."""
import numpy as np
import pytest
import torch

from instantllm_b200 import synth
from oracle import accept as A
from oracle import qwen_oracle as Q

pytestmark = pytest.mark.gpu

V = 4096


def _engine(w, seed):
    from instantllm_b200.engine import VerifyEngine

    eng = VerifyEngine(w, max_ctx=512, max_steps=96)
    prompt = (synth.make_prompt(30 + seed, seed=seed) % V).tolist()
    eng.begin(0, 64, (-1, -1))
    eng.prefill(prompt)
    return eng, prompt, eng.snapshot()


def _root(eng):
    return torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=eng.device)


def test_two_requests_per_launch_tree_equals_sequential():
    from instantllm_b200.engine import VerifyEngine

    w = synth.make_weights("q4", n_layers=2, vocab=V, seed=61)
    (ea, pa, sa), (eb, pb, sb) = _engine(w, 1), _engine(w, 2)
    root = _root(ea)
    # sequential truth of both requests, two per launch
    for _ in range(24):
        VerifyEngine.pass_multi([ea, eb], [root, root])
    ya, yb = ea.tokens(25), eb.tokens(25)
    assert ea.state()["err"] == 0 and eb.state()["err"] == 0
    # request a alone through the same entry point: the same tokens (its half of the SMs only)
    ea.restore(sa)
    for _ in range(24):
        VerifyEngine.pass_multi([ea], [root])
    assert ea.tokens(25) == ya
    # 16-row trees from the truth, both requests per launch, every committed token checked
    rng = np.random.default_rng(61)
    ea.restore(sa)
    eb.restore(sb)
    for _ in range(5):
        sta, stb = ea.state(), eb.state()
        ta = synth.seeded_tree(rng, ya[sta["step"]:sta["step"] + 9], n=16, vocab=V)
        tb = synth.seeded_tree(rng, yb[stb["step"]:stb["step"] + 9], n=16, vocab=V)
        VerifyEngine.pass_multi([ea, eb], [torch.tensor(synth.tree_to_buffer(t), device=ea.device)
                                           for t in (ta, tb)])
        for eng, y, st0, tree in ((ea, ya, sta, ta), (eb, yb, stb, tb)):
            st = eng.state()
            parents, tokens = A.to_python_numbering(tree)
            acc = A.accept_tree(parents, tokens, y, st0["step"])
            assert st["step"] == st0["step"] + acc + 1
            assert eng.tokens(st["step"]) == y[:st["step"]]
    # logits of b's last pass against the fp32 oracle over the same committed context
    m = Q.model_from_weights(w)
    cache = Q.KVCache(2, 512)
    Q.forward_causal(m, cache, pb + yb[:stb["step"] - 1], 0)
    ref = Q.tree_pass(m, cache, len(pb) + stb["step"] - 1, yb[stb["step"] - 1], tb)
    got = eb.logits().cpu().numpy()[:16]
    assert float(np.abs(got - ref).max()) < 0.05
    ea.close()
    eb.close()


def test_four_requests_per_launch_tree_equals_sequential():
    """Four shares of the SMs (37 CTAs per request on a B200: QKV, O and down one or two row-blocks
    per CTA): the sequential truth of four requests, one of them again alone and three together on
    their shares, then 16-row trees; every committed token checked, and one request's logits against
    the fp32 oracle."""
    from instantllm_b200.engine import VerifyEngine

    w = synth.make_weights("q4", n_layers=2, vocab=V, seed=64)
    es = [_engine(w, 10 + k) for k in range(4)]
    engs = [e for e, _, _ in es]
    root = _root(engs[0])
    for _ in range(40):
        VerifyEngine.pass_multi(engs, [root] * 4, shares=4)
    ys = [e.tokens(41) for e in engs]
    assert all(e.state()["err"] == 0 for e in engs)
    # the first alone and the other three together, on the same shares: the same tokens
    for e, (_, _, sn) in zip(engs, es):
        e.restore(sn)
    for _ in range(40):
        VerifyEngine.pass_multi(engs[:1], [root], shares=4)
        VerifyEngine.pass_multi(engs[1:], [root] * 3, shares=4)
    assert [e.tokens(41) for e in engs] == ys
    rng = np.random.default_rng(64)
    for e, (_, _, sn) in zip(engs, es):
        e.restore(sn)
    for _ in range(4):
        st0 = [e.state() for e in engs]
        trees = [synth.seeded_tree(rng, y[s["step"]:s["step"] + 9], n=16, vocab=V) for y, s in zip(ys, st0)]
        VerifyEngine.pass_multi(engs, [torch.tensor(synth.tree_to_buffer(t), device=engs[0].device) for t in trees],
                                shares=4)
        for e, y, s, tree in zip(engs, ys, st0, trees):
            st = e.state()
            parents, tokens = A.to_python_numbering(tree)
            assert st["step"] == s["step"] + A.accept_tree(parents, tokens, y, s["step"]) + 1
            assert e.tokens(st["step"]) == y[:st["step"]]
    _, p3, _ = es[3]
    y3, s3 = ys[3], st0[3]
    m = Q.model_from_weights(w)
    cache = Q.KVCache(2, 512)
    Q.forward_causal(m, cache, p3 + y3[:s3["step"] - 1], 0)
    ref = Q.tree_pass(m, cache, len(p3) + s3["step"] - 1, y3[s3["step"] - 1], trees[3])
    got = engs[3].logits().cpu().numpy()[:16]
    assert float(np.abs(got - ref).max()) < 0.05
    for e in engs:
        e.close()


def test_batched_prefill_matches_the_oracle():
    """vp_prefill_batch: three prompts of different lengths (37, 20 and 5 tokens: three, two and one
    16-row chunks) prefilled together on quarters of the SMs; each request's last-chunk logits
    match the fp32 oracle and its first token is the oracle's argmax."""
    from instantllm_b200.engine import VerifyEngine

    w = synth.make_weights("q4", n_layers=2, vocab=V, seed=65)
    engs = [VerifyEngine(w, max_ctx=512, max_steps=96) for _ in range(3)]
    prompts = [(synth.make_prompt(n, seed=80 + n) % V).tolist() for n in (37, 20, 5)]
    for e in engs:
        e.begin(0, 32, (-1, -1))
    VerifyEngine.prefill_batch(engs, prompts, shares=4)
    m = Q.model_from_weights(w)
    for e, p in zip(engs, prompts):
        ref = Q.forward_causal(m, Q.KVCache(2, 512), p, 0, all_logits=True)
        tail = len(p) - (len(p) - 1) // 16 * 16  # rows of the last chunk
        gl = e.logits().cpu().numpy()[:tail]
        assert float(np.abs(gl - ref[len(p) - tail:]).max()) < 0.05
        assert e.tokens(1)[0] == int(np.argmax(ref[-1]))
        assert e.state()["err"] == 0 and e.state()["pos"] == len(p)
    for e in engs:
        e.close()


def test_long_prefixes_two_per_launch_then_one_on_its_half():
    """Rows past the 320 positions of one attention segment (the segmented path), two requests of
    different prefix lengths per launch, then the survivor alone on its half: tree == sequential."""
    from instantllm_b200.engine import VerifyEngine

    w = synth.make_weights("q4", n_layers=2, vocab=V, seed=63)
    engs, snaps = [], []
    for k, n in enumerate((700, 1400)):
        eng = VerifyEngine(w, max_ctx=1600, max_steps=96)
        eng.begin(0, 64, (-1, -1))
        eng.prefill((synth.make_prompt(n, seed=70 + k) % V).tolist())
        engs.append(eng)
        snaps.append(eng.snapshot())
    ea, eb = engs
    root = _root(ea)
    for _ in range(56):  # enough truth for 5 passes of up to 9 committed tokens each
        VerifyEngine.pass_multi(engs, [root, root])
    ys = [e.tokens(57) for e in engs]
    for e, sn in zip(engs, snaps):
        assert e.state()["err"] == 0
        e.restore(sn)
    rng = np.random.default_rng(63)

    def step(which):
        st0 = [engs[i].state() for i in which]
        trees = [synth.seeded_tree(rng, ys[i][s["step"]:s["step"] + 9], n=16, vocab=V) for i, s in zip(which, st0)]
        VerifyEngine.pass_multi([engs[i] for i in which],
                                [torch.tensor(synth.tree_to_buffer(t), device=ea.device) for t in trees])
        for i, s, t in zip(which, st0, trees):
            st = engs[i].state()
            parents, tokens = A.to_python_numbering(t)
            assert st["step"] == s["step"] + A.accept_tree(parents, tokens, ys[i], s["step"]) + 1
            assert engs[i].tokens(st["step"]) == ys[i][:st["step"]]

    for _ in range(3):
        step([0, 1])
    for _ in range(2):
        step([1])
    for e in engs:
        e.close()


def test_a_bad_request_in_a_batch_leaves_its_partners_alone():
    """Failure isolation across shares: one request of a four-request launch gets a malformed tree
    (a row its own parent); it sets its own error bit and stops, without a hang, while the other
    three commit exactly what they commit without it."""
    from instantllm_b200.engine import VerifyEngine

    w = synth.make_weights("q4", n_layers=2, vocab=V, seed=66)
    es = [_engine(w, 20 + k) for k in range(4)]
    engs = [e for e, _, _ in es]
    root = _root(engs[0])
    rng = np.random.default_rng(66)
    trees = []
    for e in engs:
        first = e.tokens(1)[0]
        trees.append(synth.seeded_tree(rng, [first] * 9, n=16, vocab=V))
    bad = dict(trees[2], parent=list(trees[2]["parent"]))
    bad["parent"][5] = 5
    dev = engs[0].device
    VerifyEngine.pass_multi(engs[:2] + engs[3:], [torch.tensor(synth.tree_to_buffer(t), device=dev)
                                                  for t in (trees[0], trees[1], trees[3])], shares=4)
    alone = [e.state()["step"] for e in engs]
    outs = [e.tokens(e.state()["step"]) for e in engs]
    for e, (_, _, sn) in zip(engs, es):
        e.restore(sn)
    VerifyEngine.pass_multi(engs, [torch.tensor(synth.tree_to_buffer(t), device=dev)
                                   for t in (trees[0], trees[1], bad, trees[3])], shares=4)
    st = [e.state() for e in engs]
    assert st[2]["err"] & 1 and st[2]["done"] == 1
    for r in (0, 1, 3):
        assert st[r]["err"] == 0 and st[r]["step"] == alone[r]
        assert engs[r].tokens(st[r]["step"]) == outs[r]
    VerifyEngine.pass_multi(engs, [root] * 4, shares=4)  # the failed request's later passes return at once
    assert engs[2].state()["step"] == st[2]["step"]
    for e in engs:
        e.close()


def test_pass_multi_rejects_bad_arguments():
    import ctypes

    from instantllm_b200 import _lib

    lib = _lib.load()
    w = synth.make_weights("q4", n_layers=1, vocab=V, seed=62)
    eng, _, _ = _engine(w, 3)
    tree = _root(eng)
    one = (ctypes.c_void_p * 2)(eng.ctx.value, eng.ctx.value)
    trees = (ctypes.c_void_p * 2)(tree.data_ptr(), tree.data_ptr())
    assert lib.vp_pass_multi(one, trees, 2, None) == -1  # the same context twice
    assert lib.vp_pass_multi(one, trees, 3, None) == -1
    assert lib.vp_pass_multi(one, trees, 0, None) == -1
    assert lib.vp_pass_batch(one, trees, 2, 1, None) == -1  # more requests than shares
    assert lib.vp_pass_batch(one, trees, 1, 5, None) == -1
    assert lib.vp_pass_batch(one, trees, 1, 0, None) == -1
    ns = (ctypes.c_int32 * 2)(5, 5)
    assert lib.vp_prefill_batch(one, trees, ns, 2, 2, None) == -1  # the same context twice
    assert lib.vp_prefill_batch(one, trees, ns, 3, 2, None) == -1
    eng.close()
