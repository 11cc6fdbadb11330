"""The device drafter (vp_draft, k_draft) against the reference drafter's golden record
(tests/golden/drafter_trees.json, made by the reference's tools/draft/ildraft.py) on the table
subset tests/golden/draft_subset.ildraft: for every golden step the same tree node for node, every
expansion in the reference's order with the reference's 8 probabilities (to 1e-9), and the tree
buffer the next verify pass reads.

Candidates with identical feature rows have identical scores on the GPU, so their order is the
token order the reference's rule asks for (probability descending, then token ascending). The
reference computes its scores with a BLAS matrix product whose rounding can differ by a few ulps
between identical rows, which may order such candidates differently; so each expansion's tokens are
checked through the CPU oracle (pinned to the golden record by tests/test_drafter_oracle.py): every
token the GPU ranks k-th has, in the reference's arithmetic, the reference's k-th probability."""
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(__file__)
GOLD = json.load(open(os.path.join(HERE, "golden", "drafter_trees.json")))


def test_device_drafter_reproduces_the_reference_trees():
    from instantllm_b200 import draft_table as dt
    from instantllm_b200.drafter import DeviceDrafter
    from oracle import drafter as D

    ot = D.OracleTable(dt.DraftTable.load(os.path.join(HERE, "golden", "draft_subset.ildraft")))
    d = DeviceDrafter(os.path.join(HERE, "golden", "draft_subset.ildraft"))
    dev = d.device
    tree = torch.zeros(65, dtype=torch.int32, device=dev)
    n_steps = 0
    for case in GOLD["cases"]:
        d.begin(case["pids"], case["text"])
        req = D.Request(ot, case["pids"], case["text"])
        for st in case["steps"]:
            out = torch.tensor(st["out"] + [0], dtype=torch.int32, device=dev)  # non-empty buffer
            got = d.draft(tree, out, n_out=len(st["out"]), B=GOLD["B"], branch=GOLD["branch"], debug=True)
            assert got["status"] == 0
            assert (got["parents"], got["tokens"]) == (st["parents"], st["tokens"]), (case["text"], st["out"])
            for k, (path, top) in enumerate(st["expansions"]):
                want_p = [p for _, p in top]
                gt = [int(x) for x in got["exp_tokens"][k][:len(top)]]
                assert len(set(gt)) == len(gt) and all(x >= 0 for x in gt), (k, path)
                assert np.allclose(got["exp_probs"][k][:len(top)], want_p, rtol=1e-9, atol=0), (k, path)
                ref = dict(req.probs(list(st["out"]) + list(path)))
                assert np.allclose([ref[x] for x in gt], want_p, rtol=1e-9, atol=0), (k, path, gt)
            tb = tree.cpu().numpy()
            n = len(st["tokens"]) + 1
            assert tb[0] == n
            for i, (par, tok) in enumerate(zip(st["parents"], st["tokens"])):
                assert tb[17 + i + 1] == par + 1 and tb[33 + i + 1] == tok
                assert tb[1 + i + 1] == tb[1 + par + 1] + 1
            n_steps += 1
    assert n_steps == sum(len(c["steps"]) for c in GOLD["cases"])
    d.close()


def test_drafted_decode_loop_equals_greedy_decoding():
    """VerifyEngine.generate_drafted: every step is k_draft (the tree from the device's committed
    tokens and state, written into the pass's own tree buffer) and one pass, enqueued `depth`
    steps ahead with the shape chosen by PassShape from the counters the host has seen; no token
    or tree goes through the host. Its output must be plain greedy decoding (1-row passes through
    the same kernels) token for token, at every depth. The model is random-init, so few drafts are
    accepted and the adaptive rule must fall back to 8-row chains after the first passes."""
    from instantllm_b200 import synth
    from instantllm_b200.drafter import DeviceDrafter
    from instantllm_b200.engine import PassShape, VerifyEngine

    w = synth.make_weights("q4", seed=3)
    eng = VerifyEngine(w, max_ctx=1024, max_steps=256)
    d = DeviceDrafter(os.path.join(HERE, "golden", "draft_subset.ildraft"))
    try:
        for i, case in enumerate(GOLD["cases"]):
            depth = i % 3
            prompt = list(case["pids"])
            ref = eng.generate(prompt, 40)
            got = eng.generate_drafted(prompt, 40, d, pids=prompt, text=case["text"], depth=depth)
            assert got["tokens"] == ref["tokens"], (i, depth)
            assert got["state"]["err"] == 0
            shapes = got["shapes"]
            assert shapes[0] == (15, 8)
            rate = got["state"]["accepted"] / max(1, got["passes"])
            if rate < 1.5 and got["passes"] >= 4:
                assert (7, 1) in shapes, (i, shapes)
            assert got["passes"] <= len(shapes) <= got["passes"] + depth + 1
        # the same loop with each step replayed as a CUDA graph (vp_step_graph)
        case = GOLD["cases"][1]
        prompt = list(case["pids"])
        ref = eng.generate(prompt, 40)
        got = eng.generate_drafted(prompt, 40, d, pids=prompt, text=case["text"], depth=1, graphs=True)
        assert got["tokens"] == ref["tokens"]
        # a step graph captured for one request refuses to run after the drafter began another
        g = eng.step_graph(d, 15, 8)
        d.begin(prompt, case["text"])
        from instantllm_b200 import _lib
        with pytest.raises(_lib.VpError):
            g.launch(eng._s)
        g.close()
        # the non-adaptive tree loop gives the same tokens too
        prompt = list(GOLD["cases"][0]["pids"])
        fixed = eng.generate_drafted(prompt, 40, d, pids=prompt, text=GOLD["cases"][0]["text"],
                                     shape=PassShape(adaptive=False))
        assert fixed["tokens"] == eng.generate(prompt, 40)["tokens"]
        assert set(fixed["shapes"]) == {(15, 8)}
    finally:
        d.close()
        eng.close()


def test_batched_drafted_loop_equals_greedy_decoding_on_its_share():
    """VerifyEngine.generate_drafted_batch: four (then two) requests, each step their drafts side by
    side on their own streams and one vp_pass_batch launch; every request's output must be its
    greedy decoding on the same share of the SMs (batched prefill, then 1-row passes), token for
    token."""
    from instantllm_b200 import synth
    from instantllm_b200.drafter import DeviceDrafter
    from instantllm_b200.engine import STOP_IDS, VerifyEngine

    w = synth.make_weights("q4", seed=3)
    engs = [VerifyEngine(w, max_ctx=1024, max_steps=256) for _ in range(4)]
    ds = [DeviceDrafter(os.path.join(HERE, "golden", "draft_subset.ildraft")) for _ in range(4)]
    root = torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=engs[0].device)
    try:
        for k, depth in ((4, 1), (2, 0)):
            cases = GOLD["cases"][:k]
            prompts = [list(c["pids"]) for c in cases]
            for e in engs[:k]:
                e.begin(0, 40, STOP_IDS)
            VerifyEngine.prefill_batch(engs[:k], prompts)
            for _ in range(39):
                VerifyEngine.pass_multi(engs[:k], [root] * k, shares=k)
            truth = [e.tokens(e.state()["step"]) for e in engs[:k]]
            got = VerifyEngine.generate_drafted_batch(engs[:k], prompts, 40, ds[:k], pids=prompts,
                                                      texts=[c["text"] for c in cases], depth=depth)
            for r in range(k):
                assert got[r]["tokens"] == truth[r], (k, r)
                assert got[r]["state"]["err"] == 0 and got[r]["shapes"][0] == (15, 8)
    finally:
        for d in ds:
            d.close()
        for e in engs:
            e.close()


def test_device_drafter_long_request_matches_the_oracle():
    """A request past the kernel's shared-memory staging caps for the prompt and the committed
    output (both longer than 2,048 tokens; the distinct prompt ids stay under the 1,024-candidate
    cap) takes the global-memory paths of k_draft; every expansion's 8 probabilities and the
    probability of each token it ranks must equal the CPU oracle's (oracle/drafter.py, pinned to
    the reference's golden record)."""
    from instantllm_b200 import draft_table as dt
    from instantllm_b200.drafter import DeviceDrafter
    from oracle import drafter as D

    table = os.path.join(HERE, "golden", "draft_subset.ildraft")
    ot = D.OracleTable(dt.DraftTable.load(table))
    d = DeviceDrafter(table)
    rng = np.random.default_rng(11)
    case = GOLD["cases"][0]
    pool = rng.integers(0, 151643, size=800).tolist()
    prompt = []
    while len(prompt) < 4000:
        prompt += list(case["pids"]) + [pool[i] for i in rng.integers(0, len(pool), size=60)]
    prompt = prompt[:4000]
    out = (list(case["steps"][-1]["out"]) * 400)[:2300]
    assert len(set(prompt)) < 1000
    try:
        d.begin(prompt, case["text"])
        req = D.Request(ot, prompt, case["text"])
        tree = torch.zeros(65, dtype=torch.int32, device=d.device)
        o = torch.tensor(out, dtype=torch.int32, device=d.device)
        got = d.draft(tree, o, n_out=len(out), B=15, branch=8, debug=True)
        assert got["status"] == 0
        par, tok = got["parents"], got["tokens"]
        # expansion order: the root, then every node that was neither a stop token nor the last
        paths = [[]]
        for i in range(len(tok)):
            if tok[i] not in (151645, 151643) and i + 1 < 15:
                p, v = [], i
                while v >= 0:
                    p.append(tok[v])
                    v = par[v]
                paths.append(p[::-1])
        assert len(paths) >= 2
        for k, path in enumerate(paths[:16]):
            ref = req.probs(out + path)
            gt = [int(x) for x in got["exp_tokens"][k] if x >= 0]
            gp = got["exp_probs"][k][:len(gt)]
            want = [p for _, p in ref[:8]]
            assert len(gt) == len(want), (k, path)
            assert np.allclose(gp, want, rtol=1e-9, atol=0), (k, path)
            rd = dict(ref)
            assert np.allclose([rd[x] for x in gt], gp, rtol=1e-9, atol=0), (k, path)
    finally:
        d.close()
