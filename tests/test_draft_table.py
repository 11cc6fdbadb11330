"""The drafter table reader and lookup primitives (instantllm_b200.draft_table) against golden vectors
from the reference's own ildraft.py (tests/golden/make_draft_golden.py): hashes, context keys and
prompt words always; the reader on a small ILDRAFT1 file written here; and, when
INSTANTLLM_DRAFT_TABLE names the reference's table (tools/draft/ildraft-q4.bin), every lookup the
golden file recorded on it. CPU only."""
import json
import os
import struct

import numpy as np
import pytest

from instantllm_b200 import draft_table as dt
from oracle import drafter as D

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "draft_table.json")))


def test_hashes_and_prompt_words():
    for hexb, v in GOLD["fnv"]:
        assert dt.fnv1a64(bytes.fromhex(hexb)) == v
    for ctx, v in GOLD["ctx_key"]:
        assert dt.ctx_key(ctx) == v
    for text, words in GOLD["prompt_words"]:
        assert [w.decode() for w in dt.prompt_words(text)] == words


def _table(sections, N=6, M=6, H=2, flags=dt.FLAG_ASSOC):
    """A small ILDRAFT1 file: header, directory, 8-aligned sections."""
    F = dt.N_FEATURES
    body, dirent, off = b"", [], 64 + 16 * len(sections)
    off = (off + 7) & ~7
    start = off
    for tag, (count, data) in sections.items():
        pad = (-(start + len(body))) % 8
        body += b"\0" * pad
        dirent.append(struct.pack("<4sIQ", tag, count, start + len(body)))
        body += data
    head = struct.pack("<8sII" + "I" * 8 + "IIII", b"ILDRAFT1", 1, len(sections), N, M, 16, 12, F, H, 1, 2,
                       flags, 3, 0, 0)
    raw = head + b"".join(dirent)
    return raw + b"\0" * (start - len(raw)) + body


def test_reader_on_a_written_table():
    ctxs = {(5,): (10, [(7, 6), (9, 4)]), (1, 2): (3, [(4, 3)]), (151645, 198, 151644): (2, [(77091, 2)])}
    items = sorted((dt.ctx_key(c), v) for c, v in ctxs.items())
    nx, vals = [], []
    for _, (tot, nexts) in items:
        vals.append(struct.pack("<II", tot, (len(nx) << 3) | len(nexts)))
        nx += nexts
    words = sorted((dt.fnv1a64(w), w) for w in (b"cache", b"prime"))
    H, F = 2, dt.N_FEATURES
    mlp = np.arange(H * F + H + H + 1 + F, dtype=np.float32) / 100
    secs = {
        b"NGKY": (len(items), b"".join(struct.pack("<Q", k) for k, _ in items)),
        b"NGVL": (len(vals), b"".join(vals)),
        b"NGNX": (len(nx), b"".join(struct.pack("<II", *p) for p in nx)),
        b"WDKY": (2, b"".join(struct.pack("<Q", k) for k, _ in words)),
        b"WDVL": (2, struct.pack("<fII", 1.5, 0, 2) + struct.pack("<fII", 0.25, 2, 1)),
        b"POST": (3, struct.pack("<III", 0, 1, 1)),
        b"DNRM": (2, struct.pack("<ff", 2.0, 3.0)),
        b"SQOF": (3, struct.pack("<III", 0, 2, 5)),
        b"SQTK": (5, struct.pack("<IIIII", 11, 151645, 12, 13, 151643)),
        b"ASWK": (1, struct.pack("<Q", words[0][0])),
        b"ASWV": (1, struct.pack("<II", 0, 2)),
        b"ASTK": (2, struct.pack("<IfIf", 42, 3.5, 43, 2.5)),
        b"TFLS": (2, struct.pack("<IIII", 63, 1, 198, 8)),
        b"MLP0": (len(mlp), mlp.tobytes()),
    }
    t = dt.DraftTable(_table(secs))
    assert (t.N, t.M, t.H, t.n_docs) == (6, 6, 2, 2)
    for c, v in ctxs.items():
        assert t.ng_get(c) == v
    assert t.ng_get((5, 5)) is None
    w0 = words[0][1]
    assert t.vocab_get(w0) == (1.5, [0, 1]) and t.vocab_get(b"nothere") is None
    assert t.assoc_get(w0) == [(42, 3.5), (43, 2.5)]
    assert t.seq(0) == [11, 151645] and t.seq(1) == [12, 13, 151643]
    f = t.token_flags()
    assert f[63] == 1 and f[198] == 8 and f.sum() == 9
    m = t.mlp()
    assert m["W1"].shape == (H, F) and m["b2"] == float(mlp[H * F + 2 * H])
    with pytest.raises(ValueError, match="ILDRAFT1"):
        dt.DraftTable(b"X" * 128)


@pytest.mark.skipif(not os.environ.get("INSTANTLLM_DRAFT_TABLE"), reason="INSTANTLLM_DRAFT_TABLE not set")
def test_reader_on_the_reference_table():
    t = dt.DraftTable.load(os.environ["INSTANTLLM_DRAFT_TABLE"])
    h = GOLD["header"]
    assert (t.N, t.M, t.KNB, t.MAXM, t.H, t.minc_hi, t.flags, t.as_top, t.edit_E) == \
        (h["N"], h["M"], h["KNB"], h["MAXM"], h["H"], h["minc_hi"], h["flags"], h["as_top"], h["edit_E"])
    assert len(t.sec[b"SQOF"]) - 1 == h["n_docs"]
    for ctx, want in GOLD["ng"]:
        got = t.ng_get(ctx)
        assert (None if got is None else [got[0], [list(p) for p in got[1]]]) == want, ctx
    for w, voc, asc in GOLD["words"]:
        v = t.vocab_get(w.encode())
        assert (None if v is None else [v[0], len(v[1]), v[1][:8]]) == voc, w
        a = t.assoc_get(w.encode())
        assert (None if not a else [len(a), [list(p) for p in a[:5]]]) == asc, w
    for j, n, head in GOLD["seqs"]:
        s = t.seq(j)
        assert len(s) == n and s[:10] == head
    for j, v in GOLD["norms"]:
        assert float(t.sec[b"DNRM"][j]) == v
    m = t.mlp()
    got = {"W1": sum(sum(float(x) for x in r) for r in m["W1"]), "b1": sum(float(x) for x in m["b1"]),
           "W2": sum(float(x) for x in m["W2"]), "b2": m["b2"], "WL": sum(float(x) for x in m["WL"])}
    assert got == GOLD["mlp"]
    f = t.token_flags()
    for i, v in GOLD["tflags"]:
        assert int(f[i]) == v


def test_drafter_golden_trees_are_well_formed():
    """The reference drafter's trees recorded for a later port (make_drafter_golden.py): best-first
    order (parents[i] < i, the first node the root's most probable child), B nodes, probabilities
    sorted, outputs grown from one step to the next."""
    g = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "drafter_trees.json")))
    for case in g["cases"]:
        assert 0 < len(case["neighbours"]) <= GOLD["header"]["KNB"]
        prev = None
        for st in case["steps"]:
            par, tok, pr = st["parents"], st["tokens"], st["probs"]
            assert len(tok) == len(par) == g["B"]
            assert all(-1 <= p < i for i, p in enumerate(par))
            assert par[0] == -1 and tok[0] == pr[0][0]
            assert all(pr[i][1] >= pr[i + 1][1] for i in range(len(pr) - 1))
            assert all(0 <= x < dt.VOCAB for x in tok)
            if prev is not None:
                assert st["out"][:len(prev)] == prev and len(st["out"]) > len(prev)
            prev = st["out"]


@pytest.mark.skipif(not os.environ.get("INSTANTLLM_DRAFT_TABLE"), reason="INSTANTLLM_DRAFT_TABLE not set")
def test_neighbours_match_the_reference_drafter():
    """Drafter.begin's nearest training documents for the golden requests: same scores (float64,
    the same summation order) and the same documents (their sequence lengths)."""
    t = dt.DraftTable.load(os.environ["INSTANTLLM_DRAFT_TABLE"])
    g = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "drafter_trees.json")))
    for case in g["cases"]:
        got = t.neighbours(case["text"])
        assert [[s, 5 + len(t.seq(j))] for s, j in got] == case["neighbours"]


def _rows(feat):
    rows = np.zeros((len(feat["tokens"]), dt.N_FEATURES), dtype=np.float64)
    for i, f, v in feat["nz"]:
        rows[i, f] = v
    return rows


def test_golden_feature_rows_are_well_formed():
    g = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "drafter_trees.json")))
    for case in g["cases"]:
        for st in case["steps"]:
            rows = _rows(st["features"])
            assert np.all(rows[:, 0] == 1.0)  # the bias feature of every candidate
            assert {k for k, _ in st["probs"]} <= set(st["features"]["tokens"])


@pytest.mark.skipif(not os.environ.get("INSTANTLLM_DRAFT_TABLE"), reason="INSTANTLLM_DRAFT_TABLE not set")
def test_scorer_matches_the_reference_drafter():
    """The oracle's scorer with the table's MLP, over the reference's own feature rows, gives the
    reference's probabilities."""
    t = dt.DraftTable.load(os.environ["INSTANTLLM_DRAFT_TABLE"])
    g = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "drafter_trees.json")))
    for case in g["cases"]:
        for st in case["steps"]:
            got = D.probs_of_rows(D.OracleTable(t), st["features"]["tokens"], _rows(st["features"]))[:5]
            assert [k for k, _ in got] == [k for k, _ in st["probs"]]
            assert np.allclose([p for _, p in got], [p for _, p in st["probs"]], rtol=1e-12, atol=0)


def test_best_first_tree_matches_the_reference_trees():
    """Fed the probabilities the reference drafter computed for every node it expanded, the
    oracle's tree builder makes the reference's trees (same nodes, order and parents) and asks for exactly the
    recorded nodes."""
    g = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "drafter_trees.json")))
    for case in g["cases"]:
        for st in case["steps"]:
            rec = {tuple(path): [tuple(x) for x in top] for path, top in st["expansions"]}
            asked = []

            def probs(path):
                asked.append(tuple(path))
                return rec[tuple(path)]

            par, tok = D.best_first_tree(probs, g["B"], g["branch"])
            assert (par, tok) == (st["parents"], st["tokens"])
            assert asked == [tuple(p) for p, _ in st["expansions"]]
