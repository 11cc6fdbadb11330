"""The CPU oracle of the drafter (oracle/drafter.py) against the reference drafter's golden record
(tests/golden/drafter_trees.json, made by the reference's tools/draft/ildraft.py), on the table
subset tests/golden/draft_subset.ildraft (tests/golden/make_draft_subset.py: the entries of the
reference's shipped table those cases read; the reference reproduces its own record on it). Pins
the oracle that the GPU drafter is checked against. CPU only."""
import json
import os

import numpy as np
import pytest

from instantllm_b200 import draft_table as dt
from oracle import drafter as D

HERE = os.path.dirname(__file__)
GOLD = json.load(open(os.path.join(HERE, "golden", "drafter_trees.json")))


@pytest.fixture(scope="module")
def table():
    return D.OracleTable(dt.DraftTable.load(os.path.join(HERE, "golden", "draft_subset.ildraft")))


def test_neighbours_on_the_subset(table):
    for case in GOLD["cases"]:
        req = D.Request(table, case["pids"], case["text"])
        assert [[s, len(seq)] for s, seq, _ in req.nb] == case["neighbours"]


def test_features_probs_and_trees_equal_the_reference(table):
    for case in GOLD["cases"]:
        req = D.Request(table, case["pids"], case["text"])
        for st in case["steps"]:
            toks, rows = req.features(st["out"])
            assert toks == st["features"]["tokens"]
            nz = [[i, f, v] for i, r in enumerate(rows) for f, v in enumerate(r) if v != 0.0]
            assert len(nz) == len(st["features"]["nz"])
            for (i, f, v), (gi, gf, gv) in zip(nz, st["features"]["nz"]):
                assert (i, f) == (gi, gf) and v == pytest.approx(gv, rel=1e-12, abs=1e-15)
            pr = req.probs(st["out"])[:5]
            assert [k for k, _ in pr] == [k for k, _ in st["probs"]]
            assert np.allclose([p for _, p in pr], [p for _, p in st["probs"]], rtol=1e-12, atol=0)
            asked = []

            def probs(path, _out=st["out"]):
                asked.append(list(path))
                return req.probs(list(_out) + list(path))

            assert D.best_first_tree(probs, GOLD["B"], GOLD["branch"]) == (st["parents"], st["tokens"])
            assert asked == [p for p, _ in st["expansions"]]
            for path, top in st["expansions"]:
                got = req.probs(list(st["out"]) + list(path))[:8]
                assert [k for k, _ in got] == [k for k, _ in top]
                assert np.allclose([p for _, p in got], [p for _, p in top], rtol=1e-12, atol=0)
