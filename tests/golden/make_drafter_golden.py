"""Golden draft trees from the reference drafter (tools/draft/ildraft.py: Drafter.begin, probs,
tree, chain) on the table the reference ships, for synthetic requests: prompt ids drawn from a seeded
generator, prompt texts written for this fixture, and outputs grown by the drafter's own greedy
chain, with each step's candidate feature rows (ildraft.py FEATS order). No tokenizer is given
(the reference's space-variant and edited-neighbour features need one and are then skipped), as a
drafter without the tokenizer runs. Ground truth for a port of the drafter.

Usage: python tests/golden/make_drafter_golden.py --reference <instantllm checkout> \
           [--out tests/golden/drafter_trees.json]
"""
import argparse
import json
import os
import random
import sys

TEXTS = [  # synthetic prompts written for this fixture
    "Write a Python function that merges two sorted lists into one sorted list.",
    "Explain the difference between TCP and UDP in three sentences.",
    "List five prime numbers greater than 100 and explain how you checked them.",
    "Summarize: the cache stores 4096 entries, evicts the least recently used one, and logs misses.",
]


def golden_cases(d, t) -> dict:
    """The golden record of the TEXTS requests on table t with the reference module d (ildraft)."""
    rnd = random.Random(11)
    cases = []
    for text in TEXTS:
        pids = [rnd.randrange(1000, 100000) for _ in range(rnd.randrange(8, 24))]
        dr = d.Drafter(t)
        dr.begin(pids, text)
        out, steps = [], []
        for _ in range(3):
            calls, real = [], dr.probs

            def recording(o, _real=real, _calls=calls, _n=len(out)):
                r = _real(o)
                _calls.append([list(o[_n:]), [[int(k), float(p)] for k, p in r[:8]]])
                return r

            dr.probs = recording  # every context the tree expands: its path below `out`, top 8
            parents, tokens = dr.tree(out, 15)
            dr.probs = real
            pr = dr.probs(out)[:5]
            ftoks, rows = dr.features(out)  # candidate rows: sparse (candidate, feature, value)
            nz = [[i, f, float(v)] for i, r in enumerate(rows) for f, v in enumerate(r) if v != 0.0]
            steps.append({"out": list(out), "parents": parents, "tokens": tokens,
                          "probs": [[int(k), float(p)] for k, p in pr],
                          "features": {"tokens": [int(x) for x in ftoks], "nz": nz},
                          "expansions": calls})
            grow = dr.chain(out, 4)
            if not grow:
                break
            out = out + grow
        cases.append({"pids": pids, "text": text, "neighbours": [[float(s), len(seq)] for s, seq, _ in dr.nb],
                      "steps": steps})
    return {"B": 15, "branch": 8, "cases": cases}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "drafter_trees.json"))
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.reference, "tools", "draft"))
    import ildraft as d

    t = d.Tables.load(os.path.join(a.reference, "tools", "draft", "ildraft-q4.bin"))
    with open(a.out, "w") as f:
        json.dump(golden_cases(d, t), f, separators=(",", ":"))
    print(a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()
