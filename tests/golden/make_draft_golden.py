"""Golden vectors for instantllm_b200.draft_table, produced by the reference drafter itself
(tools/draft/ildraft.py: fnv1a64, ctx_key, prompt_words, Tables.load and its lookups) on the table
the reference ships (tools/draft/ildraft-q4.bin).

Usage: python tests/golden/make_draft_golden.py --reference <instantllm checkout> \
           [--out tests/golden/draft_table.json]
"""
import argparse
import json
import os
import random
import sys

TEXTS = [  # synthetic prompts written for this fixture
    "Write a Python function that merges two sorted lists into one sorted list.",
    "Explain the difference between TCP and UDP in three sentences.",
    "Translate 'good morning, how are you?' into French and German.",
    "List five prime numbers greater than 100 and explain how you checked them.",
    "Summarize: the cache stores 4096 entries, evicts the least recently used one, and logs misses.",
    "naïve café résumé — ÜBER 42 ÉCOLES",
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "draft_table.json"))
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.reference, "tools", "draft"))
    import ildraft as d

    t = d.Tables.load(os.path.join(a.reference, "tools", "draft", "ildraft-q4.bin"))
    c = t.cfg
    out = {"header": {"N": c.N, "M": c.M, "KNB": c.KNB, "MAXM": c.MAXM, "H": c.H, "minc_hi": c.minc_hi,
                      "flags": c.flags, "as_top": c.as_top, "edit_E": c.edit_E, "n_docs": len(t.seqs)}}
    rnd = random.Random(7)
    blobs = [b"", b"a", b"hello", bytes(range(256)), "naïve".encode()]
    out["fnv"] = [[b.hex(), d.fnv1a64(b)] for b in blobs]
    ctxs = [[151645], [198, 151644], [1, 2, 3, 4, 5, 6], [rnd.randrange(151936) for _ in range(4)]]
    out["ctx_key"] = [[x, d.ctx_key(x)] for x in ctxs]
    out["prompt_words"] = [[s, [w.decode() for w in d.prompt_words(s)]] for s in TEXTS]

    ng = []
    for doc in rnd.sample(range(len(t.seqs)), 12):
        seq = d.TAIL + t.seqs[doc]
        for _ in range(6):
            i = rnd.randrange(1, len(seq))
            n = rnd.randrange(1, c.N + 1)
            if i - n < 0:
                continue
            ctx = seq[i - n:i]
            r = t.ng_get(tuple(ctx))
            ng.append([ctx, None if r is None else [r[0], [list(p) for p in r[1]]]])
    for _ in range(8):  # mostly misses
        ctx = [rnd.randrange(151936) for _ in range(rnd.randrange(1, c.N + 1))]
        r = t.ng_get(tuple(ctx))
        ng.append([ctx, None if r is None else [r[0], [list(p) for p in r[1]]]])
    out["ng"] = ng

    words = []
    for s in TEXTS:
        for w in d.prompt_words(s):
            v = t.vocab_get(w)
            asc = t.assoc_get(w)
            words.append([w.decode(), None if v is None else [v[0], len(v[1]), v[1][:8]],
                          None if not asc else [len(asc), [list(p) for p in asc[:5]]]])
    out["words"] = words
    docs = rnd.sample(range(len(t.seqs)), 5)
    out["seqs"] = [[j, len(t.seqs[j]), t.seqs[j][:10]] for j in docs]
    out["norms"] = [[j, t.norms[j]] for j in docs]
    W = t.W
    out["mlp"] = {"W1": sum(sum(r) for r in W["W1"]), "b1": sum(W["b1"]), "W2": sum(W["W2"]),
                  "b2": W["b2"], "WL": sum(W["WL"])}
    tf = getattr(t, "tflg", b"")
    nz = [i for i in range(len(tf)) if tf[i]]
    out["tflags"] = [[i, tf[i]] for i in (nz[:10] + rnd.sample(range(len(tf)), 10))] if tf else []
    with open(a.out, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(a.out, os.path.getsize(a.out), "bytes;", len(ng), "n-gram lookups,",
          sum(1 for x in ng if x[1] is not None), "hits")


if __name__ == "__main__":
    main()
