"""A small ILDRAFT1 table holding exactly the entries of the reference's shipped drafter table
(tools/draft/ildraft-q4.bin) that the golden drafter cases (make_drafter_golden.py) read.

The reference drafter (tools/draft/ildraft.py) runs the golden cases on the full table with every
lookup recorded: the n-gram contexts, prompt words, associations, copy rates and token flags it
found, the document norms and training sequences it read. The subset keeps those entries (lookups
that missed still miss), renumbers the documents in ascending order (so score ties still resolve
the same way), and is checked by running the same cases on it: the result must equal the golden file
made from the full table. The GPU drafter tests read this file, so the reference's 5 MB table does
not have to travel with them.

Usage: python tests/golden/make_draft_subset.py --reference <instantllm checkout> \
           [--out tests/golden/draft_subset.ildraft]
"""
import argparse
import json
import os
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


class RecDict(dict):
    """A dict that records the keys its get() found."""

    def __init__(self, d):
        super().__init__(d)
        self.hits = set()

    def get(self, k, default=None):
        if dict.__contains__(self, k):
            self.hits.add(k)
        return dict.get(self, k, default)


class RecList(list):
    def __init__(self, d):
        super().__init__(d)
        self.hits = set()

    def __getitem__(self, i):
        self.hits.add(i)
        return list.__getitem__(self, i)


class RecBytes:
    def __init__(self, b):
        self.b, self.hits = b, set()

    def __len__(self):
        return len(self.b)

    def __getitem__(self, i):
        self.hits.add(i)
        return self.b[i]


def write_table(path, t, ng, words, norms_docs, seq_docs, prop, cc1, cc2, assoc, flags_tok):
    """An ILDRAFT1 v1 file (ildraft.py FORMAT) with the given entries of the loaded table t."""
    cfg = t.cfg
    docs = sorted(norms_docs)
    new = {j: i for i, j in enumerate(docs)}
    secs = []

    def add(tag, count, data):
        secs.append((tag, count, data))

    keys = sorted(ng)
    nx, vals = [], []
    for k in keys:
        tot, top = t.ngk[k]
        vals.append(struct.pack("<II", tot, (len(nx) << 3) | len(top)))
        nx += top
    add(b"NGKY", len(keys), b"".join(struct.pack("<Q", k) for k in keys))
    add(b"NGVL", len(vals), b"".join(vals))
    add(b"NGNX", len(nx), b"".join(struct.pack("<II", a, b) for a, b in nx))
    wk = sorted(words)
    post, wv = [], []
    for h in wk:
        idf, plist = t.vocabk[h]
        wv.append(struct.pack("<fII", idf, len(post), len(plist)))
        post += [new[j] for j in plist]
    add(b"WDKY", len(wk), b"".join(struct.pack("<Q", h) for h in wk))
    add(b"WDVL", len(wv), b"".join(wv))
    add(b"POST", len(post), b"".join(struct.pack("<I", j) for j in post))
    add(b"DNRM", len(docs), b"".join(struct.pack("<f", t.norms.b[j] if hasattr(t.norms, "b") else list.__getitem__(t.norms, j)) for j in docs))
    offs, toks = [0], []
    for j in docs:
        if j in seq_docs:
            toks += list.__getitem__(t.seqs, j)
        offs.append(len(toks))
    add(b"SQOF", len(offs), b"".join(struct.pack("<I", o) for o in offs))
    add(b"SQTK", len(toks), b"".join(struct.pack("<I", x) for x in toks))
    add(b"CPTK", len(prop), b"".join(struct.pack("<If", k, dict.get(t.prop, k)) for k in sorted(prop)))
    add(b"CPC1", len(cc1), b"".join(struct.pack("<If", k, dict.get(t.cc1, k)) for k in sorted(cc1)))
    c2 = sorted(((a << 32) | b, dict.get(t.cc2, (a, b))) for a, b in cc2)
    add(b"CPC2", len(c2), b"".join(struct.pack("<QfI", k, v, 0) for k, v in c2))
    ak = sorted(assoc)
    at, av = [], []
    for h in ak:
        lst = dict.get(t.assock, h)
        av.append(struct.pack("<II", len(at), len(lst)))
        at += lst
    add(b"ASWK", len(ak), b"".join(struct.pack("<Q", h) for h in ak))
    add(b"ASWV", len(av), b"".join(av))
    add(b"ASTK", len(at), b"".join(struct.pack("<If", a, b) for a, b in at))
    fl = sorted((x, t.tflg.b[x]) for x in flags_tok if t.tflg.b[x])
    add(b"TFLS", len(fl), b"".join(struct.pack("<II", x, v) for x, v in fl))
    W = t.W
    mlp = [v for row in W["W1"] for v in row] + list(W["b1"]) + list(W["W2"]) + [W["b2"]] + list(W["WL"])
    add(b"MLP0", len(mlp), b"".join(struct.pack("<f", v) for v in mlp))
    head = struct.pack("<8sII" + "I" * 8 + "IIII", b"ILDRAFT1", 1, len(secs), cfg.N, cfg.M, cfg.KNB, cfg.MAXM,
                       len(W["WL"]), cfg.H, cfg.minc_hi, len(docs), cfg.flags, cfg.as_top, cfg.edit_E, 0)
    start = 64 + 16 * len(secs)
    start += (-start) % 8
    body, dirs = b"", b""
    for tag, count, data in secs:
        body += b"\0" * ((-(start + len(body))) % 8)
        dirs += struct.pack("<4sIQ", tag, count, start + len(body))
        body += data
    raw = head + dirs
    raw += b"\0" * (start - len(raw))
    with open(path, "wb") as f:
        f.write(raw + body)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "draft_subset.ildraft"))
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.reference, "tools", "draft"))
    sys.path.insert(0, HERE)
    import ildraft as d
    from make_drafter_golden import golden_cases

    t = d.Tables.load(os.path.join(a.reference, "tools", "draft", "ildraft-q4.bin"))
    t.ngk, t.vocabk, t.prop = RecDict(t.ngk), RecDict(t.vocabk), RecDict(t.prop)
    t.cc1, t.cc2, t.assock = RecDict(t.cc1), RecDict(t.cc2), RecDict(t.assock)
    t.norms, t.seqs, t.tflg = RecList(t.norms), RecList(t.seqs), RecBytes(t.tflg)
    full = golden_cases(d, t)
    # every document of a recorded word's postings keeps its norm (the TF-IDF ranking reads them)
    norms_docs = set(j for h in t.vocabk.hits for j in dict.get(t.vocabk, h)[1])
    assert t.norms.hits <= norms_docs and t.seqs.hits <= norms_docs
    write_table(a.out, t, t.ngk.hits, t.vocabk.hits, norms_docs, t.seqs.hits, t.prop.hits, t.cc1.hits,
                t.cc2.hits, t.assock.hits, t.tflg.hits)
    sub = golden_cases(d, d.Tables.load(a.out))
    gold = json.load(open(os.path.join(HERE, "drafter_trees.json")))
    assert json.loads(json.dumps(sub)) == gold == json.loads(json.dumps(full)), "subset differs from the full table"
    print(a.out, os.path.getsize(a.out), "bytes; the golden cases reproduce on it")


if __name__ == "__main__":
    main()
