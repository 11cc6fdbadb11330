"""Acceptance / commit oracle (TEST INFRASTRUCTURE ONLY; see qwen_oracle.py for the import rule).

Restates, in plain Python:
* accept_tree          <- tools/draft/ildraft.py:750-759 (Python numbering: root -1, drafts 0..B-1)
* accept_chain         <- tools/draft/simulate.py:115-120 / Shaders.swift:322
* commit               <- Sources/Engine/Shaders.swift:281-365 (k_commit_spec, GPU numbering: root
                          row 0, drafts rows 1..n-1): argmax per row (lowest id on ties), tree walk
                          "first row whose parent is the current row and whose draft equals the
                          current row's argmax", token commit with EOS / max-steps stop, pos update,
                          KV compaction moves.
"""
from __future__ import annotations

from collections import defaultdict

import numpy as np


def accept_tree(parents, tokens, y, p):
    """Longest path from the root matching y[p], y[p+1], ...; returns its length (ildraft.py:750)."""
    children = defaultdict(dict)
    for i, (par, tok) in enumerate(zip(parents, tokens)):
        children[par].setdefault(tok, i)
    node, a = -1, 0
    while p + a < len(y) and y[p + a] in children[node]:
        node = children[node][y[p + a]]
        a += 1
    return a


def accept_chain(drafts, y, p):
    """Longest prefix of drafts equal to y[p:] (simulate.py:115-120)."""
    a = 0
    while a < len(drafts) and p + a < len(y) and drafts[a] == y[p + a]:
        a += 1
    return a


def argmax_lowest(logits: np.ndarray) -> int:
    """First maximum = lowest id on exact ties (qwen_ref.py:203, Shaders.swift:210)."""
    return int(np.argmax(logits))


def walk_tree(tree: dict, g) -> list:
    """Accepted rows (GPU numbering), Shaders.swift:311-320."""
    n = tree["n"]
    path, cur = [], 0
    while True:
        c = -1
        for i in range(1, n):
            if tree["parent"][i] == cur and tree["tok"][i] == g[cur]:
                c = i
                break
        if c < 0:
            return path
        path.append(c)
        cur = c


def commit(tree: dict, g, pos: int, step: int, maxsteps: int, eos=(151645, 151643)):
    """k_commit_spec's commit for a tree pass. Returns dict(tokens, path, pos, step, done, moves),
    moves = [(src_slot, dst_slot)] in the order the KV compaction applies them (Shaders.swift:351-365)."""
    path = walk_tree(tree, g)
    m = len(path)
    toks, done = [], False
    for i in range(m + 1):
        tok = int(g[0 if i == 0 else path[i - 1]])
        toks.append(tok)
        step += 1
        if tok in eos or step >= maxsteps:
            done = True
            break
    moves = [(pos + path[k - 1], pos + k) for k in range(1, m + 1) if path[k - 1] != k]
    return dict(tokens=toks, path=path, pos=pos + m + 1, step=step, done=done, moves=moves, m=m)


def to_python_numbering(tree: dict):
    """GPU tree (row 0 root) -> (parents, tokens) of ildraft.py (root -1, drafts 0..n-2)."""
    n = tree["n"]
    parents = [tree["parent"][i] - 1 for i in range(1, n)]
    tokens = [tree["tok"][i] for i in range(1, n)]
    return parents, tokens
