"""CPU oracle of the reference drafter: the checker of the CUDA drafter kernel (test infrastructure;
only tests/ may import it, never the product path).

Restates tools/draft/ildraft.py (the drafter's specification) on a table read by
instantllm_b200.draft_table.DraftTable:
  * Request.begin         Drafter.begin (ildraft.py:452-516): prompt ids, nearest training
                          documents and their suffix indexes, copy candidates, association map.
                          No tokenizer: the space variants and edited neighbours, which need one, are
                          empty (as in the reference without a tokenizer).
  * Request.features      Drafter.features (:519-692): the candidate tokens of the next position
                          after out and their 53 feature values, in float64.
  * score / Request.probs the scorer (:694-708): MLP + softmax with a null option, float64.
  * best_first_tree       Drafter.tree (:724-747).
The order of every step that decides a token, a probability or a tie is the reference's, because
the verify pass accepts what the drafter proposes: another order gives other trees.
"""
from __future__ import annotations

import heapq
import math

import numpy as np

from instantllm_b200.draft_table import (FLAG_ASSOC, FLAG_ASSOC_CANDS, N_FEATURES, STOPS, DraftTable, ctx_key,
                                         prompt_words)

TAIL = (151645, 198, 151644, 77091, 198)  # "<|im_end|>\n<|im_start|>assistant\n" (ildraft.py:54)
FENCE_OPEN = (73594, 13874)                # "```", "``" (:56)
TICK = 63                                  # "`" (:57)

FEATS = [  # ildraft.py:91-103
    "bias",
    "ng_p_long", "ng_top_long", "ng_ord_long", "ng_lcnt_long", "ng_p_supp3", "ng_p_supp10",
    "ng_p1", "ng_p2", "ng_p3", "ng_p4", "ng_p5", "ng_p6", "ng_rank2", "ng_rank3plus", "ng_ent_low",
    "sf_m", "sf_any", "sf_m_ge3",
    "pr_m", "pr_any", "pr_m_ge2", "pr_first",
    "nb_sum", "nb_msum", "nb_cnt", "nb_maxm", "nb_top1", "nb_top1_m",
    "is_stop", "in_prompt", "agree_ng_nb", "agree_sf_nb",
    "cp_prop", "cp_ctx1", "cp_ctx2", "cp_unused", "cp_first_unused", "cp_spacevar",
    "st_open_fence", "st_open_tick", "c_tick", "c_nl", "st_ticks_odd", "st_len", "c_repeat",
    "as_max", "as_cnt", "as_cand",
    "ed_sum", "ed_cnt", "ed_maxm", "ed_top1",
]
FI = {f: i for i, f in enumerate(FEATS)}
assert len(FEATS) == N_FEATURES


class OracleTable:
    """Dictionary views of a DraftTable for the checker (copy rates, token flags, associations)."""

    def __init__(self, t: DraftTable):
        self.t = t
        sec = t.sec
        self.prop = {int(a): float(b) for a, b in zip(sec[b"CPTK"]["token"], sec[b"CPTK"]["v"])} if b"CPTK" in sec else {}
        self.cc1 = {int(a): float(b) for a, b in zip(sec[b"CPC1"]["token"], sec[b"CPC1"]["v"])} if b"CPC1" in sec else {}
        self.cc2 = {(int(k) >> 32, int(k) & 0xFFFFFFFF): float(v) for k, v in zip(sec[b"CPC2"]["key"], sec[b"CPC2"]["v"])} \
            if b"CPC2" in sec else {}
        self.tflg = t.token_flags()
        m = t.mlp()
        self.W1, self.b1 = m["W1"].astype(np.float64), m["b1"].astype(np.float64)
        self.W2, self.b2, self.WL = m["W2"].astype(np.float64), float(m["b2"]), m["WL"].astype(np.float64)

    def tok_flag(self, x: int):
        """(backtick count, contains a newline) of token x (ildraft.py:237-243)."""
        v = int(self.tflg[x]) if 0 <= x < len(self.tflg) else 0
        return v & 7, bool(v & 8)


def suffix_index(seq, maxm: int) -> dict:
    """n-gram (1 <= n <= maxm) of seq -> index after its first occurrence that has a next token
    (ildraft.py:466-472)."""
    idx = {}
    L = len(seq)
    for n in range(1, maxm + 1):
        for i in range(0, L - n):
            k = tuple(seq[i:i + n])
            if k not in idx:
                idx[k] = i + n
    return idx


def score(ot: OracleTable, rows) -> np.ndarray:
    """The scorer's raw scores (ildraft.py:700-701): W2 . relu(W1 x + b1) + b2 + WL . x."""
    X = np.asarray(rows, dtype=np.float64)
    return np.maximum(X @ ot.W1.T + ot.b1, 0.0) @ ot.W2 + ot.b2 + X @ ot.WL


def softmax_null(s) -> np.ndarray:
    """Probabilities with a null option of score 0 (ildraft.py:702-705)."""
    m = max(float(np.max(s)), 0.0)
    e = np.exp(s - m)
    return e / (float(e.sum()) + math.exp(-m))


def probs_of_rows(ot: OracleTable, tokens, rows) -> list:
    """The scorer over given candidate feature rows (ildraft.py:694-708): [(token, p)] by p
    descending, then token ascending."""
    if len(tokens) == 0:
        return []
    ps = softmax_null(score(ot, rows))
    order = sorted(range(len(tokens)), key=lambda i: (-ps[i], int(tokens[i])))
    return [(int(tokens[i]), float(ps[i])) for i in order]


class Request:
    """The drafter's state of one request (ildraft.py Drafter, tokenizer absent)."""

    def __init__(self, ot: OracleTable, pids, text: str):
        t = ot.t
        self.ot, self.t = ot, t
        self.N, self.MAXM = t.N, t.MAXM
        self.P = [int(x) for x in pids]
        self.Pset = set(self.P)
        self.nb = []
        for s, j in t.neighbours(text):
            seq = list(TAIL) + t.seq(j)
            self.nb.append((s, seq, suffix_index(seq, t.MAXM)))
        self.ed = []  # edited neighbours need the tokenizer
        self.copy_cands = sorted(self.Pset)  # no space variants without the tokenizer
        self.as_map, as_cands = {}, []
        if t.flags & FLAG_ASSOC:
            for w in prompt_words(text):
                lst = t.assoc_get(w)
                if not lst:
                    continue
                for rank, (tok, ll) in enumerate(lst):
                    e = self.as_map.get(tok)
                    self.as_map[tok] = (max(e[0], ll), e[1] + 1) if e else (ll, 1)
                    if rank < t.as_top and (t.flags & FLAG_ASSOC_CANDS):
                        as_cands.append(tok)
        self.as_cands = sorted(set(as_cands))

    def features(self, out):
        """(sorted candidate tokens, their feature rows) for the position after out."""
        ot, t = self.ot, self.t
        ctx = list(TAIL) + list(out)
        L, Lo = len(ctx), len(out)
        cand = {}

        def row(tok):
            r = cand.get(tok)
            if r is None:
                r = [0.0] * N_FEATURES
                r[0] = 1.0
                cand[tok] = r
            return r

        dists = {}
        for n in range(min(self.N, L), 0, -1):
            e = t.ng_get(ctx[L - n:])
            if e is not None:
                dists[n] = e
        long_n = max(dists) if dists else 0
        supp3 = max((n for n, e in dists.items() if e[0] >= 3), default=0)
        supp10 = max((n for n, e in dists.items() if e[0] >= 10), default=0)
        for n, (tot, top) in dists.items():
            for rk, (tok, c) in enumerate(top):
                r = row(tok)
                if n == long_n:
                    if rk == 1:
                        r[FI["ng_rank2"]] = 1.0
                    elif rk >= 2:
                        r[FI["ng_rank3plus"]] = 1.0
        for n in range(min(self.MAXM, Lo - 1), 0, -1):  # self lookup: latest earlier occurrence
            pat = list(out[Lo - n:])
            hit = next((j + n for j in range(Lo - n - 1, -1, -1) if list(out[j:j + n]) == pat), -1)
            if hit >= 0:
                r = row(out[hit])
                r[FI["sf_m"]], r[FI["sf_any"]], r[FI["sf_m_ge3"]] = n / 4.0, 1.0, 1.0 if n >= 3 else 0.0
                break
        P = self.P
        for n in range(min(self.MAXM, Lo), 0, -1):  # prompt lookup: every occurrence
            pat = list(out[Lo - n:])
            occ = [j for j in range(0, len(P) - n) if P[j:j + n] == pat]
            if occ:
                for oi, j in enumerate(occ):
                    r = row(P[j + n])
                    r[FI["pr_m"]], r[FI["pr_any"]], r[FI["pr_m_ge2"]] = n / 4.0, 1.0, 1.0 if n >= 2 else 0.0
                    if oi == 0:
                        r[FI["pr_first"]] = 1.0
                break
        votes = {}
        for rank, (s, seq, idx) in enumerate(self.nb):
            for n in range(min(self.MAXM, L), 0, -1):
                j = idx.get(tuple(ctx[L - n:]))
                if j is not None:
                    votes.setdefault(seq[j], []).append((s, n, rank == 0))
                    break
        nnb = max(1, len(self.nb))
        for tok, vs in votes.items():
            r = row(tok)
            r[FI["nb_sum"]] = sum(s for s, _, _ in vs)
            r[FI["nb_msum"]] = sum(s * min(n, 8) / 8.0 for s, n, _ in vs)
            r[FI["nb_cnt"]] = len(vs) / nnb
            r[FI["nb_maxm"]] = max(min(n, 8) for _, n, _ in vs) / 8.0
            for s, n, first in vs:
                if first:
                    r[FI["nb_top1"]], r[FI["nb_top1_m"]] = 1.0, min(n, 8) / 8.0
        used = set(out)
        c1 = ot.cc1.get(ctx[-1], 0.1)
        c2 = ot.cc2.get((ctx[-2], ctx[-1]), 0.1)
        first_unused = next((x for x in P if x not in used and ot.prop.get(x, 0.2) > 0.3), -1)
        for x in self.copy_cands:
            r = row(x)
            inp = x in self.Pset
            pt = ot.prop.get(x, 0.2) if inp else 0.3
            r[FI["cp_prop"]] = math.log(pt / (1.0 - pt)) / 4.0
            r[FI["cp_ctx1"]], r[FI["cp_ctx2"]] = c1, c2
            r[FI["cp_unused"]] = 0.0 if x in used else 1.0
            r[FI["cp_first_unused"]] = 1.0 if x == first_unused else 0.0
            r[FI["cp_spacevar"]] = 0.0 if inp else 1.0
        for x in self.as_cands:
            row(x)[FI["as_cand"]] = 1.0
        open_fence = 1.0 if out and out[0] in FENCE_OPEN else 0.0
        open_tick = 1.0 if out and out[0] == TICK else 0.0
        ticks_odd = float(sum(ot.tok_flag(x)[0] for x in out) % 2)
        st_len = min(Lo, 32) / 32.0
        top_long, ent_low = None, False
        if long_n:
            tot, top = dists[long_n]
            top_long = top[0][0]
            ent_low = -sum((c / tot) * math.log(c / tot) for _, c in top) < 0.3
        for tok, r in cand.items():
            for n, (tot, top) in dists.items():
                c = next((cc for tk, cc in top if tk == tok), 0)
                if c:
                    p = c / tot
                    r[FI["ng_p%d" % n]] = p if n <= 6 else 0.0
                    if n == long_n:
                        r[FI["ng_p_long"]], r[FI["ng_ord_long"]], r[FI["ng_lcnt_long"]] = p, n / 6.0 * p, math.log1p(c)
                    if n == supp3:
                        r[FI["ng_p_supp3"]] = p
                    if n == supp10:
                        r[FI["ng_p_supp10"]] = p
            if tok == top_long:
                r[FI["ng_top_long"]] = 1.0
                if ent_low:
                    r[FI["ng_ent_low"]] = 1.0
            r[FI["is_stop"]] = 1.0 if tok in STOPS else 0.0
            r[FI["in_prompt"]] = 1.0 if tok in self.Pset else 0.0
            r[FI["agree_ng_nb"]] = r[FI["ng_top_long"]] * min(1.0, 2.0 * r[FI["nb_cnt"]])
            r[FI["agree_sf_nb"]] = r[FI["sf_any"]] * min(1.0, 2.0 * r[FI["nb_cnt"]])
            nt, nl = ot.tok_flag(tok)
            r[FI["st_open_fence"]], r[FI["st_open_tick"]] = open_fence, open_tick
            r[FI["c_tick"]], r[FI["c_nl"]] = 1.0 if nt > 0 else 0.0, 1.0 if nl else 0.0
            r[FI["st_ticks_odd"]], r[FI["st_len"]] = ticks_odd, st_len
            r[FI["c_repeat"]] = 1.0 if tok in used else 0.0
            ae = self.as_map.get(tok)
            if ae is not None:
                r[FI["as_max"]], r[FI["as_cnt"]] = ae[0] / 4.0, min(ae[1], 4) / 4.0
        toks = sorted(cand)
        return toks, [cand[x] for x in toks]

    def probs(self, out):
        """[(token, p)] by p descending, then token ascending (null option excluded)."""
        toks, rows = self.features(out)
        if not toks:
            return []
        ps = softmax_null(score(self.ot, rows))
        order = sorted(range(len(toks)), key=lambda i: (-ps[i], toks[i]))
        return [(toks[i], float(ps[i])) for i in order]

    def tree(self, out, B: int, branch: int = 8):
        return best_first_tree(lambda path: self.probs(list(out) + list(path)), B, branch)


def best_first_tree(probs, B: int, branch: int = 8, stops=STOPS) -> tuple:
    """The draft tree of B nodes grown best first (ildraft.py:724-747): every candidate of a node
    (the top `branch` of probs(path), path = the tokens from the root to that node) waits in a
    priority queue keyed by its path probability, the product of the probabilities along the path;
    the most probable waiting candidate becomes the next node (equal keys: the one queued first),
    and its own candidates are queued unless it is a stop token. Returns (parents, tokens): node i
    hangs under node parents[i] (-1: the root, the last accepted token), so parents[i] < i."""
    parents, tokens, path = [], [], {-1: []}
    queue, seq = [], 0
    for tok, p in probs([])[:branch]:
        heapq.heappush(queue, (-p, seq, -1, tok))
        seq += 1
    while queue and len(tokens) < B:
        key, _, par, tok = heapq.heappop(queue)
        node = len(tokens)
        parents.append(par)
        tokens.append(tok)
        path[node] = path[par] + [tok]
        if tok in stops or len(tokens) >= B:
            continue
        for tok2, p2 in probs(path[node])[:branch]:
            heapq.heappush(queue, (key * p2, seq, node, tok2))
            seq += 1
    return parents, tokens
