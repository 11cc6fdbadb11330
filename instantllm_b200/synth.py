"""Seeded synthetic inputs for the BASELINE configs: weights, prompts and draft trees.

No checkpoint or dataset is available, so every config runs on random-init weights of the
Qwen2.5-0.5B architecture in the reference's weight formats (standard layouts, see vpass.h):

* f32 (config 1, CPU only): N(0, 0.02).
* q4 (configs 2, 5): codes uniform 0..15, scale = f16(|N(0, 0.003)|), min = f16(-7.5 * scale)
  (centres the weights; the min distribution is not fixed by the config).
* q8 (config 3): codes uniform -127..127, scale = f16(|N(0, 0.0003)|) per group of 64.
* f16 (config 4): f16(N(0, 0.02)).
Norm gains are 1.0 and q/k/v biases N(0, 0.02) in every format. Each matrix draws from its own
PCG64 stream keyed by (seed, layer, matrix), so any subset regenerates identically.
"""
from __future__ import annotations

import numpy as np

HIDDEN, FFN, QKV_ROWS, VOCAB = 896, 4864, 1152, 151936
N_LAYERS = 24
PROMPT_VOCAB = 151643  # prompt ids uniform in [0, 151643): ordinary tokens, no specials
STOP_IDS = (151645, 151643)
TREE_INTS = 65

_MAT_IDS = {"embed": 0, "wqkv": 1, "wo": 2, "wgu": 3, "wd": 4, "bqkv": 5}


def _rng(seed: int, layer: int, name: str) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, layer + 1, _MAT_IDS[name]])))


def make_matrix(fmt: str, rows: int, cols: int, rng: np.random.Generator) -> dict:
    if fmt == "q4":
        codes = np.frombuffer(rng.bytes(rows * cols // 2), dtype=np.uint8).reshape(rows, cols // 2)
        s = np.abs(rng.normal(0.0, 0.003, size=(rows, cols // 64))).astype(np.float16)
        b = (-7.5 * s.astype(np.float32)).astype(np.float16)
        return {"fmt": "q4", "codes": codes, "scales": np.stack([s, b], axis=-1)}
    if fmt == "q8":
        codes = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
        s = np.abs(rng.normal(0.0, 0.0003, size=(rows, cols // 64))).astype(np.float16)
        return {"fmt": "q8", "codes": codes, "scales": s}
    if fmt == "q8g32":  # the reference's own q8: one scale per 32 columns (Convert.swift:254-282)
        codes = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
        s = np.abs(rng.normal(0.0, 0.0003, size=(rows, cols // 32))).astype(np.float16)
        return {"fmt": "q8g32", "codes": codes, "scales": s}
    if fmt == "f16":
        return {"fmt": "f16", "w": rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float16)}
    if fmt == "f32":
        return {"fmt": "f32", "w": rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)}
    raise ValueError(f"unknown format {fmt}")


def make_weights(fmt: str, n_layers: int = N_LAYERS, vocab: int = VOCAB, seed: int = 0) -> dict:
    """Synthetic weights in standard layouts: gate/up stacked as [gate; up], q/k/v as [q; k; v]."""
    layers = []
    for l in range(n_layers):
        layers.append({
            "wqkv": make_matrix(fmt, QKV_ROWS, HIDDEN, _rng(seed, l, "wqkv")),
            "bqkv": _rng(seed, l, "bqkv").normal(0.0, 0.02, size=QKV_ROWS).astype(np.float32),
            "wo": make_matrix(fmt, HIDDEN, HIDDEN, _rng(seed, l, "wo")),
            "wgu": make_matrix(fmt, 2 * FFN, HIDDEN, _rng(seed, l, "wgu")),
            "wd": make_matrix(fmt, HIDDEN, FFN, _rng(seed, l, "wd")),
            "ln1": np.ones(HIDDEN, np.float32),
            "ln2": np.ones(HIDDEN, np.float32),
        })
    return {
        "fmt": fmt,
        "n_layers": n_layers,
        "vocab": vocab,
        "embed": make_matrix(fmt, vocab, HIDDEN, _rng(seed, -1, "embed")),
        "final_norm": np.ones(HIDDEN, np.float32),
        "layers": layers,
    }


def weight_bytes(fmt: str, n_layers: int = N_LAYERS, vocab: int = VOCAB) -> int:
    """Algorithmic weight bytes one pass reads: codes + group scale data of every matrix, norms
    and biases (fp32), and the tied lm_head once. q4 full model: 278,139,392."""
    per = {"q4": lambda r, c: r * c // 2 + r * (c // 64) * 4,
           "q8": lambda r, c: r * c + r * (c // 64) * 2,
           "q8g32": lambda r, c: r * c + r * (c // 32) * 2,
           "f16": lambda r, c: r * c * 2}[fmt]
    layer = per(QKV_ROWS, HIDDEN) + per(HIDDEN, HIDDEN) + per(2 * FFN, HIDDEN) + per(HIDDEN, FFN)
    small = (2 * HIDDEN + QKV_ROWS) * 4
    return n_layers * (layer + small) + HIDDEN * 4 + per(vocab, HIDDEN)


def head_rows(embed: dict, final_norm: np.ndarray, rng: np.random.Generator, n: int,
              mix=(1.0, 0.93, 0.6)) -> np.ndarray:
    """Residual rows fp32 [n][896] for the tied lm_head with a clear winner and close runners-up, the
    shape of a trained model's logits: each row mixes a few rows of the q4 embedding (divided by
    the final norm) and adds noise. Random-init weights alone give flat logits."""
    V = embed["codes"].shape[0]
    s = embed["scales"][..., 0].astype(np.float32)
    b = embed["scales"][..., 1].astype(np.float32)
    x = np.zeros((n, HIDDEN), dtype=np.float32)
    for r in range(n):
        ids = rng.choice(V, size=len(mix), replace=False)
        for c, i in zip(mix, ids):
            q = np.empty(HIDDEN, dtype=np.float32)
            q[0::2], q[1::2] = embed["codes"][i] & 15, embed["codes"][i] >> 4
            x[r] += np.float32(c) * (q.reshape(-1, 64) * s[i][:, None] + b[i][:, None]).reshape(-1)
        x[r] /= final_norm
        x[r] += rng.normal(0, np.abs(x[r]).mean() * 0.5, HIDDEN).astype(np.float32)
    return x * np.float32(40.0)


def make_prompt(n: int, seed: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 7919])))
    return rng.integers(0, PROMPT_VOCAB, size=n, dtype=np.int64).astype(np.int32)


# ---------------------------------------------------------------------------------------------
# draft trees (buffer layout of Shaders.swift:23-30)


def tree_to_buffer(tree: dict) -> np.ndarray:
    buf = np.zeros(TREE_INTS, np.int32)
    n = tree["n"]
    buf[0] = n
    for i in range(n):
        buf[1 + i] = tree["depth"][i]
        buf[17 + i] = tree["parent"][i]
        buf[33 + i] = tree["tok"][i]
        # ancestor mask incl. the row itself; a malformed parent link only truncates the walk
        # (the device validates the tree and reports it)
        anc, cur = 1 << i, i
        for _ in range(16):
            par = tree["parent"][cur] if cur > 0 else -1
            if not 0 <= par < cur:
                break
            anc |= 1 << par
            cur = par
        buf[49 + i] = anc
    return buf


def chain_tree(drafts) -> dict:
    n = len(drafts) + 1
    return {"n": n, "depth": list(range(n)), "parent": [-1] + list(range(n - 1)),
            "tok": [0] + [int(d) for d in drafts]}


def root_tree() -> dict:
    """A 1-row pass: the sequential (no-draft) baseline through the same kernels."""
    return {"n": 1, "depth": [0], "parent": [-1], "tok": [0]}


def seeded_tree(rng: np.random.Generator, y, n: int = 16, max_depth: int = 8, p_match: float = 0.6,
                vocab: int = PROMPT_VOCAB) -> dict:
    """Best-first-style random tree of config 2: root + n-1 drafts. The parent of node i is uniform
    among earlier nodes of depth < max_depth. A node's draft is its parent's true argmax with
    probability p_match, else a uniform random id. `y[d]` is the true next token at depth d of the
    true path (from a prior sequential run); an off-path parent's "true argmax" is a random id drawn
    once for that parent."""
    depth, parent, tok = [0], [-1], [0]
    on_path = [True]
    truth = [int(y[0])]
    for i in range(1, n):
        cand = [j for j in range(i) if depth[j] < max_depth]
        p = int(cand[rng.integers(0, len(cand))])
        if rng.random() < p_match:
            t = truth[p]
        else:
            t = int(rng.integers(0, vocab))
        depth.append(depth[p] + 1)
        parent.append(p)
        tok.append(t)
        path_ok = on_path[p] and t == truth[p]
        on_path.append(path_ok)
        d = depth[-1]
        truth.append(int(y[d]) if (path_ok and d < len(y)) else int(rng.integers(0, vocab)))
    return {"n": n, "depth": depth, "parent": parent, "tok": tok}
