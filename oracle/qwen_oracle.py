"""CPU oracle for the verification pass (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may import this
module, and only as the checker or as the timed CPU baseline: the product path (instantllm_b200)
never calls it, and fails loudly when its CUDA library is missing.

A numpy restatement of the reference's fp32 CPU model, tools/reference/qwen_ref.py (instantllm),
generalised from causal prompt processing to the rows of a tree-verify pass:

* rmsnorm                   <- qwen_ref.py:72-74
* rotate_half / rope tables <- qwen_ref.py:77-78, 107-116 (angles in float64, cos/sin rounded once)
* layer math                <- qwen_ref.py:129-194 (q/k/v bias, GQA head h -> kv head h // 7,
                               scores * 0.125, exact softmax, SiLU(gate) * up, tied lm_head)
* greedy decoding           <- qwen_ref.py:196-220 (argmax = lowest id on exact ties)
* tree attention            <- Sources/Engine/Shaders.swift:893-958: row i attends to the cached
                               prefix then its ancestors in depth order; rotated as pos + depth,
                               its K/V written at slot pos + i.

Weights are injected as fp32 arrays (q4/q8/f16 weights are dequantised exactly, w = s*q + b in
fp32), so differences from the GPU path are activation rounding only. The restatement is pinned
against qwen_ref itself by tests/golden (fixtures made by importing the reference, see
tests/golden/make_golden.py).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from types import SimpleNamespace

import numpy as np

HIDDEN = 896
N_HEAD = 14
N_KV = 2
GROUP = N_HEAD // N_KV
HEAD_DIM = 64
HALF = HEAD_DIM // 2
RMS_EPS = 1e-6
ROPE_THETA = 1_000_000.0
ATTN_SCALE = HEAD_DIM ** -0.5


def rmsnorm(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """qwen_ref.py:72-74."""
    var = np.mean(x * x, axis=-1, keepdims=True)
    return (x * (1.0 / np.sqrt(var + RMS_EPS))) * w


def rotate_half(x: np.ndarray) -> np.ndarray:
    """qwen_ref.py:77-78 (pairs (i, i+32) of each head)."""
    return np.concatenate([-x[..., HALF:], x[..., :HALF]], axis=-1)


INV_FREQ = 1.0 / ROPE_THETA ** (np.arange(0, HEAD_DIM, 2, dtype=np.float64) / HEAD_DIM)


def rope_tables(positions, dtype=np.float32):
    """cos/sin [n, 64] for arbitrary positions (qwen_ref.py:112-116 with explicit positions)."""
    ang = np.asarray(positions, dtype=np.float64)[:, None] * INV_FREQ[None, :]
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(dtype), np.sin(ang).astype(dtype)


# ---------------------------------------------------------------------------------------------
# weights


def dequant(m: dict) -> np.ndarray:
    """Standard-layout matrix -> fp32 [rows, cols].

    q4: codes uint8 [R, C/2] (weight 2j in the low nibble of byte j, Convert.swift:317),
        scales float16 [R, C/64, 2] = (scale, min); w = scale * q + min (Convert.swift:290-317).
    q8: codes int8 [R, C], scales float16 [R, C/64]; w = scale * q (group 64 as BASELINE config 3).
    q8g32: codes int8 [R, C], scales float16 [R, C/32]; w = scale * q (group 32, the reference's
        quantizeQ8 layout, Convert.swift:254-282).
    f16 / f32: dense.
    """
    fmt = m["fmt"]
    if fmt in ("f16", "f32"):
        return np.asarray(m["w"], dtype=np.float32)
    codes = m["codes"]
    if fmt == "q4":
        R, half = codes.shape
        q = np.empty((R, half * 2), dtype=np.float32)
        q[:, 0::2] = codes & 15
        q[:, 1::2] = codes >> 4
        s = m["scales"][..., 0].astype(np.float32)
        b = m["scales"][..., 1].astype(np.float32)
        G = s.shape[1]
        q = q.reshape(R, G, 64)
        return (q * s[:, :, None] + b[:, :, None]).reshape(R, G * 64)
    if fmt in ("q8", "q8g32"):
        R, C = codes.shape
        s = m["scales"].astype(np.float32)
        G = s.shape[1]
        return (codes.astype(np.float32).reshape(R, G, C // G) * s[:, :, None]).reshape(R, C)
    raise ValueError(fmt)


@dataclass
class Model:
    """fp32 weights in the attribute layout of qwen_ref.Qwen2Ref (qwen_ref.py:88-104)."""

    embed: np.ndarray
    norm: np.ndarray
    layers: list = field(default_factory=list)

    @property
    def vocab(self) -> int:
        return self.embed.shape[0]


def model_from_weights(w: dict) -> Model:
    """Dequantise a synthetic weight set (instantllm_b200.synth layout) into an fp32 Model."""
    layers = []
    for L in w["layers"]:
        wqkv = dequant(L["wqkv"])
        wgu = dequant(L["wgu"])
        F = wgu.shape[0] // 2
        layers.append(SimpleNamespace(
            ln1=L["ln1"].astype(np.float32), ln2=L["ln2"].astype(np.float32),
            wq=wqkv[:HIDDEN], wk=wqkv[HIDDEN:HIDDEN + 128], wv=wqkv[HIDDEN + 128:],
            bq=L["bqkv"][:HIDDEN].astype(np.float32), bk=L["bqkv"][HIDDEN:HIDDEN + 128].astype(np.float32),
            bv=L["bqkv"][HIDDEN + 128:].astype(np.float32),
            wo=dequant(L["wo"]), wg=wgu[:F], wu=wgu[F:], wd=dequant(L["wd"]),
        ))
    return Model(embed=dequant(w["embed"]), norm=w["final_norm"].astype(np.float32), layers=layers)


# ---------------------------------------------------------------------------------------------
# forward over arbitrary rows


class KVCache:
    """Per layer K and V [kv_heads, max_len, 64] (qwen_ref.py:81-85)."""

    def __init__(self, n_layers: int, max_len: int, dtype=np.float32):
        self.k = [np.zeros((N_KV, max_len, HEAD_DIM), dtype) for _ in range(n_layers)]
        self.v = [np.zeros((N_KV, max_len, HEAD_DIM), dtype) for _ in range(n_layers)]

    def copy(self) -> "KVCache":
        c = KVCache.__new__(KVCache)
        c.k = [a.copy() for a in self.k]
        c.v = [a.copy() for a in self.v]
        return c


def forward_rows(model: Model, cache: KVCache, tokens, rope_pos, slots, attend, all_logits=True):
    """Run rows through the model.

    tokens[i]   token of row i
    rope_pos[i] position its q and k are rotated by
    slots[i]    KV slot its k and v are written to
    attend[i]   KV slots row i attends to, in order (its own slot last)
    Returns fp32 logits [n, V] (or of the last row only).
    """
    tokens = np.asarray(tokens, dtype=np.int64)
    n = tokens.shape[0]
    cos, sin = rope_tables(rope_pos)
    cos, sin = cos[:, None, :], sin[:, None, :]
    slots = np.asarray(slots, dtype=np.int64)
    x = model.embed[tokens]
    for li, L in enumerate(model.layers):
        h = rmsnorm(x, L.ln1)
        q = (h @ L.wq.T + L.bq).reshape(n, N_HEAD, HEAD_DIM)
        k = (h @ L.wk.T + L.bk).reshape(n, N_KV, HEAD_DIM)
        v = (h @ L.wv.T + L.bv).reshape(n, N_KV, HEAD_DIM)
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
        cache.k[li][:, slots] = k.transpose(1, 0, 2)
        cache.v[li][:, slots] = v.transpose(1, 0, 2)
        o = np.empty((n, N_HEAD, HEAD_DIM), dtype=np.float32)
        for r in range(n):
            sl = np.asarray(attend[r], dtype=np.int64)
            K = cache.k[li][:, sl]  # [kv, L, 64]
            V = cache.v[li][:, sl]
            qg = q[r].reshape(N_KV, GROUP, HEAD_DIM)
            s = np.matmul(qg, K.transpose(0, 2, 1)) * ATTN_SCALE  # [kv, g, L]
            s = s - s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p = p / p.sum(axis=-1, keepdims=True)
            o[r] = np.matmul(p, V).reshape(N_HEAD, HEAD_DIM)
        x = x + o.reshape(n, HIDDEN) @ L.wo.T
        h2 = rmsnorm(x, L.ln2)
        g = h2 @ L.wg.T
        u = h2 @ L.wu.T
        with np.errstate(over="ignore"):
            act = (g / (1.0 + np.exp(-g))) * u
        x = x + act @ L.wd.T
    if not all_logits:
        x = x[-1:]
    xf = rmsnorm(x, model.norm)
    return xf @ model.embed.T


def forward_causal(model: Model, cache: KVCache, tokens, pos0: int, all_logits=False):
    """Causal rows at slots/positions pos0.. (qwen_ref.Qwen2Ref.forward, qwen_ref.py:118-194).
    Returns logits [n, V] if all_logits else [V] of the last row."""
    n = len(tokens)
    pos = np.arange(pos0, pos0 + n)
    attend = [np.arange(0, p + 1) for p in pos]
    lg = forward_rows(model, cache, tokens, pos, pos, attend, all_logits=all_logits)
    return lg if all_logits else lg[0]


def greedy(model: Model, prompt, max_new: int, stop_ids=(151645, 151643), max_len=None):
    """Greedy decoding with 1-row steps (qwen_ref.py:196-220). Returns (ids incl. a stop token if
    sampled, cache, logits of every step [steps, V])."""
    max_len = max_len or len(prompt) + max_new + 1
    cache = KVCache(len(model.layers), max_len)
    logits = forward_causal(model, cache, prompt, 0)
    out, steps = [], [logits]
    pos = len(prompt)
    for _ in range(max_new):
        tok = int(np.argmax(logits))
        out.append(tok)
        if tok in stop_ids or len(out) == max_new:
            break
        logits = forward_causal(model, cache, [tok], pos)
        steps.append(logits)
        pos += 1
    return out, cache, np.stack(steps)


# ---------------------------------------------------------------------------------------------
# tree pass


def tree_rows(tree: dict, pos: int):
    """Geometry of a tree pass (Shaders.swift:23-30, 893-923): per row its rope position, KV slot and
    attended slots (prefix, then ancestors in depth order)."""
    n = tree["n"]
    depth, parent = tree["depth"], tree["parent"]
    rope_pos, slots, attend = [], [], []
    for i in range(n):
        path = [i]
        while path[-1] != 0:
            path.append(parent[path[-1]])
        path = path[::-1]
        assert len(path) == depth[i] + 1
        rope_pos.append(pos + depth[i])
        slots.append(pos + i)
        attend.append(np.concatenate([np.arange(pos), pos + np.asarray(path)]))
    return rope_pos, slots, attend


def tree_pass(model: Model, cache: KVCache, pos: int, last_token: int, tree: dict):
    """Logits [n, V] of a verify pass over `tree` whose root is `last_token` at slot `pos`."""
    toks = [last_token] + list(tree["tok"][1:tree["n"]])
    rope_pos, slots, attend = tree_rows(tree, pos)
    return forward_rows(model, cache, toks, rope_pos, slots, attend)
