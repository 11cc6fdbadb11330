"""CPU restatement of the reference's two-stage sketch lm_head. TEST INFRASTRUCTURE: only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline may use it, as the checker of the CUDA path.

Follows Sources/Engine/Shaders.swift:
  * q4_chunk_norm (:1022-1042): the row is RMS-normed with the final norm in fp32, then rounded to
    fp16 (the values every later dot product sees);
  * k_lmh_sketch_T (:1386-1447): the sketch estimate A = sum_g s_g (4 <hi_g, x_g> + 1.5 X_g) + b_g X_g
    of each vocabulary row from the high two bits of its q4 codes, sigma^2 = 1.25 sum_g s_g^2 |x_g|^2,
    and per 32-row group the max of A - K sigma and of A + K sigma;
  * k_lmh_tau (:1450-1471): tau[t] = max over groups of the lower bound;
  * k_lmh_exact_T (:1474-1513): exact q4 logits in the groups whose upper bound reaches tau[t],
    -inf elsewhere, argmax with the lowest id on ties.
The reference sums the sketch dot products in fp16 (its `half acc`); here they are fp32, so the
restatement is the algorithm's intended value and the CUDA path is compared to it with a tolerance.
Parity of the tokens is exact: they are checked against the full lm_head's.

Pinned by: the sketch byte layout of Convert.swift:150-158 (checked against convert.sketch_q4) and
by the bound property itself (exact logits within K sigma of the estimate).
"""
from __future__ import annotations

import numpy as np

H = 896
GS = 64
GROUP = 32
EPS = 1e-6


def unpack_hi(hi: np.ndarray) -> np.ndarray:
    """Sketch plane uint8 [V][224] -> high code bits uint8 [V][896] (byte c: codes 4c .. 4c + 3,
    code 4c in bits 0-1)."""
    hi = np.asarray(hi, dtype=np.uint8)
    out = np.empty((hi.shape[0], hi.shape[1], 4), dtype=np.uint8)
    for i in range(4):
        out[..., i] = (hi >> (2 * i)) & 3
    return out.reshape(hi.shape[0], -1)


def unpack_q4(codes: np.ndarray) -> np.ndarray:
    """q4 codes uint8 [V][448] (column 2j in the low nibble) -> uint8 [V][896]."""
    codes = np.asarray(codes, dtype=np.uint8)
    out = np.empty((codes.shape[0], codes.shape[1], 2), dtype=np.uint8)
    out[..., 0], out[..., 1] = codes & 15, codes >> 4
    return out.reshape(codes.shape[0], -1)


def normed_half(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """q4_chunk_norm: fp16(x * rsqrt(mean(x^2) + eps) * w) as fp32 [T][896]."""
    x = np.asarray(x, dtype=np.float32)
    ss = (x * x).sum(-1, keepdims=True, dtype=np.float32)
    scale = (1.0 / np.sqrt(ss / np.float32(H) + np.float32(EPS))).astype(np.float32)
    return (x * scale * np.asarray(w, dtype=np.float32)).astype(np.float16).astype(np.float32)


def _per_group(c: np.ndarray, xh: np.ndarray) -> np.ndarray:
    """dot[t][v][g] = <c[v, group g], xh[t, group g]> in fp32 (codes exact)."""
    V, T = c.shape[0], xh.shape[0]
    cg = c.reshape(V, H // GS, GS).astype(np.float32)
    xg = xh.reshape(T, H // GS, GS)
    out = np.empty((T, V, H // GS), dtype=np.float32)
    for g in range(H // GS):
        out[:, :, g] = (cg[:, g, :] @ xg[:, g, :].T).T
    return out


def sketch_scores(hi: np.ndarray, scales: np.ndarray, xh: np.ndarray) -> tuple:
    """(A, sigma) fp32 [T][V] of k_lmh_sketch_T for normed fp16 rows xh [T][896]."""
    s = np.asarray(scales[..., 0], dtype=np.float32)[None]  # [1][V][14]
    b = np.asarray(scales[..., 1], dtype=np.float32)[None]
    X = xh.reshape(xh.shape[0], H // GS, GS).sum(-1)[:, None, :]  # [T][1][14]
    XX = (xh * xh).reshape(xh.shape[0], H // GS, GS).sum(-1)[:, None, :]
    dot = _per_group(unpack_hi(hi), xh)
    A = (s * (4.0 * dot + 1.5 * X) + b * X).sum(-1, dtype=np.float32)
    var = 1.25 * (s * s * XX).sum(-1, dtype=np.float32)
    return A.astype(np.float32), np.sqrt(var).astype(np.float32)


def exact_logits(codes: np.ndarray, scales: np.ndarray, xh: np.ndarray) -> np.ndarray:
    """Exact q4 logits fp32 [T][V] of the normed rows (q_rows: sum_g s_g <q_g, x_g> + b_g X_g)."""
    s = np.asarray(scales[..., 0], dtype=np.float32)[None]
    b = np.asarray(scales[..., 1], dtype=np.float32)[None]
    X = xh.reshape(xh.shape[0], H // GS, GS).sum(-1)[:, None, :]
    dot = _per_group(unpack_q4(codes), xh)
    return (s * dot + b * X).sum(-1, dtype=np.float32)


def group_max(v: np.ndarray) -> np.ndarray:
    """Max over 32-row groups of the last axis (a ragged last group keeps its rows)."""
    T, V = v.shape
    ng = (V + GROUP - 1) // GROUP
    pad = np.full((T, ng * GROUP), -np.inf, dtype=np.float32)
    pad[:, :V] = v
    return pad.reshape(T, ng, GROUP).max(-1)


def sketch_head(codes, scales, hi, final_norm, x, k: float = 6.0) -> dict:
    """The whole two-stage head on residual rows x [T][896]. Returns tokens (int [T]), the group
    bounds lb / ub [T][ngrp], tau [T], the candidate mask [T][ngrp], and the full (exact) argmax."""
    xh = normed_half(x, final_norm)
    A, sig = sketch_scores(hi, scales, xh)
    lb, ub = group_max(A - np.float32(k) * sig), group_max(A + np.float32(k) * sig)
    tau = lb.max(-1)
    cand = ub >= tau[:, None]
    logits = exact_logits(codes, scales, xh)
    V = logits.shape[1]
    masked = np.where(np.repeat(cand, GROUP, axis=1)[:, :V], logits, -np.inf)
    return {"tokens": masked.argmax(-1), "full": logits.argmax(-1), "lb": lb, "ub": ub, "tau": tau,
            "cand": cand, "A": A, "sigma": sig, "logits": logits}
