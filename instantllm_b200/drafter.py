"""The learned drafter on the device (k_draft, csrc/vp_draft.cuh) and its request context.

Mirrors the reference's ILDraft.swift on the host side: the ILDRAFT1 table is handed to the library
once (vp_drafter_create); at request start the host builds the request context of Drafter.begin
(tools/draft/ildraft.py:452-516): the prompt ids, their sorted distinct ids (the copy candidates;
space variants need a tokenizer and are not built, as when the reference runs without one), the
nearest training documents by TF-IDF (draft_table.DraftTable.neighbours) with each document's
sequence (the assistant tail + its output) and the sorted keys of its n-grams, and the association
map. Every per-step part (candidates, features, scorer, the best-first tree) runs on the GPU.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib
from .draft_table import FLAG_ASSOC, FLAG_ASSOC_CANDS, DraftTable, prompt_words

TAIL = (151645, 198, 151644, 77091, 198)  # "<|im_end|>\n<|im_start|>assistant\n"
FNV_OFF = np.uint64(0xCBF29CE484222325)
FNV_PRIME = np.uint64(0x100000001B3)


def ngram_index(seq, maxm: int):
    """Sorted keys of the n-grams (1 <= n <= maxm) of seq that have a next token, and for each the
    index after its first occurrence (ildraft.py:466-472); keys are FNV-1a 64 over the order byte
    then the tokens as u32 little-endian (the n-gram context key)."""
    s = np.asarray(seq, dtype=np.uint32)
    L = len(s)
    keys, pos = [], []
    for n in range(1, maxm + 1):
        m = L - n  # starts i = 0 .. L - n - 1
        if m <= 0:
            break
        h = np.full(m, FNV_OFF, dtype=np.uint64)
        with np.errstate(over="ignore"):
            h = (h ^ np.uint64(n)) * FNV_PRIME
            for k in range(n):
                t = s[k:k + m].astype(np.uint64)
                for b in range(4):
                    h = (h ^ ((t >> np.uint64(8 * b)) & np.uint64(0xFF))) * FNV_PRIME
        u, first = np.unique(h, return_index=True)  # first occurrence of each key
        keys.append(u)
        pos.append(first.astype(np.int32) + n)
    if not keys:
        return np.zeros(0, np.uint64), np.zeros(0, np.int32)
    k = np.concatenate(keys)
    p = np.concatenate(pos)
    o = np.argsort(k, kind="stable")
    return k[o], p[o]


class _Request(ctypes.Structure):
    _P = ctypes.c_void_p
    _fields_ = [("n_prompt", ctypes.c_int32), ("prompt", _P), ("n_copy", ctypes.c_int32), ("copy", _P),
                ("n_nb", ctypes.c_int32), ("nb_score", _P), ("nb_seq_off", _P), ("nb_seq", _P),
                ("nb_key_off", _P), ("nb_keys", _P), ("nb_pos", _P), ("n_as", ctypes.c_int32),
                ("as_tok", _P), ("as_max", _P), ("as_cnt", _P), ("n_as_cand", ctypes.c_int32), ("as_cand", _P)]


class _Debug(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("parents", "tokens", "exp_tokens", "exp_probs", "status")]


def request_context(t: DraftTable, pids, text: str) -> dict:
    """Drafter.begin's request context as flat arrays (host)."""
    P = np.asarray(pids, dtype=np.int32)
    nb = t.neighbours(text)
    seqs, keys, poss = [], [], []
    for _, j in nb:
        seq = np.asarray(list(TAIL) + t.seq(j), dtype=np.int32)
        k, p = ngram_index(seq, t.MAXM)
        seqs.append(seq)
        keys.append(k)
        poss.append(p)
    as_map, as_cands = {}, set()
    if t.flags & FLAG_ASSOC:
        for w in prompt_words(text):
            lst = t.assoc_get(w)
            if not lst:
                continue
            for rank, (tok, ll) in enumerate(lst):
                e = as_map.get(tok)
                as_map[tok] = (max(e[0], ll), e[1] + 1) if e else (ll, 1)
                if rank < t.as_top and (t.flags & FLAG_ASSOC_CANDS):
                    as_cands.add(tok)
    at = sorted(as_map)

    def offs(parts):
        return np.concatenate([[0], np.cumsum([len(x) for x in parts])]).astype(np.int32)

    return {
        "prompt": P, "copy": np.unique(P).astype(np.int32),
        "nb_score": np.asarray([s for s, _ in nb], dtype=np.float64),
        "nb_seq_off": offs(seqs), "nb_seq": np.concatenate(seqs) if seqs else np.zeros(0, np.int32),
        "nb_key_off": offs(keys), "nb_keys": np.concatenate(keys) if keys else np.zeros(0, np.uint64),
        "nb_pos": np.concatenate(poss) if poss else np.zeros(0, np.int32),
        "as_tok": np.asarray(at, dtype=np.int32), "as_max": np.asarray([as_map[x][0] for x in at], dtype=np.float64),
        "as_cnt": np.asarray([as_map[x][1] for x in at], dtype=np.int32),
        "as_cand": np.asarray(sorted(as_cands), dtype=np.int32),
    }


class DeviceDrafter:
    """The drafter's table on one GPU and the current request's context."""

    def __init__(self, table_path: str, device: int = 0):
        self.lib = _lib.load()
        raw = open(table_path, "rb").read()
        self.table = DraftTable(raw)
        self.device = torch.device("cuda", device)
        h = ctypes.c_void_p()
        buf = (ctypes.c_uint8 * len(raw)).from_buffer_copy(raw)
        _lib.check(self.lib.vp_drafter_create(buf, len(raw), device, ctypes.byref(h)), "vp_drafter_create")
        self.h = h
        self._dbg = None

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.vp_drafter_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def begin(self, pids, text: str) -> dict:
        """Build and upload the request context (Drafter.begin); returns the host arrays."""
        ctx = request_context(self.table, pids, text)
        a = {k: np.ascontiguousarray(v) for k, v in ctx.items()}
        q = _Request(len(a["prompt"]), a["prompt"].ctypes.data, len(a["copy"]), a["copy"].ctypes.data,
                     len(a["nb_score"]), a["nb_score"].ctypes.data, a["nb_seq_off"].ctypes.data,
                     a["nb_seq"].ctypes.data, a["nb_key_off"].ctypes.data, a["nb_keys"].ctypes.data,
                     a["nb_pos"].ctypes.data, len(a["as_tok"]), a["as_tok"].ctypes.data, a["as_max"].ctypes.data,
                     a["as_cnt"].ctypes.data, len(a["as_cand"]), a["as_cand"].ctypes.data)
        _lib.check(self.lib.vp_drafter_begin(self.h, ctypes.byref(q)), "vp_drafter_begin")
        return a

    def draft(self, tree_out: torch.Tensor, out_tokens: torch.Tensor, n_out: Optional[int] = None,
              state_ptr: Optional[int] = None, B: int = 15, branch: int = 8, debug: bool = False,
              stream=None) -> Optional[dict]:
        """One drafting step on the device: the tree (VP_TREE_INTS int32, device tensor or pointer
        tree_out) after the output tokens out_tokens (device int32 tensor or pointer; n_out of them,
        or the step count of the device state at state_ptr). With debug, waits and returns the nodes and every expansion's
        top 8."""
        dbg = None
        if debug:
            if self._dbg is None:
                dev = self.device
                self._dbg = {"parents": torch.empty(15, dtype=torch.int32, device=dev),
                             "tokens": torch.empty(15, dtype=torch.int32, device=dev),
                             "exp_tokens": torch.full((16, 8), -1, dtype=torch.int32, device=dev),
                             "exp_probs": torch.zeros((16, 8), dtype=torch.float64, device=dev),
                             "status": torch.zeros(1, dtype=torch.int32, device=dev)}
            self._dbg["exp_tokens"].fill_(-1)
            d = self._dbg
            dbg = _Debug(*[d[k].data_ptr() for k in ("parents", "tokens", "exp_tokens", "exp_probs", "status")])
        s = stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        if out_tokens is None or isinstance(out_tokens, int):
            out_ptr = out_tokens
        else:
            out_ptr = out_tokens.data_ptr()
        tree_ptr = tree_out if isinstance(tree_out, int) else tree_out.data_ptr()
        _lib.check(self.lib.vp_draft(self.h, out_ptr, state_ptr,
                                     -1 if n_out is None else int(n_out), B, branch, tree_ptr,
                                     ctypes.byref(dbg) if dbg is not None else None, s), "vp_draft")
        if not debug:
            return None
        torch.cuda.synchronize(self.device)
        d = self._dbg
        par = d["parents"].cpu().tolist()
        tok = d["tokens"].cpu().tolist()
        n = sum(1 for x in par if x != -2)
        return {"parents": par[:n], "tokens": tok[:n], "exp_tokens": d["exp_tokens"].cpu().numpy(),
                "exp_probs": d["exp_probs"].cpu().numpy(), "status": int(d["status"].item())}
