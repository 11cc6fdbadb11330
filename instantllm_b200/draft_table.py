"""The reference drafter's table (format ILDRAFT1, tools/draft/ildraft.py:1-47 FORMAT and :352-413
Tables.load) read into flat arrays, and the lookup primitives the drafter is built on: the FNV-1a
64-bit hash (:63-68), the n-gram context key (:71-72), the prompt's distinct words (:79-88), the
n-gram, word and association lookups (:416-429).

Sections stay as the file stores them: sorted 64-bit keys searched by bisection, with parallel value
arrays and (first, n) ranges into flat arrays. That is the layout a drafter kernel reads from device
memory as well (one binary search per lookup, no hash maps). This module covers the table, the
lookups and the request's nearest training documents (the TF-IDF part of Drafter.begin, which the
host runs at request start); the candidate features, the scorer and the best-first tree run on
the GPU (csrc/vp_draft.cuh), and their CPU restatement is the checker in oracle/drafter.py.
"""
from __future__ import annotations

import re
import struct
from typing import Optional

import numpy as np

MAGIC = b"ILDRAFT1"
FNV_OFF = 0xCBF29CE484222325
FNV_PRIME = 0x100000001B3
M64 = (1 << 64) - 1
N_FEATURES = 53  # ildraft.py FEATS
FLAG_ASSOC, FLAG_ASSOC_CANDS, FLAG_EDIT = 1, 2, 4
VOCAB = 151936

_WORD = re.compile(rb"[a-z0-9]+")


def fnv1a64(b: bytes) -> int:
    """FNV-1a, 64 bits, over bytes."""
    h = FNV_OFF
    for x in b:
        h = ((h ^ x) * FNV_PRIME) & M64
    return h


def ctx_key(tokens) -> int:
    """Key of an n-gram context: FNV-1a over the order (one byte) then each token as u32 LE."""
    t = [int(x) for x in tokens]
    return fnv1a64(bytes([len(t)]) + struct.pack(f"<{len(t)}I", *t))


def prompt_words(text: str) -> list:
    """The prompt's distinct words in first-appearance order: runs of [a-z0-9] after ASCII
    lowercasing the UTF-8 bytes."""
    seen, out = set(), []
    for w in _WORD.findall(text.encode("utf-8").lower()):
        if w not in seen:
            seen.add(w)
            out.append(w)
    return out


STOPS = (151645, 151643)


# section tag -> numpy dtype of one record
_DT = {
    b"NGKY": np.dtype("<u8"), b"NGVL": np.dtype([("total", "<u4"), ("first_n", "<u4")]),
    b"NGNX": np.dtype([("token", "<u4"), ("count", "<u4")]),
    b"WDKY": np.dtype("<u8"), b"WDVL": np.dtype([("idf", "<f4"), ("first", "<u4"), ("n", "<u4")]),
    b"POST": np.dtype("<u4"), b"DNRM": np.dtype("<f4"), b"SQOF": np.dtype("<u4"), b"SQTK": np.dtype("<u4"),
    b"CPTK": np.dtype([("token", "<u4"), ("v", "<f4")]), b"CPC1": np.dtype([("token", "<u4"), ("v", "<f4")]),
    b"CPC2": np.dtype([("key", "<u8"), ("v", "<f4"), ("pad", "<u4")]),
    b"ASWK": np.dtype("<u8"), b"ASWV": np.dtype([("first", "<u4"), ("n", "<u4")]),
    b"ASTK": np.dtype([("token", "<u4"), ("loglift", "<f4")]),
    b"PTXO": np.dtype("<u4"), b"PTXB": np.dtype("u1"), b"TFLS": np.dtype([("token", "<u4"), ("flags", "<u4")]),
    b"TFLG": np.dtype("u1"), b"MLP0": np.dtype("<f4"),
}

_HEADER = struct.Struct("<8sII" + "I" * 8 + "IIII")


class DraftTable:
    """An ILDRAFT1 file: header fields as attributes (N, M, KNB, MAXM, F, H, minc_hi, n_docs, flags,
    as_top, edit_E) and each section as a read-only numpy array in `sec` (tag -> array)."""

    def __init__(self, raw: bytes):
        (magic, version, nsec, self.N, self.M, self.KNB, self.MAXM, self.F, self.H, self.minc_hi,
         self.n_docs, self.flags, self.as_top, self.edit_E, _) = _HEADER.unpack_from(raw, 0)
        if magic != MAGIC or version != 1:
            raise ValueError(f"not an ILDRAFT1 v1 table ({magic!r}, version {version})")
        if self.F != N_FEATURES:
            raise ValueError(f"table has {self.F} features, the drafter {N_FEATURES}")
        self.sec = {}
        for i in range(nsec):
            tag, cnt, off = struct.unpack_from("<4sIQ", raw, 64 + 16 * i)
            dt = _DT.get(tag)
            if dt is None:
                continue  # sections this reader does not use
            if off % 8 or off + cnt * dt.itemsize > len(raw):
                raise ValueError(f"section {tag!r} outside the file or not 8-aligned")
            self.sec[tag] = np.frombuffer(raw, dtype=dt, count=cnt, offset=off)
        for tag in (b"NGKY", b"NGVL", b"NGNX", b"WDKY", b"WDVL", b"POST", b"DNRM", b"SQOF", b"SQTK", b"MLP0"):
            if tag not in self.sec:
                raise ValueError(f"section {tag!r} missing")
        if len(self.sec[b"NGKY"]) != len(self.sec[b"NGVL"]) or len(self.sec[b"WDKY"]) != len(self.sec[b"WDVL"]):
            raise ValueError("key and value sections differ in length")

    @classmethod
    def load(cls, path: str) -> "DraftTable":
        with open(path, "rb") as f:
            return cls(f.read())

    @staticmethod
    def _find(keys: np.ndarray, k: int) -> int:
        i = int(np.searchsorted(keys, np.uint64(k)))
        return i if i < len(keys) and int(keys[i]) == k else -1

    def ng_get(self, ctx) -> Optional[tuple]:
        """(total count, [(next token, count), ...]) of an n-gram context, or None."""
        i = self._find(self.sec[b"NGKY"], ctx_key(ctx))
        if i < 0:
            return None
        v = self.sec[b"NGVL"][i]
        first, n = int(v["first_n"]) >> 3, int(v["first_n"]) & 7
        nx = self.sec[b"NGNX"][first:first + n]
        return int(v["total"]), [(int(a), int(b)) for a, b in zip(nx["token"], nx["count"])]

    def vocab_get(self, word: bytes) -> Optional[tuple]:
        """(idf, [doc ids]) of a prompt word, or None."""
        i = self._find(self.sec[b"WDKY"], fnv1a64(word))
        if i < 0:
            return None
        v = self.sec[b"WDVL"][i]
        first, n = int(v["first"]), int(v["n"])
        return float(v["idf"]), [int(d) for d in self.sec[b"POST"][first:first + n]]

    def assoc_get(self, word: bytes) -> Optional[list]:
        """[(token, loglift), ...] associated with a prompt word, or None."""
        if not (self.flags & FLAG_ASSOC) or b"ASWK" not in self.sec:
            return None
        i = self._find(self.sec[b"ASWK"], fnv1a64(word))
        if i < 0:
            return None
        v = self.sec[b"ASWV"][i]
        t = self.sec[b"ASTK"][int(v["first"]):int(v["first"]) + int(v["n"])]
        return [(int(a), float(b)) for a, b in zip(t["token"], t["loglift"])]

    def neighbours(self, text: str, knb: Optional[int] = None) -> list:
        """The request's nearest training documents (ildraft.py:455-468, Drafter.begin): TF-IDF
        cosine between the prompt's distinct words and each document, score = sum over shared
        words of idf^2 / (|q| |d|), with |q|^2 the sum of idf^2 over the prompt's words found in
        the table; the top `knb` (default KNB) as [(score, doc)] by score descending, then doc
        ascending. Scores in float64, summed per document in prompt-word order."""
        knb = self.KNB if knb is None else knb
        sc = np.zeros(self.n_docs, dtype=np.float64)
        hit = np.zeros(self.n_docs, dtype=bool)
        q2 = 0.0
        for w in prompt_words(text):
            e = self.vocab_get(w)
            if e is None:
                continue
            idf, docs = e
            ii = idf * idf
            q2 += ii
            if docs:
                d = np.asarray(docs, dtype=np.int64)
                np.add.at(sc, d, ii)
                hit[d] = True
        qn = float(np.sqrt(q2)) or 1.0
        docs = np.nonzero(hit)[0]
        norms = self.sec[b"DNRM"].astype(np.float64)
        s = [(float(sc[j]) / (qn * float(norms[j])), int(j)) for j in docs]
        s.sort(key=lambda x: (-x[0], x[1]))
        return s[:knb]

    def seq(self, doc: int) -> list:
        """Training output `doc` (generated ids and the stop token if it stopped)."""
        o = self.sec[b"SQOF"]
        return [int(x) for x in self.sec[b"SQTK"][int(o[doc]):int(o[doc + 1])]]

    def token_flags(self) -> np.ndarray:
        """uint8 [151936]: bits 0-2 the number of backticks in the token text (capped 7), bit 3 a newline."""
        out = np.zeros(VOCAB, dtype=np.uint8)
        if b"TFLS" in self.sec:
            t = self.sec[b"TFLS"]
            out[t["token"].astype(np.int64)] = t["flags"].astype(np.uint8)
        elif b"TFLG" in self.sec:
            out[:len(self.sec[b"TFLG"])] = self.sec[b"TFLG"]
        return out

    def mlp(self) -> dict:
        """Scorer weights: score(x) = W2 . relu(W1 x + b1) + b2 + WL . x."""
        f, F, H = self.sec[b"MLP0"], self.F, self.H
        p = H * F
        return {"W1": f[:p].reshape(H, F), "b1": f[p:p + H], "W2": f[p + H:p + 2 * H],
                "b2": float(f[p + 2 * H]), "WL": f[p + 2 * H + 1:p + 2 * H + 1 + F]}
