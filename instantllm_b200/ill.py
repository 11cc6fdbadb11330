"""The reference's `.ill` model container: read it into the standard layouts `VerifyEngine` packs,
and write one from them.

Restates the container of Sources/Engine/ModelFile.swift (:62-144) and the tensor layouts that
Sources/Engine/Convert.swift (:90-215) writes into it:

* a 16 KiB header: magic "ILM1" (u32), version 1 (u32), weight format (u32: 0 f16, 1 q8, 2 q4),
  tensor count (u32, 292), then a table of (offset, size) u64 pairs, one per tensor id;
* tensors 256-byte aligned in id order, the file padded to a multiple of 16 KiB;
* tensor ids (ModelFile.swift:47-60): 0 embedding codes, 1 its scale data, 2 final norm, then per
  layer l at 3 + 12 l: +0 input norm, +1 QKV codes, +2 QKV scales, +3 QKV bias, +4 O codes,
  +5 O scales, +6 post-attention norm, +7 gate/up codes, +8 gate/up scales, +9 down codes,
  +10 down scales; 291 the optional 2-bit sketch of the q4 embedding (read as "embed_hi", the
  input of sketch.SketchHead);
* q4: codes uint8 [rows][cols/2] (column 2j in the low nibble) and f16 (scale, bias) pairs
  [rows][cols/64][2]; q8: int8 codes [rows][cols] and one f16 scale per 32 columns (this
  package's "q8g32"); f16: f16 [rows][cols] and an empty scale tensor; norms and biases f32;
* QKV rows (and the QKV bias) stored in the order of `qkv_row_order` (Convert.swift:331-340),
  gate/up rows in the order of `gu_row_order` (Convert.swift:132-133).

The reference always writes 24 layers. A file written here for a smaller test model keeps the
24-layer table and leaves the missing layers' entries empty; `read_ill` counts the layers whose
QKV entry is present.
"""
from __future__ import annotations

import struct
from typing import Optional

import numpy as np

from .synth import FFN, HIDDEN, QKV_ROWS

MAGIC = 0x314D4C49  # "ILM1"
VERSION = 1
HEADER_BYTES = 16384
PAGE_BYTES = 16384
ALIGN = 256
LAYERS = 24
PER_LAYER = 12
EMBED, EMBED_SB, FINAL_NORM = 0, 1, 2
ATTN_NORM, WQKV, WQKV_SB, BQKV, WO, WO_SB, MLP_NORM, WGU, WGU_SB, WD, WD_SB = range(11)
EMBED_HI = 3 + LAYERS * PER_LAYER
COUNT = EMBED_HI + 1
FORMATS = {"f16": 0, "q8g32": 1, "q4": 2}  # the reference's q8 is group 32
FORMAT_NAMES = {v: k for k, v in FORMATS.items()}


def layer_id(l: int, k: int) -> int:
    return 3 + l * PER_LAYER + k


def qkv_row_order() -> np.ndarray:
    """Stored row i of the QKV matrix = row qkv_row_order()[i] of [q; k; v]: 36 blocks of 32 rows,
    block b holding dims 16 (b % 2) .. +16 and 32 + 16 (b % 2) .. +16 of 64-row head b // 2."""
    order = []
    for b in range(QKV_ROWS // 32):
        head, half = b // 2, b % 2
        order += [head * 64 + half * 16 + i for i in range(16)]
        order += [head * 64 + 32 + half * 16 + i for i in range(16)]
    return np.asarray(order, dtype=np.int64)


def gu_row_order(ffn: int = FFN) -> np.ndarray:
    """Stored row 4b + j of the gate/up matrix = row gu_row_order()[4b + j] of [gate; up]: gate rows
    2b, 2b + 1, then up rows 2b, 2b + 1."""
    order = []
    for b in range(ffn // 2):
        order += [2 * b, 2 * b + 1, ffn + 2 * b, ffn + 2 * b + 1]
    return np.asarray(order, dtype=np.int64)


# ---------------------------------------------------------------------------------------------
# matrices: standard-layout dicts (synth.make_matrix) <-> the two tensors of the container


def _matrix_tensors(m: dict, order: Optional[np.ndarray]) -> tuple:
    """(codes bytes, scale bytes) of a matrix, rows in `order` (None: as they are)."""
    fmt = m["fmt"]
    if fmt == "f16":
        w = np.asarray(m["w"], dtype=np.float16)
        if order is not None:
            w = w[order]
        return np.ascontiguousarray(w).tobytes(), b""
    if fmt not in ("q4", "q8g32"):
        raise ValueError(f"the .ill container holds q4, q8 (group 32) or f16 matrices, not {fmt}")
    codes, scales = np.asarray(m["codes"]), np.asarray(m["scales"], dtype=np.float16)
    if order is not None:
        codes, scales = codes[order], scales[order]
    return np.ascontiguousarray(codes).tobytes(), np.ascontiguousarray(scales).tobytes()


def _matrix_from(fmt: str, codes: np.ndarray, scales: np.ndarray, rows: int, cols: int,
                 order: Optional[np.ndarray]) -> dict:
    """Inverse of _matrix_tensors: the standard-layout dict from the stored tensors."""
    inv = None
    if order is not None:
        inv = np.empty_like(order)
        inv[order] = np.arange(order.size)
    if fmt == "f16":
        w = codes.view(np.float16).reshape(rows, cols)
        return {"fmt": "f16", "w": np.ascontiguousarray(w[inv] if inv is not None else w)}
    if fmt == "q4":
        c = codes.view(np.uint8).reshape(rows, cols // 2)
        s = scales.view(np.float16).reshape(rows, cols // 64, 2)
    else:
        c = codes.view(np.int8).reshape(rows, cols)
        s = scales.view(np.float16).reshape(rows, cols // 32)
    if inv is not None:
        c, s = c[inv], s[inv]
    return {"fmt": fmt, "codes": np.ascontiguousarray(c), "scales": np.ascontiguousarray(s)}


def _f32(a) -> bytes:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32)).tobytes()


# ---------------------------------------------------------------------------------------------
# container (ModelFile.swift:62-144: ModelFile and ModelWriter)


def write_ill(path: str, weights: dict, embed_hi: Optional[np.ndarray] = None) -> None:
    """Write standard-layout weights (synth.make_weights / read_ill) as an .ill file, rows reordered
    the way the reference's converter stores them; embed_hi: the optional 2-bit sketch of a q4
    embedding (convert.sketch_q4), stored as tensor 291."""
    fmt = weights["fmt"]
    if fmt not in FORMATS:
        raise ValueError(f"the .ill container holds q4, q8g32 or f16 weights, not {fmt}")
    if len(weights["layers"]) > LAYERS:
        raise ValueError(f"at most {LAYERS} layers")
    blobs = {}
    blobs[EMBED], blobs[EMBED_SB] = _matrix_tensors(weights["embed"], None)
    blobs[FINAL_NORM] = _f32(weights["final_norm"])
    qo, go = qkv_row_order(), gu_row_order()
    for l, L in enumerate(weights["layers"]):
        blobs[layer_id(l, ATTN_NORM)] = _f32(L["ln1"])
        blobs[layer_id(l, MLP_NORM)] = _f32(L["ln2"])
        blobs[layer_id(l, BQKV)] = _f32(np.asarray(L["bqkv"], dtype=np.float32)[qo])
        blobs[layer_id(l, WQKV)], blobs[layer_id(l, WQKV_SB)] = _matrix_tensors(L["wqkv"], qo)
        blobs[layer_id(l, WO)], blobs[layer_id(l, WO_SB)] = _matrix_tensors(L["wo"], None)
        blobs[layer_id(l, WGU)], blobs[layer_id(l, WGU_SB)] = _matrix_tensors(L["wgu"], go)
        blobs[layer_id(l, WD)], blobs[layer_id(l, WD_SB)] = _matrix_tensors(L["wd"], None)
    if embed_hi is not None:
        blobs[EMBED_HI] = np.ascontiguousarray(embed_hi, dtype=np.uint8).tobytes()
    table = np.zeros(2 * COUNT, dtype=np.uint64)
    cursor = HEADER_BYTES
    layout = []
    for tid in sorted(blobs):
        cursor = (cursor + ALIGN - 1) & ~(ALIGN - 1)
        table[2 * tid], table[2 * tid + 1] = cursor, len(blobs[tid])
        layout.append((cursor, blobs[tid]))
        cursor += len(blobs[tid])
    total = (cursor + PAGE_BYTES - 1) // PAGE_BYTES * PAGE_BYTES
    header = struct.pack("<IIII", MAGIC, VERSION, FORMATS[fmt], COUNT) + table.tobytes()
    assert len(header) <= HEADER_BYTES
    with open(path, "wb") as f:
        f.write(header)
        for off, data in layout:
            f.seek(off)
            f.write(data)
        f.truncate(total)


def read_ill(path: str) -> dict:
    """Read an .ill file (memory-mapped) into the standard layouts VerifyEngine packs. Raises
    ValueError for what ModelFile.init rejects: a bad size, magic, version, format or table."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    size = raw.size
    if size < HEADER_BYTES or size % PAGE_BYTES:
        raise ValueError(f"{path}: bad size {size}")
    magic, version, fcode, count = struct.unpack_from("<IIII", raw, 0)
    if magic != MAGIC:
        raise ValueError(f"{path}: not an instantllm model")
    if version != VERSION:
        raise ValueError(f"{path}: unsupported version {version}")
    if fcode not in FORMAT_NAMES:
        raise ValueError(f"{path}: unknown or unsupported weight format {fcode} (q4a is not read here)")
    if count != COUNT:
        raise ValueError(f"{path}: tensor table mismatch ({count} entries)")
    fmt = FORMAT_NAMES[fcode]
    table = np.frombuffer(raw[16:16 + 16 * COUNT].tobytes(), dtype=np.uint64).reshape(COUNT, 2)

    def tensor(tid: int) -> np.ndarray:
        off, n = int(table[tid, 0]), int(table[tid, 1])
        if n and (off < HEADER_BYTES or off + n > size):
            raise ValueError(f"{path}: tensor {tid} outside the file")
        return raw[off:off + n]

    def vec(tid: int, n: int) -> np.ndarray:
        v = tensor(tid).view(np.float32)
        if v.size != n:
            raise ValueError(f"{path}: tensor {tid} holds {v.size} floats, expected {n}")
        return np.array(v)

    def mat(cid: int, sid: int, rows: int, cols: int, order) -> dict:
        return _matrix_from(fmt, tensor(cid), tensor(sid), rows, cols, order)

    per_row = {"q4": HIDDEN // 2, "q8g32": HIDDEN, "f16": 2 * HIDDEN}[fmt]
    vocab = int(table[EMBED, 1]) // per_row
    qo, go = qkv_row_order(), gu_row_order()
    layers = []
    for l in range(LAYERS):
        if table[layer_id(l, WQKV), 1] == 0:
            break
        layers.append({
            "ln1": vec(layer_id(l, ATTN_NORM), HIDDEN),
            "ln2": vec(layer_id(l, MLP_NORM), HIDDEN),
            "bqkv": vec(layer_id(l, BQKV), QKV_ROWS)[np.argsort(qo)],
            "wqkv": mat(layer_id(l, WQKV), layer_id(l, WQKV_SB), QKV_ROWS, HIDDEN, qo),
            "wo": mat(layer_id(l, WO), layer_id(l, WO_SB), HIDDEN, HIDDEN, None),
            "wgu": mat(layer_id(l, WGU), layer_id(l, WGU_SB), 2 * FFN, HIDDEN, go),
            "wd": mat(layer_id(l, WD), layer_id(l, WD_SB), HIDDEN, FFN, None),
        })
    embed_hi = None
    if table[EMBED_HI, 1]:
        if fmt != "q4" or int(table[EMBED_HI, 1]) != vocab * (HIDDEN // 4):
            raise ValueError(f"{path}: sketch plane of {int(table[EMBED_HI, 1])} bytes does not fit the embedding")
        embed_hi = np.array(tensor(EMBED_HI)).reshape(vocab, HIDDEN // 4)
    return {"fmt": fmt, "n_layers": len(layers), "vocab": vocab,
            "embed": mat(EMBED, EMBED_SB, vocab, HIDDEN, None),
            "final_norm": vec(FINAL_NORM, HIDDEN), "layers": layers, "embed_hi": embed_hi}
