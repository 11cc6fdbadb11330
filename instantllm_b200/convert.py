"""Hugging Face checkpoint -> .ill model file, as the reference's converter does it.

Restates Sources/Engine/Convert.swift: the safetensors reader (:6-62), `Converter.convert`
(:90-215: which tensors, how QKV / gate-up are stacked, the optional quant file with ready q4
codes), q4 affine group-64 quantization with its clip search and least-squares refit
(`quantizeQ4Raw` / `quantGroup`, :290-370), symmetric q8 group 32 (`quantizeQ8`, :254-282), f16,
and the 2-bit sketch of the q4 embedding (:150-158). The row reordering and the container are in
`ill.py`. Arithmetic follows the reference's fp32 order (sequential sums, round half away from
zero, fp16 rounding of scale and bias) so that the codes come out the same.

Usage: python -m instantllm_b200.convert --hf DIR --out model.ill --format q4 [--quant FILE]
[--sketch]. The reference always converts 24 layers; here the layer count is read from the
checkpoint, so that small test checkpoints convert too.
"""
from __future__ import annotations

import argparse
import json
from typing import Optional

import numpy as np

from . import ill
from .synth import FFN, HIDDEN

CLIPS = np.asarray([0.0, 0.03, 0.06, 0.1, 0.15], dtype=np.float32)


class SafeTensors:
    """A safetensors file, memory-mapped: 8-byte little-endian header length, JSON header, data."""

    def __init__(self, path: str):
        self.raw = np.memmap(path, dtype=np.uint8, mode="r")
        n = int(np.frombuffer(self.raw[:8].tobytes(), dtype="<u8")[0])
        self.data_start = 8 + n
        header = json.loads(self.raw[8:8 + n].tobytes())
        self.entries = {k: v for k, v in header.items() if k != "__metadata__"}

    def has(self, name: str) -> bool:
        return name in self.entries

    def raw_tensor(self, name: str):
        if name not in self.entries:
            raise ValueError(f"missing tensor {name}")
        e = self.entries[name]
        a, b = e["data_offsets"]
        return e["shape"], e["dtype"], self.raw[self.data_start + a:self.data_start + b]

    def floats(self, name: str) -> np.ndarray:
        """A BF16 tensor as fp32 (the reference accepts only BF16 here)."""
        shape, dtype, buf = self.raw_tensor(name)
        if dtype != "BF16":
            raise ValueError(f"{name}: expected BF16, got {dtype}")
        u = np.frombuffer(buf.tobytes(), dtype="<u2").astype(np.uint32) << 16
        return u.view(np.float32).reshape(shape)

    def any_floats(self, name: str) -> np.ndarray:
        """Any float tensor (BF16, F16, F32) as fp32."""
        shape, dtype, buf = self.raw_tensor(name)
        if dtype == "F32":
            return np.frombuffer(buf.tobytes(), dtype="<f4").reshape(shape).copy()
        if dtype == "F16":
            return np.frombuffer(buf.tobytes(), dtype="<f2").astype(np.float32).reshape(shape)
        return self.floats(name)


def write_safetensors(path: str, tensors: dict) -> None:
    """Write name -> (dtype, array) as a safetensors file (test and tooling helper). dtype is one of
    BF16 (array fp32, rounded to nearest even), F16, F32, U8."""
    header, blobs, off = {}, [], 0
    for name, (dtype, a) in tensors.items():
        a = np.ascontiguousarray(a)
        if dtype == "BF16":
            u = a.astype(np.float32).view(np.uint32)
            b = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype("<u2").tobytes()
        else:
            b = a.astype({"F16": "<f2", "F32": "<f4", "U8": "u1"}[dtype]).tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(np.asarray([len(h)], dtype="<u8").tobytes())
        f.write(h)
        for b in blobs:
            f.write(b)


# ---------------------------------------------------------------------------------------------
# quantization (fp32 throughout, as the reference)


def _round_away(x: np.ndarray) -> np.ndarray:
    """Round half away from zero (Swift's Float.rounded()), exactly: x - floor(x) is exact in fp32."""
    a = np.abs(x)
    f = np.floor(a)
    return np.copysign(f + (a - f >= np.float32(0.5)).astype(np.float32), x).astype(np.float32)


def _seq_sum(a: np.ndarray) -> np.ndarray:
    """Left-to-right fp32 sum along the last axis (the reference's `+=` loop order)."""
    return np.cumsum(a, axis=-1, dtype=np.float32)[..., -1]


def quantize_q8(m: np.ndarray) -> tuple:
    """Symmetric 8-bit, one fp16 scale per 32 columns (Convert.swift:254-282): the scale is the
    fp16 nearest amax / 127, raised by one ulp if that leaves a code above 127. Returns (int8
    codes [rows][cols], fp16 scales [rows][cols / 32])."""
    m = np.asarray(m, dtype=np.float32)
    rows, cols = m.shape
    g = m.reshape(rows, cols // 32, 32)
    amax = np.max(np.abs(g), axis=-1)
    sh = (amax / np.float32(127)).astype(np.float16)
    low = sh.astype(np.float32) * np.float32(127) < amax
    sh = np.where(low, (sh.view(np.uint16) + 1).view(np.float16), sh)
    s = sh.astype(np.float32)
    inv = np.where(s > 0, np.float32(1) / np.where(s > 0, s, np.float32(1)), np.float32(0)).astype(np.float32)
    q = np.clip(_round_away(g * inv[..., None]), -127, 127).astype(np.int8)
    return q.reshape(rows, cols), sh


def _q4_groups(w: np.ndarray) -> tuple:
    """quantGroup (Convert.swift:323-370) over many 64-wide groups w [G][64] at once: for each
    pair of clip fractions (low, high) of the group's range, scale and bias from the clipped range,
    one least-squares refit, fp16 rounding of both, requantization, and the pair with the lowest
    squared error kept (first on ties). Returns (codes uint8 [G][64], scale fp16 [G], bias fp16 [G])."""
    w = np.asarray(w, dtype=np.float32)
    n = w.shape[0]
    f32 = np.float32
    mn, mx = w.min(axis=1), w.max(axis=1)
    rng = (mx - mn).astype(f32)
    flat = rng < f32(1e-12)
    sw = _seq_sum(w)
    best_err = np.full(n, np.inf, dtype=f32)
    best_s = np.zeros(n, dtype=np.float16)
    best_b = np.zeros(n, dtype=np.float16)
    best_q = np.zeros((n, 64), dtype=np.uint8)
    with np.errstate(all="ignore"):
        for a in CLIPS:
            for c in CLIPS:
                lo = (mn + a * rng).astype(f32)
                hi = (mx - c * rng).astype(f32)
                ok = (hi > lo) & ~flat
                s = ((hi - lo) / f32(15)).astype(f32)
                b = lo
                v = np.clip(_round_away((w - b[:, None]) * (f32(1) / s)[:, None]), 0, 15).astype(f32)
                sq, sqq, sqw = _seq_sum(v), _seq_sum(v * v), _seq_sum(v * w)
                den = (f32(64) * sqq - sq * sq).astype(f32)
                s2 = ((f32(64) * sqw - sq * sw) / den).astype(f32)
                refit = (den > 0) & (s2 > 0)
                b = np.where(refit, ((sw - s2 * sq) / f32(64)).astype(f32), b)
                s = np.where(refit, s2, s)
                sh, bh = s.astype(np.float16), b.astype(np.float16)
                sf, bf = sh.astype(f32), bh.astype(f32)
                ok &= sf > 0
                v = np.clip(_round_away((w - bf[:, None]) * (f32(1) / sf)[:, None]), 0, 15).astype(f32)
                d = (sf[:, None] * v + bf[:, None] - w).astype(f32)
                err = _seq_sum(d * d)
                take = ok & (err < best_err)
                best_err = np.where(take, err, best_err)
                best_s = np.where(take, sh, best_s)
                best_b = np.where(take, bh, best_b)
                best_q = np.where(take[:, None], v.astype(np.uint8), best_q)
    # a flat group: codes 0, scale 0, bias = its value
    best_s = np.where(flat, np.float16(0), best_s)
    best_b = np.where(flat, mn.astype(np.float16), best_b)
    best_q[flat] = 0
    return best_q, best_s, best_b


def quantize_q4(m: np.ndarray, chunk_rows: int = 2048) -> dict:
    """Affine 4-bit, group 64 (quantizeQ4Raw, Convert.swift:290-321): a standard-layout q4 matrix
    (codes uint8 [rows][cols/2], column 2j in the low nibble; fp16 (scale, bias) [rows][cols/64][2])."""
    m = np.asarray(m, dtype=np.float32)
    rows, cols = m.shape
    codes = np.empty((rows, cols // 2), dtype=np.uint8)
    sb = np.empty((rows, cols // 64, 2), dtype=np.float16)
    for r0 in range(0, rows, chunk_rows):
        blk = m[r0:r0 + chunk_rows]
        q, s, b = _q4_groups(blk.reshape(-1, 64))
        q = q.reshape(blk.shape[0], cols)
        codes[r0:r0 + chunk_rows] = q[:, 0::2] | (q[:, 1::2] << 4)
        sb[r0:r0 + chunk_rows, :, 0] = s.reshape(blk.shape[0], cols // 64)
        sb[r0:r0 + chunk_rows, :, 1] = b.reshape(blk.shape[0], cols // 64)
    return {"fmt": "q4", "codes": codes, "scales": sb}


def sketch_q4(codes: np.ndarray) -> np.ndarray:
    """The 2-bit sketch of a q4 matrix (Convert.swift:150-158): byte j of a row holds the high two
    bits of codes 4j .. 4j + 3 (code 4j in bits 0-1)."""
    c = np.stack([codes & 0xF, codes >> 4], axis=-1).reshape(codes.shape[0], -1) >> 2
    c = c.reshape(codes.shape[0], -1, 4).astype(np.uint8)
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)


def convert(hf_dir: str, output: str, fmt: str = "q4", quant_file: Optional[str] = None,
            sketch: bool = False, log=print) -> dict:
    """Converter.convert (Convert.swift:90-215): model.safetensors (BF16) in hf_dir -> an .ill file.
    fmt is "q4", "q8" (group 32) or "f16". A quant file may hold ready q4 codes (name + ".q" /
    ".scale" / ".bias") and float overrides of norms and biases (folded transforms). Returns the
    standard-layout weights written."""
    fmt = {"q8": "q8g32"}.get(fmt, fmt)
    if fmt not in ill.FORMATS:
        raise ValueError(f"unknown format {fmt}")
    hf = SafeTensors(hf_dir.rstrip("/") + "/model.safetensors")
    qf = SafeTensors(quant_file) if quant_file else None
    if qf is not None and fmt != "q4":
        raise ValueError("--quant files hold q4 codes; use --format q4")

    def vec(name: str) -> np.ndarray:
        if qf is not None and qf.has(name):
            return qf.any_floats(name).astype(np.float32).reshape(-1)
        return hf.floats(name).reshape(-1)

    def matrix(name: str) -> dict:
        if fmt == "q4" and qf is not None and qf.has(name + ".q"):
            shape, dtype, buf = qf.raw_tensor(name + ".q")
            sc, bi = qf.raw_tensor(name + ".scale"), qf.raw_tensor(name + ".bias")
            if dtype != "U8" or sc[1] != "F16" or bi[1] != "F16":
                raise ValueError(f"{name}: bad quant dtypes")
            rows, cols = shape[0], shape[1] * 2
            s = np.frombuffer(sc[2].tobytes(), dtype="<f2").reshape(rows, cols // 64)
            b = np.frombuffer(bi[2].tobytes(), dtype="<f2").reshape(rows, cols // 64)
            return {"fmt": "q4", "codes": np.frombuffer(buf.tobytes(), dtype=np.uint8).reshape(rows, cols // 2),
                    "scales": np.stack([s, b], axis=-1)}
        m = hf.floats(name)
        if fmt == "q4":
            return quantize_q4(m)
        if fmt == "q8g32":
            c, s = quantize_q8(m)
            return {"fmt": "q8g32", "codes": c, "scales": s}
        return {"fmt": "f16", "w": m.astype(np.float16)}

    def stack(*ms: dict) -> dict:
        if ms[0]["fmt"] == "f16":
            return {"fmt": "f16", "w": np.concatenate([m["w"] for m in ms])}
        return {"fmt": ms[0]["fmt"], "codes": np.concatenate([m["codes"] for m in ms]),
                "scales": np.concatenate([m["scales"] for m in ms])}

    n_layers = 0
    while hf.has(f"model.layers.{n_layers}.input_layernorm.weight"):
        n_layers += 1
    embed = matrix("model.embed_tokens.weight")
    log("embedding done")
    layers = []
    for l in range(n_layers):
        p = f"model.layers.{l}."
        layers.append({
            "ln1": vec(p + "input_layernorm.weight"),
            "ln2": vec(p + "post_attention_layernorm.weight"),
            "bqkv": np.concatenate([vec(p + f"self_attn.{x}_proj.bias") for x in "qkv"]),
            "wqkv": stack(*[matrix(p + f"self_attn.{x}_proj.weight") for x in "qkv"]),
            "wo": matrix(p + "self_attn.o_proj.weight"),
            "wgu": stack(matrix(p + "mlp.gate_proj.weight"), matrix(p + "mlp.up_proj.weight")),
            "wd": matrix(p + "mlp.down_proj.weight"),
        })
        log(f"layer {l} done")
    rows = embed["codes"].shape[0] if "codes" in embed else embed["w"].shape[0]
    weights = {"fmt": fmt, "n_layers": n_layers, "vocab": rows, "embed": embed,
               "final_norm": vec("model.norm.weight"), "layers": layers}
    ill.write_ill(output, weights, embed_hi=sketch_q4(embed["codes"]) if sketch and fmt == "q4" else None)
    log(f"wrote {output}")
    return weights


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Hugging Face Qwen2.5-0.5B checkpoint -> .ill model file")
    ap.add_argument("--hf", required=True, help="directory holding model.safetensors")
    ap.add_argument("--out", required=True)
    ap.add_argument("--format", default="q4", choices=["q4", "q8", "f16"])
    ap.add_argument("--quant", default=None, help="safetensors file with ready q4 codes")
    ap.add_argument("--sketch", action="store_true", help="also write the 2-bit embedding sketch")
    a = ap.parse_args(argv)
    convert(a.hf, a.out, a.format, a.quant, a.sketch)


if __name__ == "__main__":
    main()
