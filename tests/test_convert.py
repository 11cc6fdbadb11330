"""The Hugging Face -> .ill converter (Convert.swift): the q4 group quantizer against a scalar,
line-by-line restatement of quantGroup, the q8 scale rule, the sketch bits, and a whole
conversion of a small synthetic BF16 checkpoint read back through read_ill. CPU only."""
import numpy as np
import pytest

from instantllm_b200 import convert, ill, synth

F32 = np.float32


def _round_away(x):
    x = F32(x)
    a = abs(x)
    f = np.floor(a)
    r = f + (F32(1) if a - f >= F32(0.5) else F32(0))
    return F32(-r) if x < 0 else F32(r)


def _quant_group_scalar(w):
    """Convert.swift:323-370, one group, in fp32 scalar steps in the reference's order."""
    w = [F32(v) for v in w]
    mn, mx = min(w), max(w)
    if mx - mn < F32(1e-12):
        return [0] * 64, np.float16(0), np.float16(mn)
    best_err, best = F32(np.inf), (np.float16(0), np.float16(0), [0] * 64)
    rng = F32(mx - mn)
    for a in convert.CLIPS:
        for c in convert.CLIPS:
            lo, hi = F32(mn + F32(a) * rng), F32(mx - F32(c) * rng)
            if hi <= lo:
                continue
            s, b = F32((hi - lo) / F32(15)), lo
            for it in range(2):
                inv = F32(F32(1) / s)
                sq = sw = sqq = sqw = F32(0)
                for i in range(64):
                    v = F32(min(15, max(0, _round_away(F32((w[i] - b) * inv)))))
                    sq = F32(sq + v)
                    sw = F32(sw + w[i])
                    sqq = F32(sqq + F32(v * v))
                    sqw = F32(sqw + F32(v * w[i]))
                if it == 1:
                    break
                den = F32(F32(64) * sqq - F32(sq * sq))
                if den <= 0:
                    break
                s2 = F32(F32(F32(64) * sqw - F32(sq * sw)) / den)
                if s2 <= 0:
                    break
                s, b = s2, F32(F32(sw - F32(s2 * sq)) / F32(64))
            sh, bh = np.float16(s), np.float16(b)
            sf, bf = F32(sh), F32(bh)
            if sf <= 0:
                continue
            inv = F32(F32(1) / sf)
            q, err = [], F32(0)
            for i in range(64):
                v = F32(min(15, max(0, _round_away(F32((w[i] - bf) * inv)))))
                q.append(int(v))
                d = F32(F32(F32(sf * v) + bf) - w[i])
                err = F32(err + F32(d * d))
            if err < best_err:
                best_err, best = err, (sh, bh, q)
    return best[2], best[0], best[1]


def test_q4_groups_match_scalar_restatement():
    rng = np.random.default_rng(5)
    groups = [rng.normal(0, 0.02, 64), rng.normal(0, 1.0, 64), rng.uniform(-3, 1, 64),
              np.r_[rng.normal(0, 0.02, 63), 0.5], np.full(64, 0.25), rng.standard_t(2, 64) * 0.05]
    w = np.stack(groups).astype(F32)
    q, s, b = convert._q4_groups(w)
    for g in range(len(groups)):
        qs, ss, bs = _quant_group_scalar(w[g])
        assert list(q[g]) == qs, g
        assert s[g].view(np.uint16) == np.float16(ss).view(np.uint16), g
        assert b[g].view(np.uint16) == np.float16(bs).view(np.uint16), g


def test_q4_matrix_layout_and_error():
    rng = np.random.default_rng(6)
    m = rng.normal(0, 0.02, size=(8, 128)).astype(F32)
    q = convert.quantize_q4(m, chunk_rows=3)
    codes, sb = q["codes"], q["scales"].astype(F32)
    lo, hi = codes & 0xF, codes >> 4
    full = np.empty((8, 128), dtype=F32)
    full[:, 0::2], full[:, 1::2] = lo, hi
    deq = full.reshape(8, 2, 64) * sb[:, :, 0:1] + sb[:, :, 1:2]
    sse = ((deq.reshape(8, 128) - m) ** 2).reshape(8, 2, 64).sum(-1)
    # the clip search and refit do at least about as well as the plain min / max grid
    g = m.reshape(8, 2, 64)
    lo, step = g.min(-1, keepdims=True), (g.max(-1, keepdims=True) - g.min(-1, keepdims=True)) / 15
    naive = ((np.clip(np.round((g - lo) / step), 0, 15) * step + lo - g) ** 2).sum(-1)
    assert np.all(sse <= naive * 1.05)


def test_q8_scale_rule():
    rng = np.random.default_rng(7)
    m = rng.normal(0, 0.05, size=(4, 64)).astype(F32)
    m[0, :32] = 0.0  # an all-zero group: scale 0, codes 0
    codes, s = convert.quantize_q8(m)
    assert codes.dtype == np.int8 and s.shape == (4, 2)
    assert s[0, 0] == 0 and np.all(codes[0, :32] == 0)
    amax = np.abs(m.reshape(4, 2, 32)).max(-1)
    sf = s.astype(F32)
    ok = amax > 0
    assert np.all(sf[ok] * 127 >= amax[ok])  # every code in range
    below = (s.view(np.uint16) - 1).view(np.float16).astype(F32)
    assert np.all((below[ok] * 127 < amax[ok]) | (np.float16(amax[ok] / 127).astype(F32) == sf[ok]))
    assert np.all(np.abs(codes) <= 127)
    deq = codes.reshape(4, 2, 32).astype(F32) * sf[..., None]
    assert np.all(np.abs(deq.reshape(4, 64) - m) <= sf.repeat(32, axis=1) * 0.5 + 1e-7)


def test_sketch_bits():
    codes = np.array([[0x3C, 0xF1]], dtype=np.uint8)  # codes 12, 3, 1, 15
    assert convert.sketch_q4(codes)[0, 0] == (3 | (0 << 2) | (0 << 4) | (3 << 6))


def _checkpoint(path, vocab=256, n_layers=1, seed=8):
    rng = np.random.default_rng(seed)
    H, F = synth.HIDDEN, synth.FFN
    t = {"model.embed_tokens.weight": ("BF16", rng.normal(0, 0.02, (vocab, H))),
         "model.norm.weight": ("BF16", rng.normal(1, 0.1, H))}
    for l in range(n_layers):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = ("BF16", rng.normal(1, 0.1, H))
        t[p + "post_attention_layernorm.weight"] = ("BF16", rng.normal(1, 0.1, H))
        for x, r in (("q", 896), ("k", 128), ("v", 128)):
            t[p + f"self_attn.{x}_proj.weight"] = ("BF16", rng.normal(0, 0.02, (r, H)))
            t[p + f"self_attn.{x}_proj.bias"] = ("BF16", rng.normal(0, 0.02, r))
        t[p + "self_attn.o_proj.weight"] = ("BF16", rng.normal(0, 0.02, (H, H)))
        t[p + "mlp.gate_proj.weight"] = ("BF16", rng.normal(0, 0.02, (F, H)))
        t[p + "mlp.up_proj.weight"] = ("BF16", rng.normal(0, 0.02, (F, H)))
        t[p + "mlp.down_proj.weight"] = ("BF16", rng.normal(0, 0.02, (H, F)))
    convert.write_safetensors(str(path / "model.safetensors"), t)
    return convert.SafeTensors(str(path / "model.safetensors"))


@pytest.mark.parametrize("fmt", ["q8", "f16"])
def test_convert_checkpoint(fmt, tmp_path):
    st = _checkpoint(tmp_path)
    out = str(tmp_path / "m.ill")
    w = convert.convert(str(tmp_path), out, fmt, log=lambda s: None)
    r = ill.read_ill(out)
    assert r["n_layers"] == 1 and r["vocab"] == 256 and r["fmt"] == {"q8": "q8g32"}.get(fmt, fmt)
    L, src = r["layers"][0], "model.layers.0."
    assert np.array_equal(L["ln1"], st.floats(src + "input_layernorm.weight"))
    bias = np.concatenate([st.floats(src + f"self_attn.{x}_proj.bias") for x in "qkv"])
    assert np.array_equal(L["bqkv"], bias)
    q = st.floats(src + "self_attn.k_proj.weight")
    up = st.floats(src + "mlp.up_proj.weight")
    if fmt == "f16":
        assert np.array_equal(L["wqkv"]["w"][896:1024], q.astype(np.float16))
        assert np.array_equal(L["wgu"]["w"][synth.FFN:], up.astype(np.float16))
    else:
        c, s = convert.quantize_q8(q)
        assert np.array_equal(L["wqkv"]["codes"][896:1024], c) and np.array_equal(L["wqkv"]["scales"][896:1024], s)
        assert np.array_equal(L["wgu"]["codes"][synth.FFN:], convert.quantize_q8(up)[0])
    _same = [np.array_equal(a, b) for a, b in zip(w["layers"][0]["bqkv"], L["bqkv"])]
    assert all(_same)


def test_convert_q4_with_quant_file_and_sketch(tmp_path):
    """q4 with ready codes from a quant file (the reference's --quant: name.q / .scale / .bias)
    for every layer matrix and a float override of a norm; the embedding is quantized here and its
    2-bit sketch written as tensor 291."""
    st = _checkpoint(tmp_path)
    rng = np.random.default_rng(9)
    qt, want = {}, {}
    src = "model.layers.0."
    for name, rows, cols in (("self_attn.q_proj.weight", 896, 896), ("self_attn.k_proj.weight", 128, 896),
                             ("self_attn.v_proj.weight", 128, 896), ("self_attn.o_proj.weight", 896, 896),
                             ("mlp.gate_proj.weight", synth.FFN, 896), ("mlp.up_proj.weight", synth.FFN, 896),
                             ("mlp.down_proj.weight", 896, synth.FFN)):
        codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
        sc = np.abs(rng.normal(0, 0.003, (rows, cols // 64))).astype(np.float16)
        bi = (-7.5 * sc.astype(F32)).astype(np.float16)
        qt[src + name + ".q"], qt[src + name + ".scale"], qt[src + name + ".bias"] = ("U8", codes), ("F16", sc), ("F16", bi)
        want[name] = (codes, np.stack([sc, bi], axis=-1))
    norm = rng.normal(1, 0.1, synth.HIDDEN).astype(F32)
    qt[src + "input_layernorm.weight"] = ("F32", norm)
    convert.write_safetensors(str(tmp_path / "quant.safetensors"), qt)
    out = str(tmp_path / "m.ill")
    convert.convert(str(tmp_path), out, "q4", quant_file=str(tmp_path / "quant.safetensors"), sketch=True,
                    log=lambda s: None)
    r = ill.read_ill(out)
    L = r["layers"][0]
    assert np.array_equal(L["ln1"], norm)
    assert np.array_equal(L["wqkv"]["codes"][896:1024], want["self_attn.k_proj.weight"][0])
    assert np.array_equal(L["wgu"]["scales"][synth.FFN:], want["mlp.up_proj.weight"][1])
    assert np.array_equal(L["wd"]["codes"], want["mlp.down_proj.weight"][0])
    assert np.array_equal(r["embed"]["codes"], convert.quantize_q4(st.floats("model.embed_tokens.weight"))["codes"])
    raw = open(out, "rb").read()
    table = np.frombuffer(raw[16:16 + 16 * ill.COUNT], dtype=np.uint64).reshape(ill.COUNT, 2)
    o, n = int(table[ill.EMBED_HI, 0]), int(table[ill.EMBED_HI, 1])
    assert n == 256 * synth.HIDDEN // 4
    assert np.array_equal(np.frombuffer(raw[o:o + n], dtype=np.uint8).reshape(256, -1),
                          convert.sketch_q4(r["embed"]["codes"]))
    with pytest.raises(ValueError, match="use --format q4"):
        convert.convert(str(tmp_path), out, "q8", quant_file=str(tmp_path / "quant.safetensors"), log=lambda s: None)
