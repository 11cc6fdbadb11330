"""The .ill container (ModelFile.swift / Convert.swift): header and table, tensor alignment and
page padding, the reference converter's stored row orders, and the round trip back to the standard
layouts the engine packs. CPU only."""
import struct

import numpy as np
import pytest

from instantllm_b200 import ill, synth


def _weights(fmt, n_layers=2, vocab=512, seed=3):
    w = synth.make_weights(fmt, n_layers=n_layers, vocab=vocab, seed=seed)
    rng = np.random.default_rng(seed)
    for L in w["layers"]:  # norms that differ per element, so that a swapped tensor shows
        L["ln1"] = rng.normal(1.0, 0.1, synth.HIDDEN).astype(np.float32)
        L["ln2"] = rng.normal(1.0, 0.1, synth.HIDDEN).astype(np.float32)
    w["final_norm"] = rng.normal(1.0, 0.1, synth.HIDDEN).astype(np.float32)
    return w


def _same_matrix(a, b):
    assert a["fmt"] == b["fmt"]
    for k in ("w", "codes", "scales"):
        if k in a:
            assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape, k
            assert np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k


@pytest.mark.parametrize("fmt", ["q4", "q8g32", "f16"])
def test_round_trip(fmt, tmp_path):
    w = _weights(fmt)
    path = str(tmp_path / "m.ill")
    ill.write_ill(path, w)
    r = ill.read_ill(path)
    assert r["fmt"] == fmt and r["n_layers"] == 2 and r["vocab"] == 512
    _same_matrix(w["embed"], r["embed"])
    assert np.array_equal(w["final_norm"], r["final_norm"])
    for a, b in zip(w["layers"], r["layers"]):
        for k in ("wqkv", "wo", "wgu", "wd"):
            _same_matrix(a[k], b[k])
        for k in ("ln1", "ln2", "bqkv"):
            assert np.array_equal(a[k], b[k]), k


def test_header_alignment_and_stored_order(tmp_path):
    w = _weights("q4", n_layers=1)
    path = str(tmp_path / "m.ill")
    ill.write_ill(path, w)
    raw = open(path, "rb").read()
    assert len(raw) % ill.PAGE_BYTES == 0
    magic, version, fmt, count = struct.unpack_from("<IIII", raw, 0)
    assert (magic, version, fmt, count) == (0x314D4C49, 1, 2, 292)
    table = np.frombuffer(raw[16:16 + 16 * count], dtype=np.uint64).reshape(count, 2)
    present = [t for t in range(count) if table[t, 1]]
    assert present == [0, 1, 2] + [3 + k for k in range(11)]
    assert all(int(table[t, 0]) % 256 == 0 and int(table[t, 0]) >= ill.HEADER_BYTES for t in present)
    offs = [int(table[t, 0]) for t in present]
    assert offs == sorted(offs)  # id order, no overlap
    for a, b in zip(present, present[1:]):
        assert int(table[a, 0]) + int(table[a, 1]) <= int(table[b, 0])

    def tensor(tid):
        o, n = int(table[tid, 0]), int(table[tid, 1])
        return np.frombuffer(raw[o:o + n], dtype=np.uint8)

    L = w["layers"][0]
    # QKV: stored row i = original row qkv_row_order()[i]; block 0 = head 0 dims 0-15 and 32-47
    qo = ill.qkv_row_order()
    assert list(qo[:4]) == [0, 1, 2, 3] and qo[16] == 32 and qo[32] == 16 and qo[64] == 64
    assert sorted(qo) == list(range(synth.QKV_ROWS))
    codes = tensor(ill.layer_id(0, ill.WQKV)).reshape(synth.QKV_ROWS, synth.HIDDEN // 2)
    for i in (0, 17, 40, 1151):
        assert np.array_equal(codes[i], L["wqkv"]["codes"][qo[i]])
    bias = tensor(ill.layer_id(0, ill.BQKV)).view(np.float32)
    assert np.array_equal(bias, L["bqkv"][qo])
    # gate/up: stored rows 4b + j = gate 2b, gate 2b + 1, up 2b, up 2b + 1
    gu = tensor(ill.layer_id(0, ill.WGU)).reshape(2 * synth.FFN, synth.HIDDEN // 2)
    F = synth.FFN
    for b in (0, 7, F // 2 - 1):
        want = [2 * b, 2 * b + 1, F + 2 * b, F + 2 * b + 1]
        for j in range(4):
            assert np.array_equal(gu[4 * b + j], L["wgu"]["codes"][want[j]])
    sb = tensor(ill.layer_id(0, ill.WGU_SB)).view(np.float16).reshape(2 * F, synth.HIDDEN // 64, 2)
    assert np.array_equal(sb[5], L["wgu"]["scales"][3]) and np.array_equal(sb[6], L["wgu"]["scales"][F + 2])


def test_rejects_what_the_reference_rejects(tmp_path):
    w = _weights("f16", n_layers=1, vocab=64)
    path = tmp_path / "m.ill"
    ill.write_ill(str(path), w)
    good = bytearray(path.read_bytes())
    for patch, msg in ((lambda b: b.__setitem__(slice(0, 4), b"XXXX"), "not an instantllm model"),
                       (lambda b: b.__setitem__(slice(4, 8), struct.pack("<I", 2)), "version"),
                       (lambda b: b.__setitem__(slice(8, 12), struct.pack("<I", 3)), "format"),
                       (lambda b: b.__setitem__(slice(12, 16), struct.pack("<I", 291)), "table")):
        bad = bytearray(good)
        patch(bad)
        p = tmp_path / "bad.ill"
        p.write_bytes(bytes(bad))
        with pytest.raises(ValueError, match=msg):
            ill.read_ill(str(p))
    p = tmp_path / "short.ill"
    p.write_bytes(bytes(good[:-100]))
    with pytest.raises(ValueError, match="bad size"):
        ill.read_ill(str(p))
    with pytest.raises(ValueError):
        ill.write_ill(str(tmp_path / "x.ill"), synth.make_weights("q8", n_layers=1, vocab=64))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["q4", "q8g32"])
def test_engine_from_ill_matches_direct(fmt, tmp_path):
    """An engine loaded from an .ill file runs the same pass, bit for bit, as one built on the same
    weights directly."""
    from instantllm_b200.engine import VerifyEngine

    w = _weights(fmt, n_layers=2, vocab=4096)
    path = str(tmp_path / "m.ill")
    ill.write_ill(path, w)
    prompt = (synth.make_prompt(40, seed=9) % 4096).tolist()
    out = []
    for eng in (VerifyEngine(w, max_ctx=256, max_steps=64), VerifyEngine.from_ill(path, max_ctx=256, max_steps=64)):
        eng.begin(0, 32)
        eng.prefill(prompt)
        first = eng.tokens(1)[0]
        tree = synth.seeded_tree(np.random.default_rng(9), [first] * 9, n=16, vocab=4096)
        eng.verify(tree)
        lg = eng.logits().cpu().numpy()
        eng.commit()
        out.append((first, lg, eng.tokens()))
        eng.close()
    assert out[0][0] == out[1][0]
    assert np.array_equal(out[0][1], out[1][1])
    assert out[0][2] == out[1][2]


def test_sketch_tensor_round_trip(tmp_path):
    """Tensor 291 (the 2-bit sketch of the q4 embedding) is read back as embed_hi; a sketch whose
    size does not fit the embedding, or one in a non-q4 file, is rejected."""
    from instantllm_b200 import convert

    w = _weights("q4", n_layers=1, vocab=256)
    hi = convert.sketch_q4(w["embed"]["codes"])
    path = str(tmp_path / "m.ill")
    ill.write_ill(path, w, embed_hi=hi)
    r = ill.read_ill(path)
    assert r["embed_hi"] is not None and np.array_equal(r["embed_hi"], hi)
    ill.write_ill(path, w)
    assert ill.read_ill(path)["embed_hi"] is None
    ill.write_ill(path, w, embed_hi=hi[:128])
    with pytest.raises(ValueError, match="sketch plane"):
        ill.read_ill(path)
