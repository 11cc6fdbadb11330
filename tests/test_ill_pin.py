"""The .ill container and the Hugging Face converter pinned to bytes derived by hand from the
reference's source (Sources/Engine/ModelFile.swift, Sources/Engine/Convert.swift), not from this
package's code. The reference is Swift and cannot run here, so every expected value below is worked
out in its comment from the cited lines, on inputs chosen so that the arithmetic is exact.
CPU only."""
import struct

import numpy as np
import pytest

from instantllm_b200 import convert, ill, synth

F32 = np.float32

# quantGroup (Convert.swift:323-370) on w[i] = 0.25 + 0.125 (i mod 16), i < 64:
#  min 0.25, max 2.125. The first clip pair (0, 0) gives lo 0.25, hi 2.125, s = 1.875 / 15 = 0.125,
#  b = 0.25; round((w - b) / s) = i mod 16 exactly. The least-squares refit (:345-352) has
#  sum q = 480, sum w = 76, sum q^2 = 4960, sum q w = 740 (all exact in fp32), den = 64*4960 - 480^2
#  = 87040, s2 = (64*740 - 480*76) / 87040 = 0.125, b = (76 - 0.125*480) / 64 = 0.25: unchanged. Both
#  are fp16-exact, the error is 0, and no later pair can beat 0 (`err < bestErr`, :366).
#  Codes i mod 16, packed two per byte with the even column low (:316): 0x10 0x32 ... 0xFE, four
#  times. fp16 0.125 = 0x3000, 0.25 = 0x3400, stored as (scale, bias) (:312-313).
LINEAR_GROUP = F32(0.25) + F32(0.125) * (np.arange(64) % 16).astype(F32)
LINEAR_BYTES = bytes([0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE] * 4)
LINEAR_SB = (0x3000, 0x3400)

# A flat group (all 0.5): max - min < 1e-12 (:326-329) -> codes 0, scale 0, bias fp16(0.5) = 0x3800.
FLAT_GROUP = np.full(64, 0.5, dtype=F32)
FLAT_SB = (0x0000, 0x3800)

# quantizeQ8 (Convert.swift:254-282), group 32.
# (a) w = k / 128 with |k| <= 127 and some |k| = 127: amax / 127 = 2^-7 exactly, fp16 0x2000;
#     2^-7 * 127 = amax is not below amax, so no bump (:272); codes round(w * 128) = k.
Q8_K = np.array([127, -127, 0, 1, -1, 64, -64, 100, -3, 5, 17, -17, 33, 90, -90, 2] * 2)
Q8_EXACT_SCALE = 0x2000
# (b) amax 1.0: 1 / 127 = 0.0078740157 lies in [2^-7, 2^-6) where fp16 steps by 2^-17; it is
#     8.06 steps above 2^-7, so fp16 rounds to 2^-7 + 8 * 2^-17 = 0.00787353515625, and
#     127 times that is 0.99993896 < 1.0: the scale is raised one ulp (:272) to 2^-7 + 9 * 2^-17 =
#     0.0078811645507812, bits 0x2000 | 9 = 0x2009. 1 / s = 126.8848: 1.0 -> 126.88 -> 127,
#     0.5 -> 63.44 -> 63, -0.25 -> -31.72 -> -32 (half away from zero), -1.0 -> -127,
#     0.125 -> 15.86 -> 16, 0 -> 0.
Q8_BUMP_W = np.array([1.0, 0.5, -0.25, 0.0, -1.0, 0.125] + [0.0] * 26, dtype=F32)
Q8_BUMP_CODES = [127, 63, -32, 0, -127, 16] + [0] * 26
Q8_BUMP_SCALE = 0x2009


def test_q4_groups_hand_derived():
    q, s, b = convert._q4_groups(np.stack([LINEAR_GROUP, FLAT_GROUP]))
    assert list(q[0]) == [i % 16 for i in range(64)]
    assert (int(s[0].view(np.uint16)), int(b[0].view(np.uint16))) == LINEAR_SB
    assert list(q[1]) == [0] * 64
    assert (int(s[1].view(np.uint16)), int(b[1].view(np.uint16))) == FLAT_SB
    m = convert.quantize_q4(np.stack([np.r_[LINEAR_GROUP, FLAT_GROUP]]))
    assert m["codes"][0].tobytes() == LINEAR_BYTES + bytes(32)
    assert list(m["scales"][0].reshape(-1).view(np.uint16)) == [*LINEAR_SB, *FLAT_SB]


def test_q8_groups_hand_derived():
    codes, s = convert.quantize_q8(np.stack([np.r_[Q8_K.astype(F32) / F32(128), Q8_BUMP_W]]))
    assert list(codes[0, :32]) == list(Q8_K) and list(codes[0, 32:]) == Q8_BUMP_CODES
    assert list(s[0].view(np.uint16)) == [Q8_EXACT_SCALE, Q8_BUMP_SCALE]


def test_row_orders_hand_derived():
    # qkvRowOrder (Convert.swift:331-340): block b of 32 stored rows = head b / 2, half b % 2:
    # original rows 64 head + 16 half + i, then 64 head + 32 + 16 half + i, i < 16.
    qo = ill.qkv_row_order()
    assert list(qo[:64]) == list(range(0, 16)) + list(range(32, 48)) + list(range(16, 32)) + list(range(48, 64))
    assert list(qo[64:80]) == list(range(64, 80)) and list(qo[80:96]) == list(range(96, 112))
    assert list(qo[-32:]) == list(range(1104, 1120)) + list(range(1136, 1152))
    # guOrder (Convert.swift:132-133): for b < F / 2: 2b, 2b + 1, F + 2b, F + 2b + 1
    F = synth.FFN
    go = ill.gu_row_order()
    assert list(go[:8]) == [0, 1, F, F + 1, 2, 3, F + 2, F + 3]
    assert list(go[-4:]) == [F - 2, F - 1, 2 * F - 2, 2 * F - 1]


def _checkpoint(path, vocab=32):
    """A one-layer BF16 checkpoint whose embedding row 0 starts with the linear group and whose
    row 1 starts with the flat group (both exact in BF16)."""
    rng = np.random.default_rng(11)
    H, Fd = synth.HIDDEN, synth.FFN
    emb = rng.normal(0, 0.02, (vocab, H)).astype(F32)
    emb[0, :64], emb[1, :64] = LINEAR_GROUP, FLAT_GROUP
    t = {"model.embed_tokens.weight": ("BF16", emb), "model.norm.weight": ("BF16", np.ones(H, F32))}
    p = "model.layers.0."
    t[p + "input_layernorm.weight"] = ("BF16", np.ones(H, F32))
    t[p + "post_attention_layernorm.weight"] = ("BF16", np.ones(H, F32))
    for x, r in (("q", 896), ("k", 128), ("v", 128)):
        t[p + f"self_attn.{x}_proj.weight"] = ("BF16", rng.normal(0, 0.02, (r, H)))
        t[p + f"self_attn.{x}_proj.bias"] = ("BF16", np.arange(r, dtype=F32) / 1024)
    t[p + "self_attn.o_proj.weight"] = ("BF16", rng.normal(0, 0.02, (H, H)))
    t[p + "mlp.gate_proj.weight"] = ("BF16", rng.normal(0, 0.02, (Fd, H)))
    t[p + "mlp.up_proj.weight"] = ("BF16", rng.normal(0, 0.02, (Fd, H)))
    t[p + "mlp.down_proj.weight"] = ("BF16", rng.normal(0, 0.02, (H, Fd)))
    convert.write_safetensors(str(path / "model.safetensors"), t)


def test_converted_file_bytes_hand_derived(tmp_path):
    """A q4 conversion read back as raw bytes (ModelFile.swift:62-64, 115-144; Convert.swift:90-215)."""
    _checkpoint(tmp_path)
    out = tmp_path / "m.ill"
    convert.convert(str(tmp_path), str(out), "q4", log=lambda s: None)
    raw = out.read_bytes()
    # header: magic "ILM1" (0x314D4C49), version 1, format 2 (q4), tensor count 3 + 24 * 12 + 1 = 292
    assert raw[:16] == bytes([0x49, 0x4C, 0x4D, 0x31, 1, 0, 0, 0, 2, 0, 0, 0, 0x24, 0x01, 0, 0])
    assert len(raw) % 16384 == 0
    table = struct.unpack_from("<584Q", raw, 16)
    ent = [(table[2 * i], table[2 * i + 1]) for i in range(292)]
    H, Fd = synth.HIDDEN, synth.FFN
    # tensor 0, the first written, sits at the end of the 16 KiB header; q4 codes are rows x cols / 2
    # bytes, the (scale, bias) pairs rows x cols / 64 x 4 bytes; every offset is 256-byte aligned
    # and tensors follow in id order (ModelWriter.write, :122-128)
    assert ent[0] == (16384, 32 * H // 2)
    assert ent[1] == (16384 + 32 * H // 2, 32 * (H // 64) * 4)  # 14336 is already 256-aligned
    assert ent[2][1] == H * 4  # final norm, f32
    # layer 0 at ids 3 + k (TensorID.layer, ModelFile.swift:59): QKV codes 1152 x 448 bytes, QKV bias
    # 1152 f32, gate/up 9728 rows, down 896 x 4864 / 2; layers 1..23 and the sketch (291) absent
    assert ent[3 + 1][1] == 1152 * H // 2 and ent[3 + 3][1] == 1152 * 4
    assert ent[3 + 7][1] == 2 * Fd * H // 2 and ent[3 + 9][1] == H * Fd // 2
    assert all(ent[i] == (0, 0) for i in range(15, 292))
    offs = [o for o, n in ent if n]
    assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)
    # embedding row 0 starts with the linear group, row 1 with the flat group
    o0, o1 = ent[0][0], ent[1][0]
    assert raw[o0:o0 + 32] == LINEAR_BYTES
    assert raw[o0 + H // 2:o0 + H // 2 + 32] == bytes(32)
    sb = struct.unpack_from("<2H", raw, o1) + struct.unpack_from("<2H", raw, o1 + (H // 64) * 4)
    assert sb == LINEAR_SB + FLAT_SB
    # QKV bias stored in qkvRowOrder (Convert.swift:178): stored entry 16 = original row 32 (q head 0
    # dim 32), bias value 32 / 1024
    ob = ent[3 + 3][0]
    assert struct.unpack_from("<f", raw, ob + 16 * 4)[0] == pytest.approx(32 / 1024, abs=0)
