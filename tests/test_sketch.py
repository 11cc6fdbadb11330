"""The two-stage sketch lm_head (Shaders.swift:1377-1523): the CPU restatement's sketch layout and
bound property, then, on the GPU through the C ABI, the packed tile layout, stage 1's group bounds
against the restatement, and the tokens against the full lm_head (vp_head_argmax_noalloc) bit for
bit."""
import numpy as np
import pytest

from instantllm_b200 import convert, synth
from oracle import sketch as osk

VOCAB = 8192


def _embed(vocab=VOCAB, seed=41):
    return synth.make_matrix("q4", vocab, synth.HIDDEN, np.random.default_rng(seed))


def _rows(m, wnorm, rng, n):
    return synth.head_rows(m, wnorm, rng, n)


def test_unpack_matches_converter_sketch():
    m = _embed(256)
    hi = convert.sketch_q4(m["codes"])
    assert hi.shape == (256, 224)
    assert np.array_equal(osk.unpack_hi(hi), osk.unpack_q4(m["codes"]) >> 2)


def test_bound_holds_and_head_equals_full_argmax():
    """The exact q4 logit lies within K sigma of the sketch estimate for every row (the low code
    bits are uniform here, so the residual is close to normal with that sigma), and the two-stage
    argmax equals the full one."""
    rng = np.random.default_rng(42)
    m = _embed()
    hi = convert.sketch_q4(m["codes"])
    wn = rng.normal(1.0, 0.1, synth.HIDDEN).astype(np.float32)
    x = _rows(m, wn, rng, 8)
    r = osk.sketch_head(m["codes"], m["scales"], hi, wn, x, k=6.0)
    z = (r["logits"] - r["A"]) / r["sigma"]
    assert np.abs(z).max() < 6.0
    assert 0.9 < z.std() < 1.1  # sigma is the residual's standard deviation
    assert np.array_equal(r["tokens"], r["full"])
    assert r["cand"].sum(-1).max() < r["cand"].shape[1] // 10  # a handful of groups, not all


# ------------------------------------------------------------------------------------------------
# GPU, through the C ABI


def _pack_reference(hi):
    """The packed tile layout of vp_pack_sketch, restated: tile (rb, G) at (rb * 14 + G) * 256, lane
    L's 8 bytes at L * 8; byte b of word w holds k-step j = 2w + (b & 1), column parity b >> 1, and
    in bit pairs i = 0..3 the code of row gid + 8 (i & 1), column 16 j + 8 (i >> 1) + 2 tid4."""
    c = osk.unpack_hi(hi)
    V = c.shape[0]
    out = np.zeros((V // 16, 14, 32, 8), dtype=np.uint8)
    lane = np.arange(32)
    g, t4 = lane >> 2, lane & 3
    for w in range(2):
        for b in range(4):
            j, par = 2 * w + (b & 1), b >> 1
            for i in range(4):
                rows = (np.arange(V // 16)[:, None] * 16 + g[None, :] + 8 * (i & 1))  # [rb][lane]
                for G in range(14):
                    col = G * 64 + 16 * j + 8 * (i >> 1) + 2 * t4 + par  # [lane]
                    out[:, G, :, 4 * w + b] |= (c[rows, col[None, :]] << (2 * i)).astype(np.uint8)
    return out.reshape(-1)


@pytest.fixture(scope="module")
def gpu_setup():
    import torch

    from instantllm_b200.engine import VerifyEngine

    w = synth.make_weights("q4", n_layers=1, vocab=VOCAB, seed=43)
    rng = np.random.default_rng(43)
    w["final_norm"] = rng.normal(1.0, 0.1, synth.HIDDEN).astype(np.float32)
    eng = VerifyEngine(w, max_ctx=64, max_steps=8)
    yield eng, w, torch
    eng.close()


@pytest.mark.gpu
def test_pack_layout(gpu_setup):
    from instantllm_b200.sketch import SketchHead

    eng, w, torch = gpu_setup
    hi = convert.sketch_q4(w["embed"]["codes"])
    sk = SketchHead(eng, hi=hi)
    assert np.array_equal(sk.packed.cpu().numpy(), _pack_reference(hi))


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1, 3, 8, 9, 16])
def test_sketch_head_matches_full_head(gpu_setup, rows):
    import ctypes

    from instantllm_b200 import _lib
    from instantllm_b200.sketch import SketchHead

    eng, w, torch = gpu_setup
    sk = SketchHead(eng, codes=w["embed"]["codes"])
    rng = np.random.default_rng(100 + rows)
    x = _rows(w["embed"], w["final_norm"], rng, 16)
    xd = torch.from_numpy(x).to(eng.device)
    got = sk.argmax(xd, rows)

    full = torch.full((16,), -7, dtype=torch.int32, device=eng.device)
    rc = eng.lib.vp_head_argmax_noalloc(_lib.FMT["q4"], eng.vocab, eng._weights_struct.embed,
                                        eng._weights_struct.final_norm, xd.data_ptr(), rows,
                                        full.data_ptr(), eng.stream.cuda_stream)
    assert rc == 0, eng.lib.vp_last_error()
    assert np.array_equal(got, full[:rows].cpu().numpy())  # bit-identical recompute

    r = osk.sketch_head(w["embed"]["codes"], w["embed"]["scales"], convert.sketch_q4(w["embed"]["codes"]),
                        w["final_norm"], x[:rows], k=sk.k)
    assert np.array_equal(got, r["full"])  # the intended token (clear winners: no near ties)
    lb, ub = sk.last_bounds(rows)
    for a, b in ((lb, r["lb"]), (ub, r["ub"])):
        tol = 3e-3 * (np.abs(b) + np.abs(b).mean())  # fp16 rounding of the normed row differs
        assert np.all(np.abs(a - b) <= tol), np.abs(a - b).max()
    c0, call = sk.last_candidates()
    want0 = int(r["cand"][0].sum())
    assert abs(c0 - want0) <= 1 and 1 <= c0 <= call
    assert call <= int(r["cand"].any(0).sum()) + rows

    # rejected arguments
    assert eng.lib.vp_head_argmax_sketch(eng.vocab, eng._weights_struct.embed, sk.packed.data_ptr(),
                                         eng._weights_struct.final_norm, xd.data_ptr(), 17,
                                         ctypes.c_float(6.0), sk._work_ptr, sk._work_bytes,
                                         full.data_ptr(), None, eng.stream.cuda_stream) != 0
    assert eng.lib.vp_head_argmax_sketch(eng.vocab, eng._weights_struct.embed, sk.packed.data_ptr(),
                                         eng._weights_struct.final_norm, xd.data_ptr(), rows,
                                         ctypes.c_float(6.0), sk._work_ptr, 100,
                                         full.data_ptr(), None, eng.stream.cuda_stream) != 0


def test_sketch_head_rejects_bad_inputs_on_host():
    """Argument checks that run before any device work (a stub engine stands in)."""
    from instantllm_b200.sketch import SketchHead

    class Stub:
        fmt, vocab, embed_hi = "q8", 256, None

    with pytest.raises(ValueError, match="q4"):
        SketchHead(Stub())
    Stub.fmt = "q4"
    with pytest.raises(ValueError, match="no sketch plane"):
        SketchHead(Stub())
    with pytest.raises(ValueError, match="shape"):
        SketchHead(Stub(), hi=np.zeros((128, 224), dtype=np.uint8))
