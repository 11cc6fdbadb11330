"""vp_head_argmax_noalloc: the greedy lm-head argmax for callers that may not allocate device memory
(their device memory belongs to a host pool or budget, or a cudaMalloc would stall a serving loop).
Its scratch is a static device array in the library, so this checks, through the C ABI, that two
calls in a row (the second one reusing the first one's scratch) give the same tokens as the
context-based entry point, vp_debug_logits followed by argmax, on the same residual rows. Both run
the same GEMM arithmetic and break ties towards the lowest id, so the ids must be equal; the token
slots past `rows` must stay untouched."""
import ctypes

import numpy as np
import pytest
import torch

from instantllm_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _reference_ids(eng):
    lg = eng.logits().cpu().numpy()
    return lg, lg.argmax(axis=1)  # first maximum = lowest id on ties


def _noalloc(lib, eng, x, rows):
    out = torch.full((16,), -7, dtype=torch.int32, device=eng.device)
    w = eng._weights_struct
    rc = lib.vp_head_argmax_noalloc(_lib.FMT[eng.fmt], eng.vocab, w.embed, w.final_norm, x.data_ptr(),
                                    rows, out.data_ptr(), eng.stream.cuda_stream)
    assert rc == 0, lib.vp_last_error()
    o = out.cpu().numpy()
    assert (o[rows:] == -7).all(), o  # slots past `rows` are not written
    return o[:rows]


def _check(lg, ref, got):
    assert np.array_equal(ref, got), (ref, got)


def test_noalloc_argmax_matches_context_entry_point():
    from instantllm_b200.engine import VerifyEngine

    lib = _lib.load()
    w = synth.make_weights("q4", n_layers=2, seed=31)
    eng = VerifyEngine(w, max_ctx=512, max_steps=64)
    prompt = synth.make_prompt(20, seed=31).tolist()
    eng.begin(0, 32)
    eng.prefill(prompt)
    first = eng.tokens(1)[0]
    rng = np.random.default_rng(31)

    # call 1: the 16 rows of a tree pass
    eng.verify(synth.seeded_tree(rng, [first] * 9, n=16))
    x1 = eng.buffer(0, (16, 896), "<f4").clone()
    lg1, ref1 = _reference_ids(eng)
    got1 = _noalloc(lib, eng, x1, 16)
    _check(lg1, ref1, got1)

    # call 2, right after: other rows, fewer of them; stale scratch from call 1 must not leak
    eng.verify(synth.seeded_tree(rng, [first + 1] * 9, n=16))
    x2 = eng.buffer(0, (16, 896), "<f4").clone()
    lg2, ref2 = _reference_ids(eng)
    got2 = _noalloc(lib, eng, x2, 11)
    _check(lg2[:11], ref2[:11], got2)
    assert not np.array_equal(ref1, ref2)

    # sizes past the stated limits are refused before any device work
    out = torch.zeros(32, dtype=torch.int32, device=eng.device)
    assert lib.vp_head_argmax_noalloc(2, eng.vocab, w_ptr(eng), fn_ptr(eng), x2.data_ptr(), 17,
                                      out.data_ptr(), None) == -1
    assert lib.vp_head_argmax_noalloc(2, 163856, w_ptr(eng), fn_ptr(eng), x2.data_ptr(), 4,
                                      out.data_ptr(), None) == -1
    eng.close()


def w_ptr(eng):
    return eng._weights_struct.embed


def fn_ptr(eng):
    return eng._weights_struct.final_norm
