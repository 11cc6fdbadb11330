"""The C ABI library (no GPU needed): it builds for sm_100a, loads, exports every function that
include/vpass.h declares, and rejects bad arguments before touching a device."""
import ctypes
import re

import pytest

from instantllm_b200 import _lib, build
from instantllm_b200.synth import HIDDEN


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_functions():
    text = (build.ROOT / "include" / "vpass.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vp_[a-z_]+)\s*\(", text)))


def test_header_matches_binding():
    assert declared_functions() == sorted(_lib.EXPORTS)


def test_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_packed_bytes(lib):
    assert lib.vp_packed_bytes(2, 1152, 896) == 72 * 14 * 576
    assert lib.vp_packed_bytes(1, 896, 4864) == 56 * 76 * 1056
    assert lib.vp_packed_bytes(0, 896, 896) == 56 * 14 * 2048
    # q4 tiles hold exactly the standard bytes: codes + (scale, min) pairs
    assert lib.vp_packed_bytes(2, 16, 64) == 16 * 32 + 16 * 4
    assert lib.vp_packed_bytes(2, 17, 64) == 0
    assert lib.vp_packed_bytes(2, 16, 65) == 0
    assert lib.vp_packed_bytes(9, 16, 64) == 0


def test_argument_errors_without_device(lib):
    cfg = _lib.VpConfig(7, 24, 151936, 4096, 64, 0)
    ctx = ctypes.c_void_p()
    assert lib.vp_create(ctypes.byref(cfg), ctypes.byref(ctx)) == -1
    assert b"format" in lib.vp_last_error()
    cfg = _lib.VpConfig(2, 0, 151936, 4096, 64, 0)
    assert lib.vp_create(ctypes.byref(cfg), ctypes.byref(ctx)) == -1
    cfg = _lib.VpConfig(2, 24, 151930, 4096, 64, 0)
    assert lib.vp_create(ctypes.byref(cfg), ctypes.byref(ctx)) == -1
    assert lib.vp_pack_matrix(2, 1, 1000, HIDDEN, None, None, None, None) == -1
    assert lib.vp_pack_matrix(2, 0, 16, 64, None, None, None, None) == -1
    assert lib.vp_prefill(None, None, 1, None) == -1
    assert lib.vp_verify(None, None, None) == -1
    assert lib.vp_pass(None, None, None) == -1
    assert lib.vp_pass_multi(None, None, 1, None) == -1
    assert lib.vp_pass_batch(None, None, 1, 4, None) == -1
    assert lib.vp_prefill_batch(None, None, None, 1, 4, None) == -1
    assert lib.vp_commit(None, None) == -1
    st = _lib.VpState()
    assert lib.vp_read_state(None, ctypes.byref(st), None) == -1
    assert lib.vp_device_tokens(None) is None


def test_step_and_sketch_argument_errors_without_device(lib):
    """vp_step and the sketch head reject bad arguments before any CUDA call."""
    st = _lib.VpState()
    tree = (ctypes.c_int32 * _lib.TREE_INTS)()
    assert lib.vp_step(None, None, tree, ctypes.byref(st), None, None) == -1
    assert b"null context" in lib.vp_last_error()
    assert lib.vp_sketch_bytes(100) == 0 and lib.vp_sketch_work_bytes(0) == 0
    assert lib.vp_sketch_bytes(151936) == 151936 // 16 * 14 * 256
    assert lib.vp_sketch_bounds_offset() % 256 == 0
    assert lib.vp_pack_sketch(100, None, None, None) == -1
    d = ctypes.c_void_p(256)  # never dereferenced: every call below fails its checks first
    tok = ctypes.c_void_p(512)
    assert lib.vp_head_argmax_sketch(100, d, d, d, d, 1, ctypes.c_float(6.0), d, 1 << 20, tok, None, None) == -1
    assert lib.vp_head_argmax_sketch(4096, d, d, d, d, 0, ctypes.c_float(6.0), d, 1 << 20, tok, None, None) == -1
    assert lib.vp_head_argmax_sketch(4096, d, d, d, d, 1, ctypes.c_float(0.0), d, 1 << 20, tok, None, None) == -1
    assert b"k_sigma" in lib.vp_last_error()
    assert lib.vp_head_argmax_sketch(4096, d, d, d, d, 1, ctypes.c_float(6.0), d, 16, tok, None, None) == -1
    assert b"work buffer" in lib.vp_last_error()
    assert lib.vp_head_argmax_noalloc(2, 4100, d, d, d, 1, tok, None) == -1


def test_graph_argument_errors_without_device(lib):
    """The CUDA-graph entry points reject null arguments before any CUDA call."""
    out = ctypes.c_void_p()
    d = ctypes.c_void_p(256)  # never dereferenced
    assert lib.vp_pass_graph(None, d, ctypes.byref(out)) == -1 and out.value is None
    assert lib.vp_pass_graph(d, None, ctypes.byref(out)) == -1
    assert lib.vp_step_graph(None, d, 15, 8, ctypes.byref(out)) == -1
    assert lib.vp_step_graph(d, None, 15, 8, ctypes.byref(out)) == -1
    assert lib.vp_graph_launch(None, None) == -1
    assert b"null graph" in lib.vp_last_error()
    lib.vp_graph_destroy(None)  # no-op
