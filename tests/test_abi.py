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
    assert lib.vp_commit(None, None) == -1
    st = _lib.VpState()
    assert lib.vp_read_state(None, ctypes.byref(st), None) == -1
    assert lib.vp_device_tokens(None) is None
