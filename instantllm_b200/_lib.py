"""ctypes binding of libvpass.so (include/vpass.h). Fails loudly if the library is missing: there is
no CPU fallback on the product path."""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libvpass.so"

MAX_LAYERS = 24
TREE_INTS = 65
FMT = {"f16": 0, "q8": 1, "q4": 2, "q8g32": 3}
MAT_PLAIN, MAT_QKV, MAT_GATEUP = 0, 1, 2

# every symbol include/vpass.h declares
EXPORTS = (
    "vp_packed_bytes", "vp_pack_matrix", "vp_create", "vp_destroy", "vp_set_weights",
    "vp_last_error", "vp_begin", "vp_prefill", "vp_verify", "vp_verify_chain", "vp_commit",
    "vp_pass", "vp_pass_multi", "vp_pass_batch", "vp_prefill_batch", "vp_step", "vp_read_state", "vp_write_state", "vp_prefix_bytes", "vp_save_prefix", "vp_load_prefix",
    "vp_read_tokens", "vp_device_tokens", "vp_device_state",
    "vp_debug_logits", "vp_buffer", "vp_head_argmax_noalloc",
    "vp_sketch_bytes", "vp_pack_sketch", "vp_sketch_work_bytes", "vp_sketch_bounds_offset",
    "vp_head_argmax_sketch", "vp_drafter_create", "vp_drafter_destroy", "vp_drafter_begin", "vp_draft",
    "vp_pass_graph", "vp_step_graph", "vp_graph_launch", "vp_graph_destroy",
)


class VpConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("format", "n_layers", "vocab", "max_ctx", "max_steps", "device")]


STATE_FIELDS = ("pos", "n", "step", "done", "maxctx", "maxsteps", "eos0", "eos1", "nver", "vrow0",
                "passes", "accepted", "err", "last_token", "mode", "advance")


class VpState(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in STATE_FIELDS]

    def as_dict(self) -> dict:
        return {n: int(getattr(self, n)) for n in STATE_FIELDS}


_P = ctypes.c_void_p
_ARR = _P * MAX_LAYERS


class VpWeights(ctypes.Structure):
    _fields_ = [("embed", _P), ("final_norm", _P), ("wqkv", _ARR), ("bqkv", _ARR), ("wo", _ARR),
                ("wgu", _ARR), ("wd", _ARR), ("ln1", _ARR), ("ln2", _ARR)]


class VpError(RuntimeError):
    pass


_lib = None


def load(path: os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and type the library. Raises if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise VpError(f"{p} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                      "(instantllm_b200.build). There is no CPU fallback.")
    lib = ctypes.CDLL(str(p))
    i32, sz, vp = ctypes.c_int32, ctypes.c_size_t, ctypes.c_void_p
    sig = {
        "vp_packed_bytes": (sz, [i32, i32, i32]),
        "vp_pack_matrix": (ctypes.c_int, [i32, i32, i32, i32, vp, vp, vp, vp]),
        "vp_create": (ctypes.c_int, [ctypes.POINTER(VpConfig), ctypes.POINTER(vp)]),
        "vp_destroy": (None, [vp]),
        "vp_set_weights": (ctypes.c_int, [vp, ctypes.POINTER(VpWeights)]),
        "vp_last_error": (ctypes.c_char_p, []),
        "vp_begin": (ctypes.c_int, [vp, i32, i32, i32, i32, vp]),
        "vp_prefill": (ctypes.c_int, [vp, vp, i32, vp]),
        "vp_verify": (ctypes.c_int, [vp, vp, vp]),
        "vp_verify_chain": (ctypes.c_int, [vp, vp, i32, vp]),
        "vp_commit": (ctypes.c_int, [vp, vp]),
        "vp_pass": (ctypes.c_int, [vp, vp, vp]),
        "vp_pass_multi": (ctypes.c_int, [ctypes.POINTER(vp), ctypes.POINTER(vp), i32, vp]),
        "vp_pass_batch": (ctypes.c_int, [ctypes.POINTER(vp), ctypes.POINTER(vp), i32, i32, vp]),
        "vp_prefill_batch": (ctypes.c_int, [ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(i32), i32, i32, vp]),
        "vp_step": (ctypes.c_int, [vp, ctypes.c_void_p, vp, ctypes.POINTER(VpState), vp, vp]),
        "vp_read_state": (ctypes.c_int, [vp, ctypes.POINTER(VpState), vp]),
        "vp_write_state": (ctypes.c_int, [vp, ctypes.c_void_p, ctypes.c_int32, vp]),
        "vp_prefix_bytes": (ctypes.c_size_t, [vp, ctypes.c_int32]),
        "vp_save_prefix": (ctypes.c_int, [vp, ctypes.c_int32, ctypes.c_void_p, vp]),
        "vp_load_prefix": (ctypes.c_int, [vp, ctypes.c_int32, ctypes.c_void_p, vp]),
        "vp_read_tokens": (ctypes.c_int, [vp, vp, i32, vp]),
        "vp_device_tokens": (vp, [vp]),
        "vp_device_state": (vp, [vp]),
        "vp_debug_logits": (ctypes.c_int, [vp, vp, vp]),
        "vp_buffer": (ctypes.c_int, [vp, i32, ctypes.POINTER(vp), ctypes.POINTER(sz)]),
        "vp_head_argmax_noalloc": (ctypes.c_int, [i32, i32, vp, vp, vp, i32, vp, vp]),
        "vp_sketch_bytes": (sz, [i32]),
        "vp_pack_sketch": (ctypes.c_int, [i32, vp, vp, vp]),
        "vp_sketch_work_bytes": (sz, [i32]),
        "vp_sketch_bounds_offset": (sz, []),
        "vp_head_argmax_sketch": (ctypes.c_int, [i32, vp, vp, vp, vp, i32, ctypes.c_float, vp, sz, vp, vp, vp]),
        "vp_drafter_create": (ctypes.c_int, [vp, sz, i32, ctypes.POINTER(vp)]),
        "vp_drafter_destroy": (None, [vp]),
        "vp_drafter_begin": (ctypes.c_int, [vp, vp]),
        "vp_draft": (ctypes.c_int, [vp, vp, vp, i32, i32, i32, vp, vp, vp]),
        "vp_pass_graph": (ctypes.c_int, [vp, vp, ctypes.POINTER(vp)]),
        "vp_step_graph": (ctypes.c_int, [vp, vp, i32, i32, ctypes.POINTER(vp)]),
        "vp_graph_launch": (ctypes.c_int, [vp, vp]),
        "vp_graph_destroy": (None, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = load().vp_last_error()
        raise VpError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")
