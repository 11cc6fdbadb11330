"""instantllm_b200: B200-native (sm_100a) speculative-decoding verification pass for the
Qwen2.5-0.5B architecture, a drop-in for the prefill / tree-verify / commit path of instantllm.

The compute lives in libvpass.so (hand-written CUDA, C ABI in include/vpass.h); this package holds
the host side: the ctypes binding (_lib), the Engine-like driver (engine.VerifyEngine), seeded
synthetic inputs (synth) and the in-tree build (build).
"""
from . import synth  # noqa: F401

__all__ = ["synth", "engine", "build"]
