"""Build libvpass.so in-tree for sm_100a (nvcc cross-compiles without a GPU)."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
SOURCES = [PKG / "csrc" / "vpass.cu", PKG / "csrc" / "vpdraft.cu"]
HEADERS = sorted((PKG / "csrc").glob("*.cuh")) + [ROOT / "include" / "vpass.h"]
OUT = PKG / "libvpass.so"
# the trace build (performance work only): the same kernels with %globaltimer stamps at every stage
# step of one layer and of the lm_head (-DVP_TRACE_DETAIL), read by instantllm_b200.trace
TRACE_OUT = PKG / "libvpass_trace.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    # no --use_fast_math: the pass must be shape-invariant and close to the fp32 reference
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(cuda) / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def needs_build(out: Path = OUT) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> Path:
    out = TRACE_OUT if trace else OUT
    if not force and not needs_build(out):
        return out
    cmd = [nvcc(), *NVCC_FLAGS, *(["-DVP_TRACE_DETAIL"] if trace else []), "-o", str(out), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stdout + r.stderr)
    return out


if __name__ == "__main__":
    build(force=True, verbose=True)
    print(OUT)
