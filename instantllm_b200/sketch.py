"""Two-stage lm_head over the 2-bit sketch of the q4 embedding: the reference's optional sketch head
(Engine.useSketchHead / encodeSketchHead, Sources/Engine/Engine.swift:34-39 and 436-454; kernels
k_lmh_sketch_T, k_lmh_tau, k_lmh_exact_T, Shaders.swift:1377-1523), through the C ABI
(vp_pack_sketch, vp_head_argmax_sketch).

Stage 1 scores every vocabulary row from the high two bits of its q4 codes and an uncertainty
sigma for the dropped low bits; stage 2 recomputes exact logits only in the 32-row groups whose
upper bound reaches the best lower bound. The argmax equals the full lm_head's
(vp_head_argmax_noalloc) unless a residual exceeds K sigma, so, as in the reference, it is off by
default and probabilistic: a caller opts in by building a SketchHead.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from ._lib import check

DEFAULT_K = 6.0  # Engine.sketchK (ILL_SKETCH_K), Engine.swift:39
GROUP = 32       # vocabulary rows per bound group


class SketchHead:
    """The sketch head over a q4 VerifyEngine's embedding.

    hi: the reference's sketch plane, uint8 [vocab][224] (.ill tensor 291, convert --sketch);
    if None, engine.embed_hi (read from the model file) is used, else it is computed from `codes`
    (the standard q4 embedding codes, uint8 [vocab][448])."""

    def __init__(self, engine, hi: Optional[np.ndarray] = None, codes: Optional[np.ndarray] = None,
                 k: float = DEFAULT_K):
        if engine.fmt != "q4":
            raise ValueError("the sketch head reads the 2-bit sketch of a q4 embedding")
        if hi is None:
            hi = getattr(engine, "embed_hi", None)
        if hi is None and codes is not None:
            from .convert import sketch_q4

            hi = sketch_q4(np.asarray(codes, dtype=np.uint8))
        if hi is None:
            raise ValueError("no sketch plane: convert the model with --sketch or pass the embedding codes")
        hi = np.ascontiguousarray(hi, dtype=np.uint8)
        V = engine.vocab
        if hi.shape != (V, 896 // 4):
            raise ValueError(f"sketch plane of shape {hi.shape}, expected ({V}, 224)")
        self.eng, self.lib, self.k = engine, engine.lib, float(k)
        self.vocab, self.ngrp = V, (V + GROUP - 1) // GROUP
        dev, s = engine.device, engine.stream.cuda_stream
        src = torch.from_numpy(hi).to(dev)
        self.packed = torch.empty(self.lib.vp_sketch_bytes(V), dtype=torch.uint8, device=dev)
        check(self.lib.vp_pack_sketch(V, src.data_ptr(), self.packed.data_ptr(), s), "vp_pack_sketch")
        nb = self.lib.vp_sketch_work_bytes(V)
        self.work = torch.empty(nb + 256, dtype=torch.uint8, device=dev)
        base = self.work.data_ptr()
        self._work_ptr = (base + 255) & ~255
        self._work_shift = self._work_ptr - base
        self._work_bytes = nb
        self.tokens_dev = torch.empty(16, dtype=torch.int32, device=dev)
        self.ncand_dev = torch.zeros(2, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)  # the staging copy of `hi` may be freed after this

    def argmax_device(self, x: torch.Tensor, rows: Optional[int] = None) -> torch.Tensor:
        """Greedy tokens of the first `rows` rows of x (fp32 [>= rows][896] on the engine's device),
        as a device int32 tensor [rows]; no synchronisation."""
        rows = x.shape[0] if rows is None else rows
        if x.dtype != torch.float32 or x.device != self.eng.device or not x.is_contiguous():
            raise ValueError("x must be a contiguous fp32 tensor on the engine's device")
        w = self.eng._weights_struct
        check(self.lib.vp_head_argmax_sketch(
            self.vocab, w.embed, self.packed.data_ptr(), w.final_norm, x.data_ptr(), rows,
            ctypes.c_float(self.k), self._work_ptr, self._work_bytes, self.tokens_dev.data_ptr(),
            self.ncand_dev.data_ptr(), self.eng.stream.cuda_stream), "vp_head_argmax_sketch")
        return self.tokens_dev[:rows]

    def argmax(self, x: torch.Tensor, rows: Optional[int] = None) -> np.ndarray:
        return self.argmax_device(x, rows).cpu().numpy()

    def last_candidates(self) -> tuple:
        """(groups that were candidates for row 0, for any row) of the last call
        (Engine.lastSketchCandidates counts the first)."""
        c = self.ncand_dev.cpu().numpy()
        return int(c[0]), int(c[1])

    def last_bounds(self, rows: int) -> tuple:
        """(lower, upper) group bounds fp32 [rows][ngrp] of the last call."""
        off = self.lib.vp_sketch_bounds_offset()
        n = 2 * 16 * self.ngrp
        o = self._work_shift + off
        b = self.work[o:o + 4 * n].view(torch.float32).cpu().numpy().reshape(2, 16, self.ngrp)
        return b[0, :rows], b[1, :rows]
