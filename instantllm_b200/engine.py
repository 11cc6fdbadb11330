"""VerifyEngine: host side of the verification pass, mirroring the reference's Engine operator
surface (Sources/Engine/Engine.swift) on top of the C ABI (include/vpass.h).

    Engine.init(modelPath:...)          -> VerifyEngine(weights, max_ctx=..., max_steps=...)
    generate() state init  (:937-964)   -> begin(cached, max_new, eos)
    encodePrefill          (:588-601)   -> prefill(tokens)
    encodeWidePass         (:567-579)   -> verify(tree) / verify_chain(drafts)
    encodeCommitSpec       (:484-497)   -> commit()
    wide pass + commit as one unit      -> pass_(tree)    (one persistent-kernel launch)
    generate()             (:922-1038)  -> generate(prompt, max_new, tree_fn)

PyTorch only provides device memory and the stream; all compute is the CUDA library.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import numpy as np
import torch

from . import _lib
from ._lib import FMT, MAT_GATEUP, MAT_PLAIN, MAT_QKV, VpConfig, VpState, VpWeights, check
from .synth import STOP_IDS, TREE_INTS, tree_to_buffer


class _DevArray:
    """Zero-copy torch view of a raw device pointer (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2}


def _np_to_dev(a: np.ndarray, device) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if not a.flags.writeable:  # torch.from_numpy wants a writable buffer (read-only views warn)
        a = a.copy()
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    return torch.from_numpy(a.view(np.uint8).reshape(-1)).to(device)


class Graph:
    """A replayable CUDA graph made by the library (vp_pass_graph, vp_step_graph): launch() replays
    it on a stream; close() (or garbage collection) destroys it. Destroy it before its engine or
    drafter."""

    def __init__(self, lib, handle: ctypes.c_void_p):
        self.lib, self.h = lib, handle

    def launch(self, stream: int) -> None:
        check(self.lib.vp_graph_launch(self.h, stream), "vp_graph_launch")

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.vp_graph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PassShape:
    """Adaptive speculation (Engine.nextPassShape, Engine.swift:878-898): the next pass verifies the
    configured best-first tree (tree_b drafts, 8 children per expansion) while at least adapt_hi
    drafts per pass were accepted over the last few committed passes, and an 8-row chain below
    that rate (unpredictable text). A chain is the drafter's tree search with one child per
    expansion. Both shapes run through the same pass kernel, whose numerics agree for every row
    count, so the output stays that of plain greedy decoding. (The reference's adaptLo tier of
    3-row shader passes has no counterpart: one kernel serves every row count here.)"""

    def __init__(self, tree_b: int = 15, chain_rows: int = 8, adaptive: bool = True, adapt_hi: float = 1.5):
        if not 1 <= tree_b <= 15 or not 2 <= chain_rows <= 16:
            raise ValueError("tree_b must be 1..15 and chain_rows 2..16")
        self.tree_b, self.chain_rows, self.adaptive, self.adapt_hi = tree_b, chain_rows, adaptive, adapt_hi
        self.hist = []

    def reset(self) -> None:
        self.hist.clear()

    def next(self, passes: int, accepted: int):
        """(drafts B, children per expansion) of the next pass, from the request's committed pass
        and accepted-draft counters as last seen by the host."""
        tree = (self.tree_b, 8)
        if not self.adaptive:
            return tree
        if not self.hist or self.hist[-1][0] != passes:
            self.hist.append((passes, accepted))
        if len(self.hist) < 3:
            return tree
        p0, a0 = self.hist[-4:][0]
        if passes - p0 < 2:
            return tree
        if (accepted - a0) / (passes - p0) >= self.adapt_hi:
            return tree
        return (self.chain_rows - 1, 1)


class VerifyEngine:
    def __init__(self, weights: dict, max_ctx: int = 4096, max_steps: int = 4096, device: int = 0):
        self.lib = _lib.load()
        self.device = torch.device("cuda", device)
        torch.cuda.set_device(self.device)
        self.fmt = weights["fmt"]
        if self.fmt not in FMT:
            raise ValueError(f"the GPU path runs q4, q8 or f16 weights, not {self.fmt}")
        self.n_layers = weights["n_layers"]
        self.vocab = weights["vocab"]
        self.embed_hi = weights.get("embed_hi")  # optional 2-bit sketch plane (sketch.SketchHead)
        self.max_ctx, self.max_steps = max_ctx, max_steps
        self._keep = []
        self._staging = []
        self.stream = torch.cuda.current_stream(self.device)
        w = VpWeights()
        w.embed = self._pack(weights["embed"], MAT_PLAIN)
        w.final_norm = self._vec(weights["final_norm"])
        for l, L in enumerate(weights["layers"]):
            w.wqkv[l] = self._pack(L["wqkv"], MAT_QKV)
            w.bqkv[l] = self._vec(L["bqkv"])
            w.wo[l] = self._pack(L["wo"], MAT_PLAIN)
            w.wgu[l] = self._pack(L["wgu"], MAT_GATEUP)
            w.wd[l] = self._pack(L["wd"], MAT_PLAIN)
            w.ln1[l] = self._vec(L["ln1"])
            w.ln2[l] = self._vec(L["ln2"])
        torch.cuda.synchronize(self.device)
        self._staging = []  # standard-layout uploads are no longer needed
        cfg = VpConfig(FMT[self.fmt], self.n_layers, self.vocab, max_ctx, max_steps, device)
        ctx = ctypes.c_void_p()
        check(self.lib.vp_create(ctypes.byref(cfg), ctypes.byref(ctx)), "vp_create")
        self.ctx = ctx
        check(self.lib.vp_set_weights(self.ctx, ctypes.byref(w)), "vp_set_weights")
        self._weights_struct = w
        self._prompt = torch.empty(max_ctx, dtype=torch.int32, device=self.device)
        self._tree_host = torch.empty(TREE_INTS, dtype=torch.int32).pin_memory()
        self._step_out = VpState()
        self._step_tok = np.full(16, -1, dtype=np.int32)

    # ---- weights ----
    def _pack(self, m: dict, kind: int) -> int:
        fmt = FMT[self.fmt]
        if m["fmt"] != self.fmt:
            raise ValueError("mixed weight formats")
        if self.fmt == "f16":
            rows, cols = m["w"].shape
            codes, scales = _np_to_dev(m["w"], self.device), None
        else:
            rows = m["codes"].shape[0]
            cols = m["codes"].shape[1] * (2 if self.fmt == "q4" else 1)
            codes = _np_to_dev(m["codes"], self.device)
            scales = _np_to_dev(m["scales"], self.device)
        nbytes = self.lib.vp_packed_bytes(fmt, rows, cols)
        out = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        check(self.lib.vp_pack_matrix(fmt, kind, rows, cols, codes.data_ptr(),
                                      scales.data_ptr() if scales is not None else None,
                                      out.data_ptr(), self.stream.cuda_stream), "vp_pack_matrix")
        self._keep.append(out)
        self._staging.append((codes, scales))  # released once the pack kernels have run
        return out.data_ptr()

    def _vec(self, a: np.ndarray) -> int:
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(self.device)
        self._keep.append(t)
        return t.data_ptr()

    @classmethod
    def from_ill(cls, path: str, **kw) -> "VerifyEngine":
        """An engine on the weights of an .ill model file (Engine.init(modelPath:), Engine.swift:71):
        the file is read into the standard layouts (ill.read_ill) and packed for the tensor cores."""
        from .ill import read_ill

        return cls(read_ill(path), **kw)

    def close(self) -> None:
        if getattr(self, "ctx", None):
            self.lib.vp_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- operator surface ----
    @property
    def _s(self):
        return self.stream.cuda_stream

    def begin(self, cached: int, max_new: int, eos=STOP_IDS) -> None:
        check(self.lib.vp_begin(self.ctx, cached, max_new, eos[0], eos[1], self._s), "vp_begin")

    def prefill(self, tokens) -> None:
        toks = torch.as_tensor(np.asarray(tokens, dtype=np.int32))
        n = int(toks.numel())
        if n > self._prompt.numel():  # the device checks the context bound, not this buffer
            self._prompt = torch.empty(n, dtype=torch.int32, device=self.device)
        self._prompt[:n].copy_(toks, non_blocking=False)
        check(self.lib.vp_prefill(self.ctx, self._prompt.data_ptr(), n, self._s), "vp_prefill")

    def _tree_ptr(self, tree) -> int:
        buf = tree if isinstance(tree, np.ndarray) else tree_to_buffer(tree)
        self.stream.synchronize()  # the pinned staging buffer is reused
        self._tree_host.copy_(torch.from_numpy(np.asarray(buf, dtype=np.int32)))
        return self._tree_host.data_ptr()

    def verify(self, tree) -> None:
        check(self.lib.vp_verify(self.ctx, self._tree_ptr(tree), self._s), "vp_verify")

    def verify_chain(self, drafts) -> None:
        d = torch.as_tensor(np.asarray(drafts, dtype=np.int32)).to(self.device)
        self._keep_chain = d
        check(self.lib.vp_verify_chain(self.ctx, d.data_ptr() if d.numel() else None, int(d.numel()),
                                       self._s), "vp_verify_chain")

    def commit(self) -> None:
        check(self.lib.vp_commit(self.ctx, self._s), "vp_commit")

    def pass_(self, tree) -> None:
        check(self.lib.vp_pass(self.ctx, self._tree_ptr(tree), self._s), "vp_pass")

    def step(self, tree, state_in: Optional[VpState] = None) -> VpState:
        """One decode step from host memory (vp_step): optionally write `state_in`, copy the tree,
        run the pass (verify + commit), read the state and this pass's committed tokens back;
        synchronises. Returns the state as a VpState (fields as attributes, `.as_dict()`); the
        committed tokens are in `last_tokens()`. Both are refilled by the next call: copy them to
        keep them."""
        buf = tree if isinstance(tree, np.ndarray) else tree_to_buffer(tree)
        buf = np.ascontiguousarray(buf, dtype=np.int32)
        out = self._step_out
        rc = self.lib.vp_step(self.ctx, ctypes.addressof(state_in) if state_in is not None else None,
                              buf.ctypes.data, ctypes.byref(out), self._step_tok.ctypes.data, self._s)
        if rc not in (0, -5):
            check(rc, "vp_step")
        return out

    def last_tokens(self) -> list:
        """Tokens the last step() committed, in order."""
        t = self._step_tok
        return t[:int(np.argmax(t < 0)) if (t < 0).any() else t.size].tolist()

    def pass_device(self, tree_dev: torch.Tensor) -> None:
        """Graph pass with a device-resident tree buffer (no host round trip)."""
        check(self.lib.vp_pass(self.ctx, tree_dev.data_ptr(), self._s), "vp_pass")

    def pass_graph(self, tree_dev: torch.Tensor) -> Graph:
        """One fused pass reading the device tree buffer tree_dev, captured as a CUDA graph
        (vp_pass_graph): Graph.launch(stream) replays it."""
        h = ctypes.c_void_p()
        check(self.lib.vp_pass_graph(self.ctx, tree_dev.data_ptr(), ctypes.byref(h)), "vp_pass_graph")
        return Graph(self.lib, h)

    def step_graph(self, drafter, B: int, branch: int) -> Graph:
        """One step of the device-resident decode loop (the drafter's tree for the committed
        tokens, written into this context's tree buffer, then the pass) captured as a CUDA graph
        (vp_step_graph), for the drafter's current request."""
        h = ctypes.c_void_p()
        check(self.lib.vp_step_graph(self.ctx, drafter.h, int(B), int(branch), ctypes.byref(h)), "vp_step_graph")
        return Graph(self.lib, h)

    @staticmethod
    def pass_multi(engines, trees_dev, shares: int = 2) -> None:
        """One verify pass + commit of each engine's request in one launch, each request on
        1/shares of the SMs (vp_pass_batch; shares 2 is vp_pass_multi); trees_dev: one device
        int32[65] tree buffer per engine. A request's passes must all use one share."""
        if not engines or len(engines) != len(trees_dev):
            raise ValueError("one tree per engine")
        n = len(engines)
        ctxs = (ctypes.c_void_p * n)(*[e.ctx.value for e in engines])
        trees = (ctypes.c_void_p * n)(*[t.data_ptr() for t in trees_dev])
        e0 = engines[0]
        if shares == 2:
            check(e0.lib.vp_pass_multi(ctxs, trees, n, e0._s), "vp_pass_multi")
        else:
            check(e0.lib.vp_pass_batch(ctxs, trees, n, shares, e0._s), "vp_pass_batch")

    # ---- results ----
    def state(self) -> dict:
        st = VpState()
        rc = self.lib.vp_read_state(self.ctx, ctypes.byref(st), self._s)
        d = st.as_dict()
        if rc not in (0, -5):
            check(rc, "vp_read_state")
        return d

    def snapshot(self):
        """The device state as (host VpState, device int32[16] copy), e.g. right after a prefill."""
        st = VpState()
        rc = self.lib.vp_read_state(self.ctx, ctypes.byref(st), self._s)
        if rc not in (0, -5):
            check(rc, "vp_read_state")
        dev = torch.tensor([getattr(st, n) for n in _lib.STATE_FIELDS], dtype=torch.int32,
                           device=self.device)
        return st, dev

    def restore(self, snap, on_device: bool = True):
        """Write a snapshot back into the device state (stream-ordered): the next pass runs from
        that point over the same cached prefix."""
        st, dev = snap
        if on_device:
            check(self.lib.vp_write_state(self.ctx, dev.data_ptr(), 1, self._s), "vp_write_state")
        else:
            check(self.lib.vp_write_state(self.ctx, ctypes.addressof(st), 0, self._s), "vp_write_state")

    # ---- prefix KV cache on disk (Engine.savePrefix / loadPrefix, Engine.swift:788-838) ----
    PREFIX_MAGIC = 0x3156_4B4C_4C49  # "ILLKV1"

    def _prefix_key(self, model_path: Optional[str]) -> list:
        """The reference's file key: magic, model file size and mtime (s, ns), max context."""
        import os

        if model_path is None:  # synthetic weights: no model file
            return [self.PREFIX_MAGIC, 0, 0, 0, self.max_ctx]
        stt = os.stat(model_path)
        return [self.PREFIX_MAGIC, stt.st_size, int(stt.st_mtime), stt.st_mtime_ns % 1_000_000_000, self.max_ctx]

    def save_prefix(self, path: str, tokens, model_path: Optional[str] = None) -> None:
        """Save the K/V rows of the first len(tokens) cached positions (their tokens are `tokens`)
        in the reference's prefix-file layout."""
        toks = np.asarray(tokens, dtype=np.int32)
        n = int(toks.size)
        body = np.empty(int(self.lib.vp_prefix_bytes(self.ctx, n)), dtype=np.uint8)
        if body.size == 0:
            raise ValueError("bad prefix length")
        check(self.lib.vp_save_prefix(self.ctx, n, body.ctypes.data, self._s), "vp_save_prefix")
        head = np.array(self._prefix_key(model_path) + [n], dtype=np.uint64)
        with open(path, "wb") as f:
            f.write(head.tobytes())
            f.write(toks.tobytes())
            f.write(body.tobytes())

    def load_prefix(self, path: str, model_path: Optional[str] = None) -> Optional[list]:
        """Load a saved prefix made for this model and context size into the KV cache; returns its
        tokens (then begin(len(tokens), ...) skips prefilling them), or None if the file does not
        match."""
        import os

        if not os.path.exists(path):
            return None
        d = np.fromfile(path, dtype=np.uint8)
        if d.size <= 48:
            return None
        head = d[:48].view(np.uint64)
        if list(map(int, head[:5])) != self._prefix_key(model_path):
            return None
        n = int(head[5])
        nb = int(self.lib.vp_prefix_bytes(self.ctx, n)) if 0 < n < self.max_ctx else 0
        if nb == 0 or d.size != 48 + 4 * n + nb:
            return None
        toks = d[48:48 + 4 * n].view(np.int32).tolist()
        body = np.ascontiguousarray(d[48 + 4 * n:])
        check(self.lib.vp_load_prefix(self.ctx, n, body.ctypes.data, self._s), "vp_load_prefix")
        torch.cuda.synchronize(self.device)
        return toks

    def tokens(self, count: Optional[int] = None) -> list:
        st = self.state()
        count = st["step"] if count is None else count
        out = np.empty(count, np.int32)
        if count:
            check(self.lib.vp_read_tokens(self.ctx, out.ctypes.data, count, self._s), "vp_read_tokens")
        return out.tolist()

    def buffer(self, which: int, shape, dtype: str) -> torch.Tensor:
        ptr, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
        check(self.lib.vp_buffer(self.ctx, which, ctypes.byref(ptr), ctypes.byref(nbytes)), "vp_buffer")
        return torch.as_tensor(_DevArray(ptr.value, shape, dtype), device=self.device)

    def argmax_partials(self):
        """Per-CTA argmax partials of the last pass, (value fp32 [16][parts], id int32 [16][parts]):
        what the commit reduces."""
        ptr, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
        check(self.lib.vp_buffer(self.ctx, 4, ctypes.byref(ptr), ctypes.byref(nbytes)), "vp_buffer")
        parts = nbytes.value // (16 * 4)
        return self.buffer(4, (16, parts), "<f4"), self.buffer(5, (16, parts), "<i4")

    def kv(self):
        shape = (self.n_layers, 2, self.max_ctx, 64)
        return self.buffer(2, shape, "<f2"), self.buffer(3, shape, "<f2")

    def logits(self) -> torch.Tensor:
        """fp32 logits [16, vocab] of the rows of the last pass (parity helper)."""
        out = torch.empty((16, self.vocab), dtype=torch.float32, device=self.device)
        check(self.lib.vp_debug_logits(self.ctx, out.data_ptr(), self._s), "vp_debug_logits")
        return out

    # ---- generate (Engine.generate, Engine.swift:922-1038) ----
    def generate(self, prompt, max_new: int, tree_fn: Optional[Callable] = None, eos=STOP_IDS,
                 fused: bool = True, cached: int = 0) -> dict:
        """Prefill `prompt`, then verify passes until max_new tokens or a stop token. tree_fn(out)
        returns the next pass's tree given the tokens committed so far (None: 1-row passes, i.e.
        plain greedy decoding through the same kernels, the reference's noDraft run). fused=False
        runs each pass as verify + a separate commit launch instead of one pass launch. cached: the
        first `cached` prompt tokens are already in the KV cache (load_prefix) and not prefilled."""
        from .synth import root_tree

        self.begin(cached, max_new, eos)
        self.prefill(list(prompt)[cached:])
        st = self.state()
        out = self.tokens(st["step"])
        passes = 0
        while not st["done"]:
            tree = tree_fn(out) if tree_fn else root_tree()
            if fused:
                st = self.step(tree).as_dict()  # tree in, pass, state and tokens out: one call
                out = out + self.last_tokens()
            else:
                self.verify(tree)
                self.commit()
                st = self.state()
                out = self.tokens(st["step"])
            passes += 1
            if st["err"]:
                raise _lib.VpError(f"device error bits {st['err']}")
        assert len(out) == st["step"], (len(out), st["step"])
        return {"tokens": out, "passes": passes, "state": st}

    @staticmethod
    def prefill_batch(engines, prompts, shares: Optional[int] = None) -> None:
        """Prefill of several requests together (vp_prefill_batch), each on 1/shares of the SMs
        (shares = the number of requests unless given): launch c runs the 16-row chunk c of every
        prompt that has one. Each engine must have begun its request (begin)."""
        k = len(engines)
        shares = k if shares is None else shares
        if len(prompts) != k:
            raise ValueError("one prompt per engine")
        ptrs, ns = [], []
        for eng, p in zip(engines, prompts):
            toks = torch.as_tensor(np.asarray(p, dtype=np.int32))
            n = int(toks.numel())
            if n > eng._prompt.numel():
                eng._prompt = torch.empty(n, dtype=torch.int32, device=eng.device)
            eng._prompt[:n].copy_(toks, non_blocking=False)
            ptrs.append(eng._prompt.data_ptr())
            ns.append(n)
        ctxs = (ctypes.c_void_p * k)(*[eng.ctx.value for eng in engines])
        arr = (ctypes.c_void_p * k)(*ptrs)
        narr = (ctypes.c_int32 * k)(*ns)
        e0 = engines[0]
        check(e0.lib.vp_prefill_batch(ctxs, arr, narr, k, shares, e0._s), "vp_prefill_batch")

    @staticmethod
    def generate_drafted_batch(engines, prompts, max_new: int, drafters, pids=None, texts=None, eos=STOP_IDS,
                               shares: Optional[int] = None, depth: int = 1, adaptive: bool = True) -> list:
        """generate_drafted for up to four requests at once, one engine and one drafter each: every
        step drafts each live request's next tree (k_draft, one CTA, each on its own side stream, so
        the drafts run side by side) and then verifies all of them in one launch (vp_pass_batch,
        each request on 1/shares of the SMs, shares = the number of requests unless given); the
        prompts are prefilled together on the same shares (prefill_batch). Steps
        are enqueued `depth` ahead of the last one the host has seen finish; each request's shape
        follows its own counters (PassShape); a request the host has seen stop leaves the batch
        (the others keep their shares). A request's output is its greedy decoding on the same share
        (prefill_batch, then 1-row vp_pass_batch passes), token for token: its arithmetic depends on
        its share only, not on its partners. Returns one generate_drafted result per request."""
        k = len(engines)
        shares = k if shares is None else shares
        if not 1 <= k <= shares <= 4:
            raise ValueError("need 1 <= requests <= shares <= 4")
        if len(prompts) != k or len(drafters) != k or len({id(e) for e in engines}) != k:
            raise ValueError("one prompt and one drafter per engine, engines distinct")
        e0 = engines[0]
        if any(e.device != e0.device or d.device != e0.device for e, d in zip(engines, drafters)):
            raise ValueError("engines and drafters on one device")
        if depth < 0:
            raise ValueError("depth must be >= 0")
        pids = [None] * k if pids is None else pids
        texts = [""] * k if texts is None else texts
        main = e0.stream
        for e in engines:
            e.begin(0, max_new, eos)
        VerifyEngine.prefill_batch(engines, [list(p) for p in prompts], shares)
        for d, p, q, t in zip(drafters, prompts, pids, texts):
            d.begin(list(p) if q is None else list(q), t)  # overlaps the prefill
        tree_ptrs = [e.buffer(7, (TREE_INTS,), "<i4").data_ptr() for e in engines]
        st_ptrs = [e.lib.vp_device_state(e.ctx) for e in engines]
        tok_ptrs = [e.lib.vp_device_tokens(e.ctx) for e in engines]
        nf = len(_lib.STATE_FIELDS)
        st_devs = [torch.as_tensor(_DevArray(p, (nf,), "<i4"), device=e0.device) for p in st_ptrs]
        i_passes = _lib.STATE_FIELDS.index("passes")
        i_acc = _lib.STATE_FIELDS.index("accepted")
        i_done = _lib.STATE_FIELDS.index("done")
        slots = depth + 2
        host = torch.zeros((slots, k, nf), dtype=torch.int32).pin_memory()
        side = [torch.cuda.Stream(device=e0.device) for _ in range(k)]
        shape = [PassShape(adaptive=adaptive) for _ in range(k)]
        seen = [[0, 0, 0] for _ in range(k)]  # passes, accepted, done
        shapes = [[] for _ in range(k)]
        from collections import deque

        pending = deque()
        waits, encoded, seen_steps = 0, 1, 1
        with torch.cuda.stream(main):
            while True:
                while pending and pending[0][0].query():
                    _, slot, live = pending.popleft()
                    seen_steps += 1
                    for r in live:
                        row = host[slot, r].tolist()
                        seen[r] = [row[i_passes], row[i_acc], row[i_done]]
                live = [r for r in range(k) if not seen[r][2]]
                if not live:
                    break
                if encoded < max_new and encoded - seen_steps <= depth:
                    fork = torch.cuda.Event()
                    fork.record(main)
                    for r in live:
                        B, branch = shape[r].next(seen[r][0], seen[r][1])
                        shapes[r].append((B, branch))
                        side[r].wait_event(fork)
                        drafters[r].draft(tree_ptrs[r], tok_ptrs[r], state_ptr=st_ptrs[r], B=B, branch=branch,
                                          stream=side[r].cuda_stream)
                        join = torch.cuda.Event()
                        join.record(side[r])
                        main.wait_event(join)
                    n = len(live)
                    ctxs = (ctypes.c_void_p * n)(*[engines[r].ctx.value for r in live])
                    trees = (ctypes.c_void_p * n)(*[tree_ptrs[r] for r in live])
                    check(e0.lib.vp_pass_batch(ctxs, trees, n, shares, main.cuda_stream), "vp_pass_batch")
                    slot = encoded % slots
                    for r in live:
                        host[slot, r].copy_(st_devs[r], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(main)
                    pending.append((ev, slot, live))
                    encoded += 1
                    continue
                if not pending:
                    break
                pending[0][0].synchronize()
                waits += 1
        out = []
        for r, e in enumerate(engines):
            st = e.state()
            if st["err"]:
                raise _lib.VpError(f"request {r}: device error bits {st['err']}")
            if not st["done"]:
                raise _lib.VpError(f"request {r}: decode loop ended before the request's stop")
            out.append({"tokens": e.tokens(st["step"]), "passes": st["passes"] - 1, "state": st,
                        "shapes": shapes[r], "host_waits": waits})
        return out

    def generate_drafted(self, prompt, max_new: int, drafter, pids=None, text: str = "", eos=STOP_IDS,
                         cached: int = 0, depth: int = 1, shape: Optional[PassShape] = None,
                         graphs: bool = False) -> dict:
        """Engine.generate with the learned drafter (Engine.swift:922-1030), device-resident: after
        the prefill, every step is k_draft (the next tree from the committed tokens and the device
        state, written into a device tree buffer) followed by one pass, both on this engine's
        stream, so no token or tree goes through the host. As the reference does, the host keeps
        `depth` steps enqueued ahead of the last one it has seen finish (encode-ahead), reads each
        finished step's state from a pinned copy made on the stream (no synchronisation while the
        GPU has work queued), and picks every new step's shape from those counters (PassShape).
        Steps enqueued past the stop run as early exits: every kernel of a finished request
        returns at once. drafter: a DeviceDrafter on this engine's device; pids / text: the
        request context of Drafter.begin (the prompt's ids and its text), built on the host while
        the GPU prefills. graphs: each step is the replay of a CUDA graph of the two launches
        (step_graph, captured once per shape for this request) instead of two library calls. Returns the tokens (as generate), the passes, the shapes enqueued, the
        host waits and the final state (passes: the verify passes that committed, as generate
        counts them)."""
        if drafter.device != self.device:
            raise ValueError("the drafter's table must be on the engine's device")
        if depth < 0:
            raise ValueError("depth must be >= 0")
        shape = shape if shape is not None else PassShape()
        shape.reset()
        prompt = list(prompt)
        self.begin(cached, max_new, eos)
        self.prefill(prompt[cached:])
        drafter.begin(prompt if pids is None else list(pids), text)  # overlaps the prefill
        tree_ptr = self.buffer(7, (TREE_INTS,), "<i4").data_ptr()  # the pass reads it in place
        slots = depth + 2  # at most depth + 1 copies in flight
        host = getattr(self, "_loop_host", None)
        if host is None or host.shape[0] < slots:
            host = self._loop_host = torch.zeros((slots, len(_lib.STATE_FIELDS)), dtype=torch.int32).pin_memory()
        st_ptr = self.lib.vp_device_state(self.ctx)
        tok_ptr = self.lib.vp_device_tokens(self.ctx)
        st_dev = torch.as_tensor(_DevArray(st_ptr, (len(_lib.STATE_FIELDS),), "<i4"), device=self.device)
        i_passes = _lib.STATE_FIELDS.index("passes")
        i_acc = _lib.STATE_FIELDS.index("accepted")
        i_done = _lib.STATE_FIELDS.index("done")
        from collections import deque

        pending = deque()
        seen_passes = seen_acc = seen_done = 0
        shapes = []
        waits = 0
        encoded = 1  # the prefill (as Engine.generate counts it)
        step_graphs = {}
        with torch.cuda.stream(self.stream):
            while True:
                while pending and pending[0][0].query():
                    _, k = pending.popleft()
                    row = host[k].tolist()
                    seen_passes, seen_acc, seen_done = row[i_passes], row[i_acc], row[i_done]
                if seen_done:
                    break
                # the prefill yields one token and every pass at least one, so max_new - 1 passes
                # always reach the stop; `passes` counts the prefill's commit too, and the prefill
                # counts as seen from the start (Engine.generate's `done = 1 + passes`)
                if encoded < max_new and encoded - max(seen_passes, 1) <= depth:
                    B, branch = shape.next(seen_passes, seen_acc)
                    shapes.append((B, branch))
                    if graphs:
                        if (B, branch) not in step_graphs:
                            step_graphs[(B, branch)] = self.step_graph(drafter, B, branch)
                        step_graphs[(B, branch)].launch(self._s)
                    else:
                        drafter.draft(tree_ptr, tok_ptr, state_ptr=st_ptr, B=B, branch=branch, stream=self._s)
                        check(self.lib.vp_pass(self.ctx, tree_ptr, self._s), "vp_pass")
                    k = encoded % slots
                    host[k].copy_(st_dev, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.stream)
                    pending.append((ev, k))
                    encoded += 1
                    continue
                if not pending:
                    break
                pending[0][0].synchronize()
                waits += 1
        st = self.state()
        for g in step_graphs.values():
            g.close()
        if st["err"]:
            raise _lib.VpError(f"device error bits {st['err']}")
        if not st["done"]:
            raise _lib.VpError("decode loop ended before the request's stop")
        out = self.tokens(st["step"])
        return {"tokens": out, "passes": st["passes"] - 1, "state": st, "shapes": shapes, "host_waits": waits}
