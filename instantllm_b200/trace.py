"""Stage trace of the verify pass (performance work).

The trace build of the library (`libvpass_trace.so`: the same kernels compiled with
-DVP_TRACE_DETAIL, `instantllm_b200.build.build(trace=True)`) stamps %globaltimer on every CTA at
each step of the stages of one layer (layer 5) and of the lm_head, and at every lm_head job of every
warp. This module runs one config-2 tree pass through it on cuda:0 (q4 weights, a 256-token cached
prefix, a seeded 16-row tree after the true continuation) and prints the timeline:

    python -m instantllm_b200.trace [--layers 24] [--passes 6] [--rows 16]

(--rows 1 traces a 1-row pass, plain decoding, instead of the 16-row tree.)

Layout of the stamps (trace[MK_TRACE_BASE + 256 * event + cta], csrc/vp_mega.cuh): event
8 * stage + step for the GEMM stages (stages QKV, O, gate/up, down, lm_head; steps entry, inputs in
shared memory, group sums, jobs done, pieces released, epilogue done), 40 / 41 / 42 attention unit
start / records done / combined, 48 + 2k / 49 + 2k arrival at / exit from the k-th grid barrier of
the layer, 56 layer start, and 288 + (warp * 5 + round) * 3 + s the lm_head job of each warp in each
round (s = 0 start, 1 its first piece in the ring, 2 folded into the warp's running argmax). The
stamps cost about 1.5 us per layer; the arithmetic is the product kernel's.
"""
from __future__ import annotations

import argparse

import numpy as np

TRACE_BASE = 2048
TRACE_LAYER = 5
TRACE_LEN = TRACE_BASE + (64 + 16 * 8 + 96 + 16 * 5 * 3) * 256
STAGES = ("QKV", "O", "gate/up", "down", "lm_head")
STEPS = ("entry", "inputs", "gsums", "jobs", "released", "epilogue")
LM_ROUNDS = 5


def stage_event(stage: int, step: int) -> int:
    return 8 * stage + step


def lm_job_event(warp: int, rnd: int, s: int) -> int:
    return 288 + (warp * LM_ROUNDS + rnd) * 3 + s


def _events(buf: np.ndarray, ev: int, G: int) -> np.ndarray:
    """Stamps of event ev over the first G CTAs in us, NaN where a CTA did not stamp."""
    v = buf[TRACE_BASE + 256 * ev: TRACE_BASE + 256 * ev + G].astype(np.float64)
    v[v <= 0] = np.nan
    return v / 1000.0


def timeline(buf: np.ndarray, G: int) -> dict:
    """The stage timeline of one traced pass from its stamp buffer (int64 ns, TRACE_LEN entries):
    per stage and step the median and max over the stamping CTAs in us after the layer start, and the
    lm_head's per-round wait (start -> first piece) and compute (first piece -> folded) over all
    warps, in us after the lm_head's earliest entry."""
    t0 = np.nanmin(_events(buf, 56, G))
    out = {"layer": {}, "lm_head": {}}
    for st, name in enumerate(STAGES[:4]):
        row = {}
        for k, step in enumerate(STEPS):
            v = _events(buf, stage_event(st, k), G) - t0
            if np.any(np.isfinite(v)):
                row[step] = (float(np.nanmedian(v)), float(np.nanmax(v)))
        out["layer"][name] = row
    att = {}
    for ev, step in ((40, "unit start"), (41, "records"), (42, "combined")):
        v = _events(buf, ev, G) - t0
        if np.any(np.isfinite(v)):
            att[step] = (float(np.nanmedian(v)), float(np.nanmax(v)))
    out["layer"]["attention"] = att
    bar = {}
    for k in range(4):
        a, e = _events(buf, 48 + 2 * k, G) - t0, _events(buf, 49 + 2 * k, G) - t0
        if np.any(np.isfinite(a)):
            bar[k] = (float(np.nanmax(a)), float(np.nanmedian(e)))
    out["layer"]["barriers"] = bar
    l0 = np.nanmin(_events(buf, stage_event(4, 0), G))
    lm = {}
    for k, step in enumerate(STEPS[:5]):
        v = _events(buf, stage_event(4, k), G) - l0
        if np.any(np.isfinite(v)):
            lm[step] = (float(np.nanmedian(v)), float(np.nanmax(v)))
    rounds = []
    for r in range(LM_ROUNDS):
        s = np.stack([_events(buf, lm_job_event(w, r, 0), G) for w in range(16)]) - l0
        rd = np.stack([_events(buf, lm_job_event(w, r, 1), G) for w in range(16)]) - l0
        dn = np.stack([_events(buf, lm_job_event(w, r, 2), G) for w in range(16)]) - l0
        if not np.any(np.isfinite(s)):
            continue
        rounds.append({"round": r, "jobs": int(np.isfinite(s).sum()), "start_med": float(np.nanmedian(s)),
                       "wait_mean": float(np.nanmean(rd - s)), "compute_mean": float(np.nanmean(dn - rd)),
                       "done_med": float(np.nanmedian(dn)), "done_max": float(np.nanmax(dn))})
    lm["rounds"] = rounds
    out["lm_head"] = lm
    return out


def run(layers: int = 24, passes: int = 6, seed: int = 0, rows: int = 16) -> dict:
    """Build the trace library if needed, run `passes` identical config-2 tree passes (rows = 16) or
    1-row passes (rows = 1) through it and return the timeline of the last one, with the CUDA-event
    time of every pass."""
    from pathlib import Path

    import torch

    from . import _lib, build, synth

    if _lib._lib is not None and Path(_lib.LIB_PATH) != build.TRACE_OUT:
        raise RuntimeError("the product library is loaded in this process: trace in a fresh one")
    _lib.LIB_PATH = build.build(trace=True)
    from .engine import VerifyEngine

    if layers <= TRACE_LAYER:
        raise ValueError(f"the traced layer is {TRACE_LAYER}: run at least {TRACE_LAYER + 1} layers")
    w = synth.make_weights("q4", n_layers=layers, seed=seed)
    eng = VerifyEngine(w, max_ctx=4096, max_steps=4096, device=0)
    try:
        dev = eng.device
        prompt = synth.make_prompt(256, seed=1000)
        eng.begin(0, 24, (-1, -1))
        eng.prefill(prompt)
        snap = eng.snapshot()
        root = torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=dev)
        for _ in range(23):
            eng.pass_device(root)
        y = eng.tokens(24)
        if rows not in (1, 16):
            raise ValueError("rows must be 1 or 16")
        tree = synth.seeded_tree(np.random.default_rng(seed + 7), y[1:10], n=16) if rows == 16 else synth.root_tree()
        tb = torch.tensor(synth.tree_to_buffer(tree), device=dev)
        buf = eng.buffer(6, (TRACE_LEN,), "<i8")
        G = eng.argmax_partials()[0].shape[1]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        times = []
        for _ in range(passes):
            eng.restore(snap)
            buf.zero_()
            ev[0].record(eng.stream)
            eng.pass_device(tb)
            ev[1].record(eng.stream)
            torch.cuda.synchronize()
            times.append(ev[0].elapsed_time(ev[1]) * 1000.0)
        out = timeline(buf.cpu().numpy().astype(np.int64), G)
        out["pass_us"] = times
        out["ctas"] = G
        return out
    finally:
        eng.close()


def report(t: dict) -> str:
    lines = [f"pass us (trace build, CUDA events): {' '.join(f'{x:.1f}' for x in t['pass_us'])}",
             f"layer {TRACE_LAYER}, us after the layer start (median over the stage's CTAs / max):"]
    for name in ("QKV", "attention", "O", "gate/up", "down"):
        row = t["layer"][name]
        lines.append(f"  {name:9s} " + "  ".join(f"{k} {m:.2f}/{x:.2f}" for k, (m, x) in row.items()))
    for k, (a, e) in t["layer"]["barriers"].items():
        lines.append(f"  grid barrier {k}: last arrival {a:.2f}, median exit {e:.2f}")
    lm = t["lm_head"]
    lines.append("lm_head, us after its first CTA's entry (median / max over CTAs): "
                 + "  ".join(f"{k} {v[0]:.2f}/{v[1]:.2f}" for k, v in lm.items() if k != "rounds"))
    for r in lm["rounds"]:
        lines.append(f"  round {r['round']}: {r['jobs']} jobs, start {r['start_med']:.2f}, wait for the first "
                     f"piece {r['wait_mean']:.2f}, 14 tiles + fold {r['compute_mean']:.2f}, done "
                     f"{r['done_med']:.2f} (max {r['done_max']:.2f})")
    return "\n".join(lines)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--passes", type=int, default=6)
    ap.add_argument("--rows", type=int, default=16, choices=(1, 16))
    a = ap.parse_args()
    print(report(run(a.layers, a.passes, rows=a.rows)))


if __name__ == "__main__":
    main()
