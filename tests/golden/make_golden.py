#!/usr/bin/env python3
"""Generate the golden fixtures that pin the oracle to the reference's own code.

Run in a container that has the reference checkout (not needed at test time):
    python tests/golden/make_golden.py --reference /path/to/instantllm

It imports the reference's numpy fp32 model (tools/reference/qwen_ref.py, class Qwen2Ref, built with
__new__ and seeded weights injected as attributes, qwen_ref.py:88-110) and its tree-acceptance
function (tools/draft/ildraft.py:750-759), runs them on seeded inputs from instantllm_b200.synth,
and writes small JSON / npz files next to this script:

  qwen_small_{f32,q4}.npz  2-layer, 2048-vocab model: prompt, greedy ids, prefill logits (all rows),
                           8 decode-step logits (qwen_ref.Qwen2Ref.forward / greedy).
  qwen_full_f32.json       full 24-layer, 151936-vocab model, BASELINE config 1 (64-token prompt,
                           32 greedy tokens): ids and top-5 (id, logit) per step.
  accept_tree.json         random trees and target sequences with accept_tree's answer.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from instantllm_b200 import synth  # noqa: E402


def ref_model(qr, w: dict):
    """A reference Qwen2Ref with the seeded weights (fp32, dequantised exactly)."""
    from oracle.qwen_oracle import dequant  # same dequantisation the oracle uses, pinned below

    m = qr.Qwen2Ref.__new__(qr.Qwen2Ref)
    m.dtype = np.dtype(np.float32)
    m.embed = dequant(w["embed"])
    m.norm = w["final_norm"].astype(np.float32)
    m.layers = []
    for L in w["layers"]:
        wqkv, wgu = dequant(L["wqkv"]), dequant(L["wgu"])
        F = wgu.shape[0] // 2
        m.layers.append(SimpleNamespace(
            ln1=L["ln1"], ln2=L["ln2"], wq=wqkv[:896], bq=L["bqkv"][:896], wk=wqkv[896:1024],
            bk=L["bqkv"][896:1024], wv=wqkv[1024:], bv=L["bqkv"][1024:], wo=dequant(L["wo"]),
            wg=wgu[:F], wu=wgu[F:], wd=dequant(L["wd"])))
    m.inv_freq = 1.0 / qr.ROPE_THETA ** (np.arange(0, qr.HEAD_DIM, 2, dtype=np.float64) / qr.HEAD_DIM)
    return m


def small(qr, fmt: str):
    w = synth.make_weights(fmt, n_layers=2, vocab=2048, seed=11)
    m = ref_model(qr, w)
    prompt = (synth.make_prompt(12, seed=5) % 2048).astype(np.int64)
    cache = m.new_cache(64)
    pre = m.forward(list(prompt), cache, all_logits=True)
    r = m.greedy(list(prompt), max_new=8, stop_ids=(), keep_decode_logits=8)
    np.savez_compressed(HERE / f"qwen_small_{fmt}.npz", prompt=prompt, prefill_logits=pre.astype(np.float32),
                        output_ids=np.asarray(r["output_ids"], np.int64),
                        decode_logits=np.stack(r["decode_logits"]).astype(np.float32))


def full(qr):
    w = synth.make_weights("f32", n_layers=24, seed=0)
    m = ref_model(qr, w)
    prompt = synth.make_prompt(64, seed=1).astype(np.int64)
    r = m.greedy(list(prompt), max_new=32, stop_ids=(151645, 151643))
    rec = {"config": "BASELINE config 1: seeded N(0,0.02) fp32 weights, 64-token prompt, 32 greedy tokens",
           "weights": "instantllm_b200.synth.make_weights('f32', n_layers=24, seed=0)",
           "prompt": prompt.tolist(), "output_ids": r["output_ids"], "stop_token": r["stop_token"],
           "step_top5": r["step_top5"]}
    (HERE / "qwen_full_f32.json").write_text(json.dumps(rec))


def accept_cases(ild):
    rng = np.random.default_rng(2024)
    cases = []
    for _ in range(300):
        B = int(rng.integers(1, 16))
        parents, tokens = [], []
        for i in range(B):
            parents.append(int(rng.integers(-1, i)))
            tokens.append(int(rng.integers(0, 4)))  # small alphabet: many matches and duplicates
        y = [int(v) for v in rng.integers(0, 4, size=int(rng.integers(1, 12)))]
        p = int(rng.integers(0, len(y)))
        cases.append({"parents": parents, "tokens": tokens, "y": y, "p": p,
                      "a": ild.accept_tree(parents, tokens, y, p)})
    (HERE / "accept_tree.json").write_text(json.dumps(cases))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="instantllm checkout")
    ap.add_argument("--skip-full", action="store_true")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "tools" / "reference"))
    sys.path.insert(0, str(ref / "tools" / "draft"))
    sys.dont_write_bytecode = True
    import ildraft  # noqa: E402
    import qwen_ref as qr  # noqa: E402

    accept_cases(ildraft)
    small(qr, "f32")
    small(qr, "q4")
    if not args.skip_full:
        full(qr)
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()
