#!/usr/bin/env python3
"""Benchmark of the q4 16-row tree-verify pass on 1..8 B200s.

One step = one 16-row tree verify pass + greedy accept/commit of one request over a 256-token
cached prefix: the prompt is prefilled before timing and every step starts from that state (the
64-byte device state is written back before each pass, part of the timed step). Trees follow BASELINE config 2:
root + 15 drafts, parents uniform among earlier nodes of depth < 8, drafts equal to the parent's
true argmax with p = 0.6. The "true argmax" comes from a prior sequential run of the same request
through the same kernels (1-row passes), and the committed tokens of the timed tree passes are
checked against it (tree == sequential) for every step after the timed loop.

value  = accepted (committed) tokens per second over all ranks, inputs resident in HBM.
e2e    = the same through the C ABI from host memory: one vp_step per step (the post-prefill state
         and the tree in, the pass, the committed state back to the host).
N > 1  = one independent request per rank (request-level sharding, weak scaling, no collective on
         the data path; torch.distributed over gloo is used only for the barrier around the timed
         region and the max-time reduce; no NCCL).

--impl reference times the reference's CPU path (the numpy fp32 restatement in oracle/, a port of
tools/reference/qwen_ref.py: the Swift/Metal engine cannot run here) on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "q4 16-row tree-verify pass µs & accepted tok/s; HBM GB/s vs B200 peak"
PREFIX = 256
ROWS = 16
L2_NOTE = "weights (278 MB/pass) exceed the 126 MB L2: no flush needed"
WORKLOAD2 = "BASELINE config 2: q4 16-row tree verify + greedy commit, 256-token cached prefix, one request per GPU"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workload", choices=["config2", "batch2", "batch3", "batch4", "config3", "config4", "config5",
                                           "sketch_head", "decode_loop"],
                    default="config2",
                    help="batch2 / batch3 / batch4: two, three or four config-2 requests per launch "
                         "(vp_pass_batch, each on 1/k of the SMs), aggregate tok/s (1 GPU); "
                         "config3 / config4: the q8 8-row chain and f16 16-row tree workloads (1 GPU, "
                         "their own line); config5: BASELINE config 5, independent requests sharded "
                         "over the ranks; sketch_head: the optional two-stage lm_head against the full "
                         "one (1 GPU); decode_loop: the device-resident loop with the learned drafter "
                         "(1 GPU)")
    ap.add_argument("--requests", type=int, default=256, help="config5: number of requests")
    ap.add_argument("--c5-requests", type=int, default=64,
                    help="requests of the config-5 sub-object of the default line (0: skip it)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


PROFILE = ROOT / "profiles" / "k_pass_q4_config2.md"


def ncu_traffic():
    """DRAM bytes (read + write) of one k_pass launch of this workload from the committed ncu
    summary (line 'dram_bytes_per_launch: N'), or None."""
    import re

    if PROFILE.exists():
        m = re.search(r"dram_bytes_per_launch:\s*(\d+)", PROFILE.read_text())
        if m:
            return int(m.group(1))
    return None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled every 5 ms through NVML in a background
    thread; stop() keeps the samples taken inside the timed region (mark_start .. stop)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, gpu: int):
        import threading

        self.gpu = gpu
        self.samples = []  # (t, sm_mhz, reasons bitmask)
        self.t0 = None
        self.err = None
        self.max_mhz = None
        self.run = threading.Event()
        self.thread = threading.Thread(target=self._loop, daemon=True)

    def _loop(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            while self.run.is_set():
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                except AttributeError:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.samples.append((time.perf_counter(), float(sm), int(rs)))
                time.sleep(0.005)
            nv.nvmlShutdown()
        except Exception as e:  # no NVML: report it instead of clocks
            self.err = f"{type(e).__name__}: {e}"

    def start(self):
        self.run.set()
        self.thread.start()
        for _ in range(400):  # sampling is running before the timed region starts
            if self.samples or self.err:
                break
            time.sleep(0.005)

    def mark_start(self):
        self.t0 = time.perf_counter()

    def stop(self) -> dict:
        t1 = time.perf_counter()
        self.run.clear()
        self.thread.join(timeout=5)
        if self.err:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [f"NVML unavailable ({self.err})"],
                    "samples": 0}
        inside = [x for x in self.samples if self.t0 is None or self.t0 <= x[0] <= t1]
        if not inside and self.samples:  # region shorter than one sampling period
            inside = [min(self.samples, key=lambda x: abs(x[0] - t1))]
        mask = 0
        for x in inside:
            mask |= x[2]
        return {"sm_mhz": float(np.median([x[1] for x in inside])) if inside else None,
                "sm_max_mhz": self.max_mhz,
                "reasons": sorted(k for k, v in self.REASONS.items() if mask & v),
                "samples": len(inside)}


# ---------------------------------------------------------------------------------------------
# workload


def plan_trees(y_full, start: int, n_steps: int, seed: int):
    """Trees for n_steps passes starting after y_full[:start] is committed. Returns (tree buffers,
    committed counts, expected token stream)."""
    from instantllm_b200 import synth
    from oracle import accept as A

    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 4242])))
    pos, bufs, counts = start, [], []
    for _ in range(n_steps):
        y = y_full[pos:pos + 9]
        if len(y) < 9:
            raise RuntimeError("sequential run too short for the tree plan")
        tree = synth.seeded_tree(rng, y, n=ROWS)
        parents, tokens = A.to_python_numbering(tree)
        a = A.accept_tree(parents, tokens, list(y), 0)
        bufs.append(synth.tree_to_buffer(tree))
        counts.append(a + 1)
        pos += a + 1
    return np.stack(bufs), counts, pos


def run_ours(args, rank, world, local):
    import torch

    from instantllm_b200 import synth
    from instantllm_b200.engine import VerifyEngine

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # the engine runs on a stream of its own, so that its timed steps can be captured as a graph
    torch.cuda.set_stream(torch.cuda.Stream(device=dev))
    t_setup = time.time()
    w = synth.make_weights("q4", n_layers=args.layers, seed=args.seed)
    n_steps = args.warmup + args.steps
    seq_len = 24
    eng = VerifyEngine(w, max_ctx=4096, max_steps=4096, device=local)
    prompt = synth.make_prompt(PREFIX, seed=1000 + rank)
    no_eos = (-1, -1)

    # 1) sequential reference run (1-row passes through the same kernels), untimed
    eng.begin(0, seq_len, no_eos)
    eng.prefill(prompt)
    tree1 = torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=dev)
    for _ in range(seq_len - 1):
        eng.pass_device(tree1)
    y_full = eng.tokens(seq_len)

    # 2) one seeded tree per step, every step from the same state: the 256-token prompt cached and
    #    its first token committed (config 2: one 16-row tree pass over a 256-token prefix)
    trees, counts = [], []
    for i in range(n_steps):
        t, c, _ = plan_trees(y_full, 1, 1, (args.seed + rank) * 100003 + i)
        trees.append(t[0])
        counts.append(c[0])
    trees = np.stack(trees)
    trees_dev = torch.tensor(trees, device=dev)
    n_tok_timed = int(sum(counts[args.warmup:]))

    eng.begin(0, seq_len, no_eos)
    eng.prefill(prompt)
    snap = eng.snapshot()
    for i in range(args.warmup):
        eng.restore(snap)
        eng.pass_device(trees_dev[i])
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    s = eng.stream

    def timed_steps(evs):
        # an event between consecutive steps: per-step device times (p50 / p90) and their sum
        evs[0].record(s)
        for k, i in enumerate(range(args.warmup, n_steps)):
            eng.restore(snap)  # 64-byte device-to-device state write: part of the step
            eng.pass_device(trees_dev[i])
            evs[k + 1].record(s)

    # The K timed steps are captured once as a CUDA graph (the state writes, the passes and the
    # events as its nodes) and replayed once untimed and once timed; a graph whose capture fails
    # falls back to stream launches of the same steps.
    timed_as = "one CUDA graph of the timed steps (state write + pass each)"
    try:
        evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(args.steps + 1)]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            timed_steps(evs)
        graph.replay()
        torch.cuda.synchronize()
        run_timed = graph.replay
    except Exception as exc:  # capture unsupported here: time the same steps as stream launches
        torch.cuda.synchronize()
        timed_as = f"stream launches (graph capture failed: {type(exc).__name__})"
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        run_timed = lambda: timed_steps(evs)  # noqa: E731
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.start()
    clocks.mark_start()
    run_timed()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = evs[0].elapsed_time(evs[-1])
    step_ms = [evs[k].elapsed_time(evs[k + 1]) for k in range(args.steps)]

    # tree == sequential, every step: the committed tokens of each pass are the sequential run's
    ok = True
    for i in range(n_steps):
        eng.restore(snap)
        eng.pass_device(trees_dev[i])
        st = eng.state()
        ok = ok and st["step"] == 1 + counts[i] and eng.tokens(st["step"]) == y_full[:st["step"]]

    # 3) end to end through the C ABI, one vp_step per step: the post-prefill state and the tree
    # (host buffers, VP_TREE_INTS int32 as the drafter hands it over) in, the pass, the state out
    host_trees = [np.ascontiguousarray(t, dtype=np.int32) for t in trees]
    snap_host = snap[0]
    for i in range(args.warmup):
        eng.step(host_trees[i], snap_host)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_tok, e2e_ok = 0, True
    for i in range(args.warmup, n_steps):
        # state + tree -> device, pass, state + the pass's committed tokens -> host
        stt = eng.step(host_trees[i], snap_host)
        got = eng.last_tokens()
        e2e_tok += len(got)
        e2e_ok = e2e_ok and got == y_full[1:1 + len(got)] and stt.step == 1 + len(got)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    return dict(ms=ms, step_ms=step_ms, tok=n_tok_timed, ok=ok and e2e_ok, clocks=clk, e2e_s=e2e_s, e2e_tok=e2e_tok,
                timed_as=timed_as,
                setup_s=time.time() - t_setup, eng=eng, w=w, prompt=prompt, y=y_full, trees=trees,
                counts=counts)


GEN = 64  # config 5: tokens generated per request


C5_MODES = (1, 2, 4)  # requests per launch measured in config 5 (each request on 1/k of the SMs)
C5_HEADLINE = 4       # the serving mode of the config-5 headline value


def run_config5(args, rank, world, local, w=None, n_requests=None):
    """BASELINE config 5 on this rank: its share of the requests (prefixes uniform in 128-2048,
    shard.assign), each prefilled, then decoded with 16-row tree passes to 64 tokens in three serving
    modes over the same requests: one request per launch (vp_pass on all SMs), two and four per
    launch (vp_pass_batch over the groups of shard.groups, each request on 1/k of the SMs to its end:
    once a request of a group has its tokens, the others go on without it). In each mode the
    requests are first decoded with 1-row passes of that mode (untimed: the true continuation that
    the seeded trees draft from; a share of the SMs sums some projections in another order than the
    whole GPU, so each mode has its own truth), and the committed tokens are checked against it
    (tree == sequential). Only the tree passes are timed (CUDA events around each group's passes,
    all enqueued at once from device-resident trees)."""
    import torch

    from instantllm_b200 import shard, synth
    from instantllm_b200.engine import VerifyEngine

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    prefixes = shard.config5_requests(n=n_requests or args.requests)
    mine = shard.assign(prefixes, world)[rank]
    if w is None:
        w = synth.make_weights("q4", n_layers=args.layers, seed=args.seed)
    kmax = max(C5_MODES)
    engs = [VerifyEngine(w, max_ctx=2048 + GEN + 16 + 32, max_steps=GEN + 16, device=local) for _ in range(kmax)]
    no_eos = (-1, -1)
    tree1 = torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=dev)
    s = engs[0].stream  # every engine runs on the device's current stream

    def plan(i, y):
        # trees planned from the true continuation; the device follows the planned acceptances
        trees, counts, pos = plan_trees(y, 1, 1, args.seed * 7 + i)
        bufs, cnts = [trees[0]], [counts[0]]
        while 1 + sum(cnts) < GEN:
            t, c, _ = plan_trees(y, 1 + sum(cnts), 1, args.seed * 7 + i * 1009 + len(bufs))
            bufs.append(t[0])
            cnts.append(c[0])
        return dict(y=y, tb=torch.tensor(np.stack(bufs), device=dev), cnts=cnts)

    def timed(fn):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        fn()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    res = {k: dict(ms=0.0, tok=0, passes=0, launches=0, nbytes=0.0, ok=True, differ=0) for k in C5_MODES}
    wbytes = synth.weight_bytes("q4", args.layers)

    def run_mode(sub, k):
        """Requests sub = [(engine, request)] decoded together with k shares (k = 1: alone on the
        whole GPU)."""
        r = res[k]
        for e, rq in sub:
            e.restore(rq["snap"])  # back to the post-prefill state over the same cached prefix
        es = [e for e, _ in sub]
        for _ in range(GEN + 8):
            if k == 1:
                es[0].pass_device(tree1)
            else:
                VerifyEngine.pass_multi(es, [tree1] * len(es), shares=k)
        plans = []
        for e, rq in sub:
            y = e.tokens(GEN + 9)
            if k == 1:
                rq["y1"], rq["plan1"] = y, plan(rq["i"], y)
            r["differ"] += int(y != rq["y1"])
            plans.append(rq["plan1"] if y == rq["y1"] else plan(rq["i"], y))
            e.restore(rq["snap"])
        L = max(len(p["tb"]) for p in plans)

        def go():
            for j in range(L):
                act = [q for q in range(len(sub)) if j < len(plans[q]["tb"])]
                if k == 1:
                    es[0].pass_device(plans[0]["tb"][j])
                else:
                    VerifyEngine.pass_multi([es[q] for q in act], [plans[q]["tb"][j] for q in act], shares=k)

        r["ms"] += timed(go)
        r["launches"] += L
        for (e, rq), p in zip(sub, plans):
            st = e.state()
            r["ok"] = r["ok"] and e.tokens(st["step"]) == p["y"][:st["step"]] and st["step"] >= GEN
            r["tok"] += st["step"] - 1  # the first token comes from the prefill
            n = len(p["cnts"])
            r["passes"] += n
            pre = prefixes[rq["i"]]
            r["nbytes"] += n * wbytes + 12288 * sum(pre + 1 + sum(p["cnts"][:j]) + ROWS for j in range(n)) * args.layers / 24

    for grp in shard.groups(mine, prefixes, kmax):
        reqs = []
        for e, i in zip(engs, grp):
            e.begin(0, GEN + 9, no_eos)
            e.prefill(synth.make_prompt(prefixes[i], seed=5000 + i))
            reqs.append(dict(i=i, snap=e.snapshot()))
        sub = list(zip(engs, reqs))
        for k in sorted(C5_MODES):
            for j in range(0, len(sub), k):
                if k == 1:
                    run_mode(sub[j:j + 1], 1)
                else:
                    run_mode(sub[j:j + k], k)
    for e in engs:
        e.close()
    return dict(modes=res, n=len(mine))


def config5_table(args, r, world):
    """Per-rank config-5 figures gathered on every rank: per mode of C5_MODES [device ms, tokens,
    request passes, launches, ok, GB/s, requests whose truth differs from the whole-GPU one]."""
    import torch

    vals = []
    for k in C5_MODES:
        m = r["modes"][k]
        gbs = m["nbytes"] / (max(m["ms"], 1e-9) * 1e-3) / 1e9
        vals += [m["ms"], float(m["tok"]), float(m["passes"]), float(m["launches"]), 1.0 if m["ok"] else 0.0, gbs,
                 float(m["differ"])]
    if world > 1:
        rows = [torch.zeros(len(vals), dtype=torch.float64) for _ in range(world)]
        torch.distributed.all_gather(rows, torch.tensor(vals, dtype=torch.float64))
        return [x.tolist() for x in rows]
    return [vals]


def config5_summary(table, n_requests) -> dict:
    """The headline value is C5_HEADLINE requests per launch; every mode of C5_MODES, on the same
    requests and trees, is reported under "modes"."""
    F = 7
    modes = {}
    for q, k in enumerate(C5_MODES):
        col = [t[q * F:(q + 1) * F] for t in table]
        tok = sum(c[1] for c in col)
        ms = max(c[0] for c in col)
        modes[str(k)] = {"value": tok / (ms * 1e-3), "unit": "tok/s", "tokens": int(tok),
                         "request_passes": int(sum(c[2] for c in col)), "launches": int(sum(c[3] for c in col)),
                         "ms_per_rank": [round(c[0], 3) for c in col],
                         "per_gpu_hbm_gbs": [round(c[5], 1) for c in col],
                         "tree_equals_sequential": all(c[4] > 0 for c in col),
                         "truth_differs_from_whole_gpu": int(sum(c[6] for c in col))}
    h = modes[str(C5_HEADLINE)]
    return {"value": h["value"], "unit": "tok/s", "requests": n_requests, "requests_per_launch": C5_HEADLINE,
            "tokens": h["tokens"], "ms_per_rank": h["ms_per_rank"], "per_gpu_hbm_gbs": h["per_gpu_hbm_gbs"],
            "tree_equals_sequential": all(m["tree_equals_sequential"] for m in modes.values()),
            "modes": modes}


def main_config5(args, rank, world):
    r = run_config5(args, rank, world, int(os.environ.get("LOCAL_RANK", str(rank))))
    table = config5_table(args, r, world)
    if rank == 0:
        line = {
            "metric": "config 5: aggregate accepted tok/s of independent q4 requests (16-row tree passes)",
            "n_gpus": world, "higher_is_better": True, "scaling": "strong",
            **config5_summary(table, args.requests),
            "config": {"workload": "BASELINE config 5: requests with prefixes uniform in [128, 2048], "
                                   "64 tokens each, seeded 16-row trees as in config 2, "
                                   "longest-processing-time-first sharding (no collective), "
                                   f"{C5_HEADLINE} requests per launch (vp_pass_batch); one, two and four "
                                   "per launch under modes",
                       "layers": args.layers, "timed": "tree passes only (device time, max over ranks)"},
            "data": "synthetic (seeded random-init q4 weights, uniform prompt ids, seeded trees)",
        }
        print(json.dumps(line), flush=True)


def cpu_baseline(w, prompt, y_full, trees, seconds: float) -> dict:
    """The oracle (numpy fp32 port of the reference CPU path) on a bounded sample of the same
    workload: tree passes over the same trees after the same 256-token prefix."""
    from oracle import accept as A
    from oracle import qwen_oracle as Q

    threads = host_threads()
    m = Q.model_from_weights(w)
    cache = Q.KVCache(len(m.layers), 4096)
    logits = Q.forward_causal(m, cache, list(prompt), 0)
    first = int(np.argmax(logits))
    tok, passes = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds and passes < len(trees):
        # every pass from the same state, as in the GPU arm: prefix cached, first token committed
        tb = trees[passes]
        n = int(tb[0])
        tree = {"n": n, "depth": list(tb[1:17]), "parent": list(tb[17:33]), "tok": list(tb[33:49])}
        lg = Q.tree_pass(m, cache, PREFIX, first, tree)
        g = lg.argmax(axis=1)
        res = A.commit(tree, g, PREFIX, 1, 1 << 30, eos=())
        for src, dst in res["moves"]:
            for li in range(len(m.layers)):
                cache.k[li][:, dst] = cache.k[li][:, src]
                cache.v[li][:, dst] = cache.v[li][:, src]
        tok += len(res["tokens"])
        passes += 1
    dt = time.perf_counter() - t0
    return {"value": tok / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{passes} q4 16-row tree passes (fp32 numpy, dequantised weights) after a "
                      f"{PREFIX}-token prefix, {dt:.1f} s", "pass_ms": 1000 * dt / max(passes, 1)}


def host_threads() -> int:
    """All host threads for numpy's BLAS, set explicitly: torchrun starts ranks with
    OMP_NUM_THREADS=1, which would leave the reference arm single-threaded at N > 1."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(limits=n)
        got = [d.get("num_threads") for d in threadpool_info() if d.get("user_api") == "blas"]
        return int(got[0]) if got else n
    except ImportError:
        return n


def run_reference(args):
    """--impl reference: the reference's CPU path (numpy fp32 port of tools/reference/qwen_ref.py;
    the Swift/Metal engine cannot run here) on the workload of the GPU arm: the same N requests that
    the N ranks serve (prompt seed 1000 + rank), each prefilled once, then one 16-row tree pass +
    commit per step from the post-prefill state, steps taking the requests in turn. Value = committed
    tokens / CPU time, so it does not depend on N."""
    from instantllm_b200 import synth
    from oracle import accept as A
    from oracle import qwen_oracle as Q

    threads = host_threads()
    world = max(1, args.gpus)
    w = synth.make_weights("q4", n_layers=args.layers, seed=args.seed)
    m = Q.model_from_weights(w)
    n_steps = args.warmup + args.steps
    reqs = []
    for rk in range(world):
        prompt = synth.make_prompt(PREFIX, seed=1000 + rk)
        cache = Q.KVCache(len(m.layers), 4096)
        logits = Q.forward_causal(m, cache, list(prompt), 0)
        # true continuation for the tree plans: the CPU model's own sequential greedy run
        y, pos = [int(np.argmax(logits))], PREFIX
        seq_cache = cache.copy()
        while len(y) < 10:
            lg = Q.forward_causal(m, seq_cache, [y[-1]], pos)
            y.append(int(np.argmax(lg)))
            pos += 1
        reqs.append((cache, y))
    times, toks = [], []
    for i in range(n_steps):
        rk = i % world
        cache, y = reqs[rk]
        # trees seeded as in the GPU arm's rank rk
        rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([(args.seed + rk) * 100003 + i, 4242])))
        tree = synth.seeded_tree(rng, y[1:10], n=ROWS)
        t0 = time.perf_counter()
        lg = Q.tree_pass(m, cache, PREFIX, y[0], tree)
        res = A.commit(tree, lg.argmax(axis=1), PREFIX, 1, 1 << 30, eos=())
        for src, dst in res["moves"]:
            for li in range(len(m.layers)):
                cache.k[li][:, dst] = cache.k[li][:, src]
                cache.v[li][:, dst] = cache.v[li][:, src]
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
            toks.append(len(res["tokens"]))
    total = sum(times)
    v = sum(toks) / total
    sample = (f"{len(times)} q4 16-row tree passes + commits over the {world} request(s) of the GPU arm, "
              f"numpy fp32 port of tools/reference/qwen_ref.py with {threads} BLAS threads "
              "(the Swift/Metal engine needs an Apple GPU)")
    line = {
        "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * total / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD2, "rows": ROWS, "prefix": PREFIX, "layers": args.layers,
                   "requests": world},
        "impl": "reference",
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_batch(args, k: int):
    """k config-2 requests per launch (vp_pass_batch with k shares: each request on 1/k of the SMs):
    each request prefilled with its own 256-token prompt, decoded with 1-row passes k per launch (the
    truth), then every step = all k requests' seeded 16-row tree passes + commits from their
    post-prefill states in one launch. Also times one request alone on its share (n = 1) and the
    plain whole-GPU pass. One JSON line of its own, 1 GPU."""
    import torch

    from instantllm_b200 import synth
    from instantllm_b200.engine import VerifyEngine

    w = synth.make_weights("q4", n_layers=args.layers, seed=args.seed)
    engs, snaps = [], []
    for r in range(k):
        eng = VerifyEngine(w, max_ctx=4096, max_steps=4096, device=0)
        eng.begin(0, 24, (-1, -1))
        eng.prefill(synth.make_prompt(PREFIX, seed=1000 + r))
        engs.append(eng)
        snaps.append(eng.snapshot())
    dev, s = engs[0].device, engs[0].stream
    root = torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=dev)
    for _ in range(23):
        VerifyEngine.pass_multi(engs, [root] * k, shares=k)
    ys = [e.tokens(24) for e in engs]
    n_steps = args.warmup + args.steps
    plans = [[plan_trees(ys[r], 1, 1, (args.seed + r) * 100003 + i) for i in range(n_steps)] for r in range(k)]
    trees = [torch.tensor(np.stack([p[0][0] for p in plans[r]]), device=dev) for r in range(k)]
    counts = [[p[1][0] for p in plans[r]] for r in range(k)]

    def timed(fn):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(args.warmup, n_steps):
            fn(i)
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    def all_k(i):
        for e, sn in zip(engs, snaps):
            e.restore(sn)
        VerifyEngine.pass_multi(engs, [trees[r][i] for r in range(k)], shares=k)

    def one(i):
        engs[0].restore(snaps[0])
        VerifyEngine.pass_multi(engs[:1], [trees[0][i]], shares=k)

    def whole(i):
        engs[0].restore(snaps[0])
        engs[0].pass_device(trees[0][i])

    clocks = ClockSampler(0)
    clocks.start()
    clocks.mark_start()
    msk = timed(all_k)
    clk = clocks.stop()
    ms1 = timed(one)
    msw = timed(whole)
    ok = True
    for i in range(n_steps):  # every step's committed tokens against the truth, all requests
        all_k(i)
        for r in range(k):
            st = engs[r].state()
            ok = ok and st["step"] == 1 + counts[r][i] and engs[r].tokens(st["step"]) == ys[r][:st["step"]]
    tokk = sum(sum(counts[r][args.warmup:]) for r in range(k))
    hbm_peak, peak_kind = peaks()
    wbytes = synth.weight_bytes("q4", args.layers)
    kv = 12288 * (PREFIX + ROWS) * args.layers / 24 + 12288 * ROWS * args.layers / 24
    launch_ms = msk / args.steps
    achieved = k * (wbytes + kv) / (launch_ms * 1e-3) / 1e9
    words = {2: "two", 3: "three", 4: "four"}
    line = {
        "metric": f"batched verify: {words.get(k, k)} requests per launch, aggregate accepted tok/s (q4 16-row trees)",
        "value": tokk / (msk * 1e-3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "requests_per_launch": k,
        "launch_us": 1000 * launch_ms, "one_request_share_us": 1000 * ms1 / args.steps,
        "one_request_whole_us": 1000 * msw / args.steps,
        "single_request_tok_s": sum(counts[0][args.warmup:]) / (msw * 1e-3),
        "tree_equals_sequential": bool(ok),
        "hbm_gbs": achieved,
        # each request streams its own weights, so the bytes per committed token do not fall with k
        "bytes_per_committed_token": k * (wbytes + kv) * args.steps / max(1, tokk),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "bytes_per_launch": k * (wbytes + kv), "peak_kind": peak_kind,
                     "note": "each request streams its own copy of the weights (no shared weight stream)"},
        "dtype": "q4 weights, fp16 activations, fp32 accumulate",
        "data": "synthetic (seeded random-init q4 weights, uniform prompt ids, seeded trees)",
        "config": {"workload": f"{k} BASELINE config 2 requests (256-token cached prefixes, seeded 16-row "
                               f"trees) per launch, each on 1/{k} of the SMs", "layers": args.layers},
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    for e in engs:
        e.close()


def run_decode_loop(args):
    """The device-resident decode loop (VerifyEngine.generate_drafted): one request with a
    256-token prompt decoded 64 tokens, every step k_draft (the learned drafter on the device, on
    the committed table subset tests/golden/draft_subset.ildraft) + one verify pass, enqueued one
    step ahead, the shape from the adaptive rule. Against it: the same request by plain greedy
    decoding (1-row passes), by the loop with fixed trees and by the loop replaying each step as a
    CUDA graph; k_draft alone; and four requests at once (generate_drafted_batch, each on a quarter
    of the SMs, batch4_*). The weights are
    random-init, so the drafter's candidates (trained on real text) are rarely accepted: the line
    measures the loop's overhead, not a speed-up. One JSON line of its own, 1 GPU."""
    import os

    import torch

    from instantllm_b200 import synth
    from instantllm_b200.drafter import DeviceDrafter
    from instantllm_b200.engine import PassShape, VerifyEngine

    w = synth.make_weights("q4", n_layers=args.layers, seed=args.seed)
    eng = VerifyEngine(w, max_ctx=4096, max_steps=4096, device=0)
    d_path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden", "draft_subset.ildraft")
    d = DeviceDrafter(d_path)
    s = eng.stream
    prompt = synth.make_prompt(PREFIX, seed=args.seed + 7).tolist()
    n_new = 64

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        outs = []
        e0.record(s)
        for _ in range(args.steps):
            outs.append(fn())
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps, outs[-1]

    clocks = ClockSampler(0)
    clocks.start()
    clocks.mark_start()
    ms_loop, r = timed(lambda: eng.generate_drafted(prompt, n_new, d, pids=prompt, text="", depth=1))
    clk = clocks.stop()
    ms_tree, rt = timed(lambda: eng.generate_drafted(prompt, n_new, d, pids=prompt, text="", depth=1,
                                                     shape=PassShape(adaptive=False)))
    ms_graph, rg = timed(lambda: eng.generate_drafted(prompt, n_new, d, pids=prompt, text="", depth=1,
                                                      graphs=True))
    ms_greedy, g = timed(lambda: eng.generate(prompt, n_new))
    # k_draft alone, after the request's last committed token (device state as the loop left it)
    tree_ptr = eng.buffer(7, (synth.TREE_INTS,), "<i4").data_ptr()
    st_ptr, tok_ptr = eng.lib.vp_device_state(eng.ctx), eng.lib.vp_device_tokens(eng.ctx)
    n_tok = len(r["tokens"])
    draft_us = {}
    for B, br in ((15, 8), (7, 1)):
        def draft():
            d.draft(tree_ptr, tok_ptr, n_out=n_tok, B=B, branch=br, stream=eng._s)
        for _ in range(3):
            draft()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(20):
            draft()
        e1.record(s)
        torch.cuda.synchronize()
        draft_us[f"B{B}_branch{br}"] = 1000 * e0.elapsed_time(e1) / 20
    # the prefill alone (the 256-token prompt in 16-row chunks on all SMs), part of every loop above
    def prefill():
        eng.begin(0, n_new, synth.STOP_IDS)
        eng.prefill(prompt)
    ms_prefill, _ = timed(prefill)
    # four requests at once (generate_drafted_batch): drafts side by side, one vp_pass_batch launch
    # per step, each request on a quarter of the SMs; checked against greedy 1-row passes on the
    # same share
    K = 4
    engs = [eng] + [VerifyEngine(w, max_ctx=4096, max_steps=4096, device=0) for _ in range(K - 1)]
    ds = [d] + [DeviceDrafter(d_path) for _ in range(K - 1)]
    prompts = [synth.make_prompt(PREFIX, seed=args.seed + 7 + q).tolist() for q in range(K)]
    ms_b, rb = timed(lambda: VerifyEngine.generate_drafted_batch(engs, prompts, n_new, ds, pids=prompts, depth=1))
    root = torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=eng.device)
    for e in engs:
        e.begin(0, n_new, synth.STOP_IDS)
    VerifyEngine.prefill_batch(engs, prompts)
    for _ in range(n_new - 1):
        VerifyEngine.pass_multi(engs, [root] * K, shares=K)
    batch_equal = all(e.tokens(e.state()["step"]) == q["tokens"] for e, q in zip(engs, rb))

    def prefill4():
        for e in engs:
            e.begin(0, n_new, synth.STOP_IDS)
        VerifyEngine.prefill_batch(engs, prompts)
    ms_prefill4, _ = timed(prefill4)
    batch_tok = sum(len(q["tokens"]) for q in rb)
    for x in ds[1:]:
        x.close()
    for x in engs[1:]:
        x.close()
    ntok = len(r["tokens"])
    line = {
        "metric": "device-resident decode loop (k_draft + verify pass per step, one step enqueued ahead): "
                  "tok/s of one request, prefill included",
        "value": ntok / (ms_loop * 1e-3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True,
        "ms_per_request": ms_loop, "tokens": ntok, "passes": r["passes"],
        "accepted_per_pass": r["state"]["accepted"] / max(1, r["passes"]),
        "shapes": {f"B{b}_branch{br}": r["shapes"].count((b, br)) for b, br in sorted(set(r["shapes"]))},
        "host_waits": r["host_waits"],
        "fixed_tree_loop_tok_s": len(rt["tokens"]) / (ms_tree * 1e-3),
        "graph_loop_tok_s": len(rg["tokens"]) / (ms_graph * 1e-3),
        "greedy_tok_s": len(g["tokens"]) / (ms_greedy * 1e-3),
        "tokens_equal_greedy": r["tokens"] == g["tokens"] == rt["tokens"] == rg["tokens"],
        "k_draft_us": draft_us,
        "prefill_ms": ms_prefill,
        "decode_tok_s": ntok / ((ms_loop - ms_prefill) * 1e-3),
        "batch4_loop_tok_s": batch_tok / (ms_b * 1e-3),
        "batch4_prefill_ms": ms_prefill4,
        "batch4_decode_tok_s": batch_tok / ((ms_b - ms_prefill4) * 1e-3),
        "batch4_ms": ms_b,
        "batch4_tokens_equal_greedy_on_share": bool(batch_equal),
        "dtype": "q4 weights, fp16 activations, fp32 accumulate; drafter float64",
        "data": "synthetic (seeded random-init q4 weights, uniform prompt ids); drafter table: the committed "
                "subset of the reference's table",
        "config": {"workload": f"one request, {PREFIX}-token prompt, {n_new} new tokens, learned drafter on "
                               "the device, adaptive tree / chain", "layers": args.layers},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    d.close()
    eng.close()


def run_cfg34(args, which: str):
    """BASELINE config 3 (q8 group-64 weights, 1024-token cached prefix, 8-row chain passes whose
    draft i equals the true next token with p = 0.5, 64 tokens) or config 4 (f16 weights, a
    512-token prompt prefilled in 16-row chunks, then 16-row seeded trees as in config 2 to 64
    tokens). Truth = the same request decoded with 1-row passes through the same kernels; every
    committed token is checked against it. Timed: the verify passes (device time), and for config 4
    also the chunked prefill. One JSON line of its own, 1 GPU."""
    import torch

    from instantllm_b200 import synth
    from instantllm_b200.engine import VerifyEngine
    from oracle import accept as A
    from oracle import qwen_oracle as Q

    fmt, prefix, rows = ("q8", 1024, 8) if which == "config3" else ("f16", 512, 16)
    gen = 64
    w = synth.make_weights(fmt, n_layers=args.layers, seed=args.seed)
    eng = VerifyEngine(w, max_ctx=prefix + gen + 3 * ROWS + 16, max_steps=gen + ROWS + 2, device=0)
    dev, s = eng.device, eng.stream
    prompt = synth.make_prompt(prefix, seed=3000 + (3 if which == "config3" else 4))
    no_eos = (-1, -1)
    eng.begin(0, gen + ROWS + 1, no_eos)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    eng.prefill(prompt)
    e1.record(s)
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    snap = eng.snapshot()
    tree1 = torch.tensor(synth.tree_to_buffer(synth.root_tree()), device=dev)
    for _ in range(gen + ROWS):
        eng.pass_device(tree1)
    y = eng.tokens(gen + ROWS + 1)
    # pass plan from the truth: the device follows the planned acceptances
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([args.seed, 34, prefix])))
    bufs, counts, pos = [], [], 1
    while pos < gen:
        if which == "config3":
            drafts = [y[pos + i] if rng.random() < 0.5 else int(rng.integers(0, synth.PROMPT_VOCAB))
                      for i in range(rows - 1)]
            tree = synth.chain_tree(drafts)
        else:
            tree = synth.seeded_tree(rng, y[pos:pos + 9], n=rows)
        parents, tokens = A.to_python_numbering(tree)
        a = A.accept_tree(parents, tokens, list(y), pos)
        bufs.append(synth.tree_to_buffer(tree))
        counts.append(a + 1)
        pos += a + 1
    tb = torch.tensor(np.stack(bufs), device=dev)
    for _ in range(args.warmup):  # warm-up passes from the same state, then back to it
        eng.restore(snap)
        eng.pass_device(tb[0])
    eng.restore(snap)
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    clocks.mark_start()
    e0.record(s)
    for k in range(len(bufs)):
        eng.pass_device(tb[k])
    e1.record(s)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    st = eng.state()
    got = eng.tokens(st["step"])
    ok = got == y[:st["step"]] and st["step"] == 1 + sum(counts)
    n_pass = len(bufs)
    pass_ms = ms / n_pass
    hbm_peak, peak_kind = peaks()
    wbytes = synth.weight_bytes(fmt, args.layers)
    # KV bytes per pass: the unique slots read (cached context + the pass's rows) and the rows written
    ctx = [prefix + 1 + sum(counts[:k]) for k in range(n_pass)]
    kv = np.mean([12288 * (c + rows) + 12288 * rows for c in ctx]) * args.layers / 24
    achieved = (wbytes + kv) / (pass_ms * 1e-3) / 1e9
    line = {
        "metric": f"{which}: {fmt} {rows}-row {'chain' if which == 'config3' else 'tree'} verify pass us "
                  "& accepted tok/s; HBM GB/s vs B200 peak",
        "value": (st["step"] - 1) / (ms * 1e-3), "unit": "tok/s", "n_gpus": 1, "higher_is_better": True,
        "passes": n_pass, "pass_us": 1000 * pass_ms, "tokens_per_pass": sum(counts) / n_pass,
        "tree_equals_sequential": bool(ok), "dtype": f"{fmt} weights, fp16 activations, fp32 accumulate",
        "data": "synthetic (seeded random-init weights, uniform prompt ids)",
        "config": {"workload": ("BASELINE config 3: q8 group-64, 1024-token cached prefix, 8-row chains, "
                                "draft i = true token with p = 0.5, 64 tokens") if which == "config3" else
                               ("BASELINE config 4: f16, 512-token prompt prefilled in 16-row chunks, "
                                "16-row seeded trees to 64 tokens"),
                   "layers": args.layers, "timed": "verify passes, device time"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "bytes_per_launch": wbytes + kv, "peak_kind": peak_kind},
        "clocks": clk,
    }
    if which == "config4":
        line["prefill_ms"] = prefill_ms
        line["prefill_tok_s"] = prefix / (prefill_ms * 1e-3)
    if not args.no_cpu_baseline:
        # the oracle (numpy fp32 port of the reference CPU path) on a bounded sample: the prompt,
        # then the same passes until cpu_seconds run out
        threads = host_threads()
        m = Q.model_from_weights(w)
        cache = Q.KVCache(len(m.layers), prefix + gen + 3 * ROWS + 16)
        t0 = time.perf_counter()
        lg = Q.forward_causal(m, cache, list(prompt), 0)
        t_pre = time.perf_counter() - t0
        first, cpos, step, tok, n = int(np.argmax(lg)), prefix, 1, 0, 0
        t1 = time.perf_counter()
        while n < n_pass and time.perf_counter() - t1 < args.cpu_seconds:
            b = bufs[n]
            tr = {"n": int(b[0]), "depth": list(b[1:17]), "parent": list(b[17:33]), "tok": list(b[33:49])}
            lg = Q.tree_pass(m, cache, cpos, first, tr)
            res = A.commit(tr, lg.argmax(axis=1), cpos, step, 1 << 30, eos=())
            for src, dst in res["moves"]:
                for li in range(len(m.layers)):
                    cache.k[li][:, dst] = cache.k[li][:, src]
                    cache.v[li][:, dst] = cache.v[li][:, src]
            tok += len(res["tokens"])
            first, cpos, step, n = res["tokens"][-1], res["pos"], step + len(res["tokens"]), n + 1
        dt = time.perf_counter() - t1
        line["cpu_baseline"] = {"value": tok / dt, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"the {prefix}-token prompt ({t_pre:.1f} s) then {n} of the same "
                                          f"passes ({dt:.1f} s), numpy fp32 with dequantised weights",
                                "pass_ms": 1000 * dt / max(n, 1)}
    print(json.dumps(line), flush=True)
    eng.close()


def main_sketch(args):
    """The optional two-stage sketch lm_head (instantllm_b200.sketch) against the full q4 lm_head
    (vp_head_argmax_noalloc) at the full vocabulary, 1, 4, 8 and 16 rows: device time per call with
    L2 flushed before each call by reading a 256 MiB buffer (the q4 embedding, 76.6 MB, fits in the
    126 MB L2)."""
    import torch

    from instantllm_b200 import _lib, synth
    from instantllm_b200.engine import VerifyEngine
    from instantllm_b200.sketch import SketchHead

    w = synth.make_weights("q4", n_layers=1, seed=args.seed)
    rng = np.random.default_rng(args.seed + 1)
    w["final_norm"] = rng.normal(1.0, 0.1, synth.HIDDEN).astype(np.float32)
    eng = VerifyEngine(w, max_ctx=64, max_steps=8)
    sk = SketchHead(eng, codes=w["embed"]["codes"])
    V, s = eng.vocab, eng.stream
    x = torch.from_numpy(synth.head_rows(w["embed"], w["final_norm"], rng, 16)).to(eng.device)
    tok = torch.empty(16, dtype=torch.int32, device=eng.device)
    flush = torch.ones(64 << 20, dtype=torch.float32, device=eng.device)  # 256 MiB, twice the L2
    flush_sum = torch.zeros((), dtype=torch.float32, device=eng.device)
    ws = eng._weights_struct

    def full(rows):
        _lib.check(eng.lib.vp_head_argmax_noalloc(_lib.FMT["q4"], V, ws.embed, ws.final_norm, x.data_ptr(),
                                                  rows, tok.data_ptr(), s.cuda_stream), "noalloc")

    def sketch(rows):
        sk.argmax_device(x, rows)

    def timed(fn, rows):
        for _ in range(args.warmup):
            fn(rows)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        for a, b in ev:
            flush_sum.copy_(flush.sum())  # a read leaves L2 holding clean lines: no write-backs in the call
            a.record(s)
            fn(rows)
            b.record(s)
        torch.cuda.synchronize()
        return float(np.median([a.elapsed_time(b) for a, b in ev])) * 1000.0

    hbm_peak, peak_kind = peaks()
    sk_bytes = V // 16 * 14 * (256 + 64)  # sketch tiles + the q4 tiles' scale blocks
    full_bytes = V // 16 * 14 * 576
    res = []
    for rows in (1, 4, 8, 16):
        sketch(rows)
        got = sk.argmax(x, rows)
        full(rows)
        torch.cuda.synchronize()
        same = bool(np.array_equal(got, tok[:rows].cpu().numpy()))
        tf, ts = timed(full, rows), timed(sketch, rows)
        c0, call = sk.last_candidates()
        res.append({"rows": rows, "full_us": round(tf, 2), "sketch_us": round(ts, 2),
                    "speedup": round(tf / ts, 3), "same_tokens": same, "cand_groups_row0": c0,
                    "cand_groups_any": call,
                    "full_hbm_gbs": round(full_bytes / (tf * 1e-6) / 1e9, 1),
                    "sketch_stream_gbs": round(sk_bytes / (ts * 1e-6) / 1e9, 1)})
    line = {"metric": "lm_head latency: two-stage sketch head vs full q4 head (median device us per call)",
            "value": res[0]["sketch_us"], "unit": "us", "higher_is_better": False, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "rows": res,
            "config": {"workload": "tied q4 lm_head, vocab 151936, rows mixing embedding rows + noise "
                                   "(clear winners, close runners-up), K = 6", "l2": "flushed before each call (256 MiB read)"},
            "peak_gbs": hbm_peak, "peak_kind": peak_kind,
            "data": "synthetic (seeded random-init q4 embedding)"}
    print(json.dumps(line), flush=True)
    eng.close()


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return
    import torch

    from instantllm_b200 import synth

    if world > 1:
        # requests are independent: no collective on the data path. gloo (host) carries only the
        # barrier around the timed region and the max / sum over ranks of the device timings.
        torch.distributed.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=300))
    if args.workload == "sketch_head":
        main_sketch(args)
        return
    if args.workload in ("config3", "config4"):
        run_cfg34(args, args.workload)
        return
    if args.workload in ("batch2", "batch3", "batch4"):
        run_batch(args, int(args.workload[-1]))
        return
    if args.workload == "decode_loop":
        run_decode_loop(args)
        return
    if args.workload == "config5":
        main_config5(args, rank, world)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    r = run_ours(args, rank, world, local)
    ms, tok = r["ms"], r["tok"]
    e2e_s, e2e_tok = r["e2e_s"], r["e2e_tok"]
    ok = 1.0 if r["ok"] else 0.0
    p50, p90 = (float(np.percentile(r["step_ms"], q)) for q in (50, 90))
    if world > 1:
        t = torch.tensor([ms, float(tok), e2e_s, float(e2e_tok), ok, p50, p90], dtype=torch.float64)
        mx = t.clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        sm = t.clone()
        torch.distributed.all_reduce(sm, op=torch.distributed.ReduceOp.SUM)
        mn = t.clone()
        torch.distributed.all_reduce(mn, op=torch.distributed.ReduceOp.MIN)
        ms, tok, e2e_s, e2e_tok = mx[0].item(), sm[1].item(), mx[2].item(), sm[3].item()
        ok = mn[4].item()
        p50, p90 = mx[5].item(), mx[6].item()
    line = None
    if rank == 0:
        hbm_peak, peak_kind = peaks()
        wbytes = synth.weight_bytes("q4", args.layers)
        pass_ms = r["ms"] / args.steps
        # KV bytes: the unique slots read (the 256 cached + the pass's 16 rows) and the 16 written,
        # 12,288 B per slot at 24 layers
        kv_bytes = 12288 * (PREFIX + ROWS) * args.layers / 24 + 12288 * ROWS * args.layers / 24
        alg = wbytes + kv_bytes
        achieved = alg / (pass_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": tok / (ms * 1e-3),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "step_us_p50": 1000 * p50,  # per-step device time (CUDA events between steps), max over ranks
            "step_us_p90": 1000 * p90,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,  # BASELINE.md publishes a pass time (3.8 ms, Apple M5), not tok/s
            "reference_published": {"pass_us": 3800.0, "hardware": "Apple M5 (README.md:87-88)",
                                    "pass_time_ratio": 3800.0 / (1000 * pass_ms)},
            "dtype": "q4 weights, fp16 activations, fp32 accumulate",
            "data": "synthetic (seeded random-init q4 weights, uniform prompt ids, seeded trees)",
            "config": {"workload": WORKLOAD2, "rows": ROWS, "prefix": PREFIX, "layers": args.layers,
                       "l2": L2_NOTE, "parallelism": f"request sharding x{world}", "timed_as": r["timed_as"]},
            "pass_us": 1000 * pass_ms,
            "tokens_per_pass": tok / max(1, args.steps * world),
            "hbm_gbs": achieved,
            "tree_equals_sequential": bool(ok),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": ncu_traffic(),
                         "kernel": "k_pass: the persistent verify-pass kernel (one launch per pass), rank 0",
                         "bytes_per_launch": alg, "peak_kind": peak_kind},
            # vp_step moves state (64 B) + token slots (64 B) + tree (260 B) in and state + the
            # pass's committed tokens (128 B) out per step
            "e2e": {"value": e2e_tok / e2e_s, "unit": "tok/s",
                    "h2d_bytes_per_step": 64 + 64 + 65 * 4, "d2h_bytes_per_step": 128},
            "gpu_launches": args.steps,  # one persistent k_pass launch per verify pass
            "clocks": r["clocks"],
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(r["w"], r["prompt"], r["y"], r["trees"], args.cpu_seconds)
        else:
            line["cpu_baseline"] = None
    r["eng"].close()
    if args.c5_requests > 0:
        # BASELINE config 5 on the same ranks (strong scaling: a fixed set of requests split over
        # the ranks, longest-processing-time first, no collective on the data path)
        r5 = run_config5(args, rank, world, local, w=r["w"], n_requests=args.c5_requests)
        table = config5_table(args, r5, world)
        if rank == 0:
            line["config5"] = dict(config5_summary(table, args.c5_requests), scaling="strong",
                                   workload="BASELINE config 5: prefixes uniform in [128, 2048], 64 tokens "
                                            f"each, seeded 16-row trees; {C5_HEADLINE} requests per launch "
                                            "(vp_pass_batch), and one, two and four per launch on the same "
                                            "requests under modes; device time of the tree passes, max "
                                            "over ranks")
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
