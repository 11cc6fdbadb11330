"""Request-level sharding across GPUs.

A single request's verify pass does not shard: its 24 layers form one serial chain of ~100 short
dependent steps, so splitting a pass across GPUs would add collectives inside a pass that is
shorter than a collective. Independent requests shard trivially: every GPU holds a full weight
replica (278 MB at q4) and serves its own queue, with no NCCL and no peer traffic on the data path.

The reference serves one request at a time on one device (Server.swift:131); this module only adds
the assignment of a request list to ranks.
"""
from __future__ import annotations

import heapq

import numpy as np

GEN_TOKENS = 64


def request_cost(prefix: int, gen: int = GEN_TOKENS) -> float:
    """Relative cost of a request: its passes stream the weights once each and read a KV prefix
    that grows with the context; dominated by the pass count, so weight the prefix lightly."""
    return gen * (1.0 + (prefix + gen / 2) / 16384.0)


def assign(prefixes, world: int, gen: int = GEN_TOKENS) -> list:
    """Longest-processing-time-first assignment of requests to `world` ranks.

    Returns one list of request indices per rank. Deterministic: ties broken by index and rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(prefixes)), key=lambda i: (-request_cost(prefixes[i], gen), i))
    heap = [(0.0, r) for r in range(world)]
    out = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + request_cost(prefixes[i], gen), r))
    for lst in out:
        lst.sort()
    return out


def config5_requests(n: int = 256, seed: int = 5, lo: int = 128, hi: int = 2048):
    """Prefix lengths of config 5: n requests with prefixes uniform in [lo, hi]."""
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 55])))
    return [int(v) for v in rng.integers(lo, hi + 1, size=n)]


def groups(indices, prefixes, k: int) -> list:
    """A rank's requests grouped k per launch (vp_pass_batch puts each request of a group on 1/k of
    the SMs, and the launch lasts as long as its slowest share): sorted by prefix length, longest
    first, and grouped with their neighbours, so the shares of a launch read KV prefixes of similar
    length. The last group holds the shortest requests left (fewer than k if k does not divide the
    count). Deterministic: ties broken by index."""
    if k < 1:
        raise ValueError("k must be >= 1")
    order = sorted(indices, key=lambda i: (-prefixes[i], i))
    return [tuple(order[j:j + k]) for j in range(0, len(order), k)]


def pairs(indices, prefixes) -> list:
    """groups(indices, prefixes, 2): two requests per launch."""
    return groups(indices, prefixes, 2)
