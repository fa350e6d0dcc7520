"""Timed CPU runs of the oracle on bounded samples of the bench workload —
TEST INFRASTRUCTURE ONLY (used by ``bench.py``'s ``cpu_baseline`` leg and its
``--impl reference`` arm, never by the product path).

A *unit* is one (sequence, Q head) of the workload restricted to a set of
query blocks: the oracle quantises that head's Q and its KV head's K exactly
as the reference's forward does (quantisation is per block and head, so a
one-head slice gives the same codes) and runs the routed attention for the
chosen blocks. Units run in a ``spawn`` process pool, one per worker, so the
sample uses every host core it is given; numpy is pinned to one thread per
worker.
"""
from __future__ import annotations

import os
import time

import numpy as np


def causal_block_flops(block: int, block_m: int, head_dim: int, seqlen: int) -> float:
    """Algorithmic FLOPs of one query block: 4 * D * (number of causal (q, k) pairs)."""
    lo = block * block_m
    hi = min(seqlen, lo + block_m)
    pairs = (hi * (hi + 1) - lo * (lo + 1)) // 2
    return float(4 * head_dim * pairs)


def run_unit(args) -> float:
    """Runs one unit; returns its wall time in seconds."""
    from oracle.attention_oracle import tilemix_attention_with_quant

    q, k, v, words, q_blocks, block_m, block_n, block_n_mask = args
    T = q.shape[0]
    cu = np.array([0, T], dtype=np.int32)
    t0 = time.perf_counter()
    tilemix_attention_with_quant(q, k, v, cu, cu, T, T, words, block_m=block_m, block_n=block_n,
                                 block_n_mask=block_n_mask, causal=True, routing_mode="mixed",
                                 scalar_scales=(block_m == 128 and block_n == 64), int8_use_fp16_v=True,
                                 q_blocks=q_blocks)
    return time.perf_counter() - t0


def _init_worker():
    os.environ["OMP_NUM_THREADS"] = "1"


def host_cores(cap: int = 96) -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, min(n, cap))


def make_pool(workers: int):
    import multiprocessing as mp

    os.environ.setdefault("OMP_NUM_THREADS", "1")
    return mp.get_context("spawn").Pool(workers, initializer=_init_worker)
