#!/usr/bin/env python
"""Benchmark of the B200 TileMix hot path: routed FP16/INT8 flash attention.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

Workload (the reference's headline attention configuration): 8 sequences x
4096 tokens, 24 query heads / 8 KV heads (Llama-3.2-3B), head_dim 128, fp16
Q/K/V ~ N(0, 1) with 4 outlier channels per (tensor, head) scaled x20 on Q and
K, causal, SpTrans routing at 50% INT8, tiles (128, 64, 64). A *step* is one
forward over the batch: per-block INT8 quantisation of K, then the fused
attention kernel (Q is quantised inside it); the routing map is built once
beforehand, as the model integration caches it.

One process per GPU (torchrun for N > 1), strong scaling: the one workload's
64 (sequence x KV-head) units are split over the ranks with no collective
(with N dividing the 8 KV heads, rank r owns KV heads [8r/N, 8(r+1)/N) of every
sequence and writes its output in place); ``value`` is the workload's FLOPs
divided by the slowest rank's time. Rank 0 prints one JSON line, which at N=1
also carries the reference's own Triton kernels timed on the same GPU and
inputs (``triton_reference``) and the all-FP16 / all-INT8 patterns.

``--impl reference`` times the reference's CPU path on the host cores: the
CPU restatement of its kernels (the oracle, bit-exact with the reference run
under the Triton interpreter) on a bounded sample of the same workload; under
torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import datetime as _dt
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

METRIC = "attention TFLOP/s (SpTrans50, 8x4096, Llama-3.2-3B heads)"
UNIT = "TFLOP/s"
CFG = dict(batch=8, seq_len=4096, heads_q=24, heads_k=8, head_dim=128, outliers=4, outlier_scale=20.0,
           pattern="sptrans", percentage=0.5, block_m=128, block_n=64, block_n_mask=64)
FALLBACK_PEAKS = dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0)
# The reference's own CPU path is its Triton kernels under TRITON_INTERPRET=1; measured on one
# unit of this workload (3 Q heads / 1 KV head, T = 4096, sptrans 50 %) it ran at this rate.
INTERPRETER_NOTE = ("the reference's kernels under TRITON_INTERPRET=1 ran one (sequence, KV-head) unit of this "
                    "workload (3 Q heads, T = 4096) in 50.8 s on one core: 0.254 GFLOP/s per core, about 3x "
                    "slower per core than the port timed here")


def config_dict(n_gpus: int, shard: str = "") -> dict:
    c = CFG
    tokens = c["batch"] * c["seq_len"]
    rd = tokens * (c["heads_q"] + 2 * c["heads_k"]) * c["head_dim"] * 2
    wr = tokens * (2 * c["heads_q"] + c["heads_k"]) * c["head_dim"]
    return {
        "workload": f"attention op, config 2: {c['batch']} x {c['seq_len']} tokens, 24 q / 8 kv heads, head_dim 128, "
                    "causal, sptrans 50% INT8, tiles (128, 64, 64), 4 outlier channels x20",
        "batch": c["batch"], "seq_len": c["seq_len"], "heads_q": c["heads_q"], "heads_k": c["heads_k"],
        "head_dim": c["head_dim"], "pattern": c["pattern"], "int8_percentage": c["percentage"],
        "block_m": c["block_m"], "block_n": c["block_n"], "block_n_mask": c["block_n_mask"],
        "parallelism": f"shard{n_gpus}: the {c['batch'] * c['heads_k']} (sequence x KV-head) units of the one "
                       f"workload split over {n_gpus} GPU(s), no collective" + (f"; rank 0: {shard}" if shard else ""),
        "l2": f"inputs larger than L2 (126 MB): each step reads Q, K, V ({rd / 1e6:.0f} MB) and writes O and K8 "
              f"({wr / 1e6:.0f} MB) over all ranks; no flush",
    }


def attention_flops() -> float:
    c = CFG
    T = c["seq_len"]
    return float(4 * c["head_dim"] * c["heads_q"] * c["batch"] * T * (T + 1) // 2)


def make_inputs(seed: int):
    """Seeded fp16 inputs of the workload, packed token-major [B*T, H, D] on the CPU."""
    import torch

    c = CFG
    g = torch.Generator().manual_seed(seed)
    n = c["batch"] * c["seq_len"]
    q = torch.randn((n, c["heads_q"], c["head_dim"]), generator=g).to(torch.float16)
    k = torch.randn((n, c["heads_k"], c["head_dim"]), generator=g).to(torch.float16)
    v = torch.randn((n, c["heads_k"], c["head_dim"]), generator=g).to(torch.float16)
    for t, heads in ((q, c["heads_q"]), (k, c["heads_k"])):
        for h in range(heads):
            ch = torch.randperm(c["head_dim"], generator=g)[: c["outliers"]]
            t[:, h, ch] = (t[:, h, ch].float() * c["outlier_scale"]).to(torch.float16)
    return q, k, v


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profiled_traffic(kernel_tag: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    p = REPO / "profiles" / f"{kernel_tag}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def int8_share(words, block_m: int, block_n: int, block_n_mask: int, T: int) -> float:
    """Executed INT8 share of the QK tile work of one KV head under the map (causal)."""
    group = block_n_mask // block_n
    tot = int8 = 0
    n_tiles = (T + block_n - 1) // block_n
    for r, w in enumerate(words):
        n = min(n_tiles, ((r + 1) * block_m + block_n - 1) // block_n)
        for t in range(n):
            tot += 1
            int8 += (int(w) >> (t // group)) & 1
    return int8 / tot if tot else 0.0


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.6)
        except OSError:
            self.proc = None

    def mark(self, t0: float, t1: float):
        self.window = (t0, t1)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi unavailable"}
        time.sleep(0.15)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = []
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                ts = _dt.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[1]), float(parts[2]), parts[3:7]))
            except ValueError:
                continue
        inside = [r for r in rows if self.window and self.window[0] <= r[0] <= self.window[1]]
        used = inside or rows
        reasons = sorted({self.REASONS[i] for r in used for i, s in enumerate(r[3]) if s.lower() == "active"})
        return {
            "sm_mhz": statistics.median([r[1] for r in used]) if used else None,
            "sm_max_mhz": max(r[2] for r in used) if used else None,
            "reasons": reasons,
            "samples": len(used),
            "window": "run-up + timed region" if inside else "whole run (no sample inside the timed region)",
        }


def gpu_id_for(device_index: int) -> str:
    import torch

    try:
        uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        return uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[device_index] if vis else str(device_index)


# ---------------------------------------------------------------------------
# CPU legs (oracle), shared by the cpu_baseline field and --impl reference
# ---------------------------------------------------------------------------
def cpu_units(q, k, v, words, n_units: int, step_budget_s: float, rate_flops: float = 0.9e9):
    """Tasks of one CPU step: n_units (sequence, Q head) units of the workload, each
    restricted to evenly spread query blocks so that a unit takes about step_budget_s."""
    import numpy as np
    from oracle.cpu_sample import causal_block_flops

    c = CFG
    T, bm, D = c["seq_len"], c["block_m"], c["head_dim"]
    nblk = (T + bm - 1) // bm
    full = sum(causal_block_flops(b, bm, D, T) for b in range(nblk))
    want = step_budget_s * rate_flops
    count = nblk if want >= full else max(1, int(round(nblk * want / full)))
    blocks = sorted({int(x) for x in np.linspace(0, nblk - 1, count).round()})
    group = c["heads_q"] // c["heads_k"]
    words_np = np.asarray(words, dtype=np.uint64)
    tasks, flops = [], 0.0
    for i in range(n_units):
        b = i % c["batch"]
        hq = (i // c["batch"]) % c["heads_q"]
        hk = hq // group
        sl = slice(b * T, (b + 1) * T)
        tasks.append((q[sl, hq:hq + 1].copy(), k[sl, hk:hk + 1].copy(), v[sl, hk:hk + 1].copy(), words_np, blocks,
                      bm, c["block_n"], c["block_n_mask"]))
        flops += sum(causal_block_flops(x, bm, D, T) for x in blocks)
    sample = (f"{n_units} (sequence, Q head) units of the workload, {len(blocks)} of {nblk} query blocks each "
              f"(spread over the causal triangle), Q/K quantisation included")
    return tasks, flops, sample


def oracle_map_words():
    from oracle.precision_maps_oracle import make_precision_bitmask

    c = CFG
    return make_precision_bitmask(c["seq_len"], c["block_m"], c["block_n_mask"], None, c["percentage"], c["pattern"],
                                  {"percentage": c["percentage"]}, c["block_n"])


def run_reference(args) -> None:
    """--impl reference: the CPU restatement of the reference's kernels on the host cores."""
    from oracle.cpu_sample import host_cores, make_pool

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = host_cores()
    pool = make_pool(cores)
    try:
        q, k, v = (t.numpy() for t in make_inputs(0))
        words = oracle_map_words()
        budget = min(20.0, max(1.0, 150.0 / max(1, args.steps + args.warmup)))
        tasks, flops, sample = cpu_units(q, k, v, words, cores, budget)
        for _ in range(args.warmup):
            pool.map(run_unit_proxy(), tasks, chunksize=1)
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            pool.map(run_unit_proxy(), tasks, chunksize=1)
            times.append(time.perf_counter() - t0)
    finally:
        pool.close()
        pool.join()
    step_s = sum(times) / len(times)
    value = flops / step_s / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16+int8", "data": "synthetic (seeded N(0,1) with outlier channels)",
        "config": config_dict(args.gpus), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU restatement of the reference's Triton kernels (bit-exact with them under TRITON_INTERPRET=1), "
                "numpy, one process per host core",
    }
    print(json.dumps(line), flush=True)


def run_unit_proxy():
    from oracle.cpu_sample import run_unit

    return run_unit


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def make_problems(q, k, v, o, cu, words, rank: int, world: int):
    """This rank's share of the workload as launches over views of the resident tensors.

    Units are (sequence x KV-head) pairs; every one is independent, so no data crosses
    ranks. When the world size divides the KV heads a rank owns a contiguous KV-head block
    of every sequence: its Q/K/V/O are strided views of the full tensors and its output
    lands in place. Otherwise units are dealt longest-processing-time first
    (tilemix_b200/sharding.py) and packed into one single-KV-head problem before the timed
    region; its output then has to be scattered back (timed separately)."""
    import torch

    from tilemix_b200.sharding import head_block_views, kv_head_block, pack_units, plan_units

    c = CFG
    B, T, HQ, HK, bm = c["batch"], c["seq_len"], c["heads_q"], c["heads_k"], c["block_m"]
    g = HQ // HK
    mb = (T + bm - 1) // bm
    hb = kv_head_block(HK, world, rank)
    if hb is not None:
        h0, h1 = hb
        pm_all = words.view(torch.int64).repeat(HK).view(torch.uint64)
        qv, kv, vv, ov, pm = head_block_views(q, k, v, o, pm_all, mb, hb)
        return [dict(q=qv, k=kv, v=vv, o=ov, cu=cu, T=T, pm=pm,
                     units=[(b, h) for b in range(B) for h in range(h0, h1)])], \
            f"kv-head block [{h0}, {h1}) of every sequence (views, output in place)"
    units = plan_units([T] * B, HK, world, g)[rank]
    cu_list = [i * T for i in range(B + 1)]
    q_r, k_r, v_r, cu_r, _ = pack_units(q, k, v, cu_list, units)
    # every KV head reads the same routing words in this workload (the map is head-independent)
    return [dict(q=q_r, k=k_r, v=v_r, o=torch.empty_like(q_r), cu=cu_r, T=T, pm=words, units=units,
                 packed=True)], f"{len(units)} (sequence x KV-head) units dealt longest first, packed"


def problem_flops(p) -> float:
    c = CFG
    g = c["heads_q"] // c["heads_k"]
    T = c["seq_len"]
    return float(4 * c["head_dim"] * g * len(p["units"]) * T * (T + 1) // 2)


def measure_int8_peak(dev) -> dict:
    """Dense INT8 tensor throughput of this GPU: torch._int_mm (cuBLASLt) on 8192^3, best of 10."""
    import torch

    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev).t().contiguous().t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return {"int8_tops": 2 * n ** 3 / (best * 1e-3) / 1e12, "how": "torch._int_mm int8 8192^3 -> int32, best of 10"}


MAP_PATTERNS = ("zero", "one", "band", "global", "row_rand", "align_sparse", "bigbird", "sptrans")


def map_builder_leg(dev, reps: int = 50) -> dict:
    """The routing-map kernel (``tm_build_precision_map``) for every pattern at the workload's
    geometry (T, block_m, block_n_mask, block_n) and 50 % INT8: CUDA-event time per build over
    ``reps`` back-to-back asynchronous launches, and the achieved HBM rate of its algorithmic
    traffic (it reads no tensor and writes one uint64 word per query block)."""
    import torch

    from tilemix_b200.attention.precision_maps import make_precision_bitmask

    c = CFG
    T, bm, bnm, bn, pct = c["seq_len"], c["block_m"], c["block_n_mask"], c["block_n"], c["percentage"]
    out = {}
    for pattern in MAP_PATTERNS:
        params = {"percentage": pct} if pattern not in ("zero", "one") else {}

        def build(check=False):
            return make_precision_bitmask(T, bm, bnm, None, pct, pattern, params, bn, device=dev, check_retarget=check)

        words = build(check=True)
        for _ in range(3):
            build()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            build()
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        nbytes = words.numel() * 8
        out[pattern] = {"us_per_build": us, "bytes_written": nbytes, "gb_per_s": nbytes / (us * 1e-6) / 1e9}
    return {"kernel": "build_map_kernel (tm_build_precision_map)", "seq_len": T, "block_m": bm,
            "block_n_mask": bnm, "percentage": pct, "patterns": out,
            "note": "one CTA per map; latency-bound by the reference's sequential retarget walk and MT19937 "
                    "draws, not by HBM (the whole map is ceil(T / block_m) words); each time includes the "
                    "host-side launch of its call"}


def triton_reference_leg(q, k, v, cu, pm_by_pattern: dict, steps: int, warmup: int) -> dict:
    """The reference's own Triton implementation on this GPU (unmodified, from baseline/_ref):
    tilemix_attention_with_quant (Q and K quantisation + attn_fwd) with the configuration its
    prefill benchmark forces (TILEMIX_FORCE_CONFIG=128,64,8,2,0), timed with CUDA events like
    our step, beside the same call through this package's drop-in API on the same inputs, and
    the largest / mean absolute difference of the two outputs."""
    import torch

    ref_root = REPO / "baseline" / "_ref"
    if not (ref_root / "attention" / "triton" / "tilemix.py").exists():
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    if str(ref_root) not in sys.path:
        sys.path.append(str(ref_root))
    os.environ["TILEMIX_FORCE_CONFIG"] = "128,64,8,2,0"
    try:
        from attention.triton.tilemix import tilemix_attention_with_quant as ref_call
    except Exception as e:  # noqa: BLE001 - report, do not fail the bench line
        return {"unavailable": f"importing the reference failed: {type(e).__name__}: {e}"}
    from tilemix_b200.attention.tilemix import tilemix_attention_with_quant as our_call

    c = CFG
    T = c["seq_len"]
    flops = attention_flops()

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / steps

    out = {"impl": "reference Triton kernels (attention/triton/tilemix.py:1340-1447, unmodified) on this GPU",
           "config": "TILEMIX_FORCE_CONFIG=128,64,8,2,0 (BLOCK_M 128, BLOCK_N 64, 8 warps, 2 stages)",
           "step": "tilemix_attention_with_quant: Q and K quantisation + attn_fwd", "patterns": {}}
    cases = [(name, pm, mode, True) for name, (pm, mode) in pm_by_pattern.items()]
    cases.append(("sptrans, int8_use_fp16_v=False (the API default)", pm_by_pattern["sptrans"][0], "mixed", False))
    for name, pm, mode, fp16_v in cases:
        kw = dict(block_m=c["block_m"], block_n=c["block_n"], block_n_mask=c["block_n_mask"], causal=True,
                  routing_mode=mode, scalar_scales=True, int8_use_fp16_v=fp16_v)
        try:
            o_ref, _ = ref_call(q, k, v, cu, cu, T, T, pm, **kw)
            ms_ref = timed(lambda: ref_call(q, k, v, cu, cu, T, T, pm, **kw))
        except Exception as e:  # noqa: BLE001
            out["patterns"][name] = {"unavailable": f"{type(e).__name__}: {e}"}
            continue
        o_ours, _ = our_call(q, k, v, cu, cu, T, T, pm, **kw)
        ms_ours = timed(lambda: our_call(q, k, v, cu, cu, T, T, pm, **kw))
        d = (o_ours.float() - o_ref.float()).abs()
        out["patterns"][name] = {
            "triton_ms": ms_ref, "triton_tflops": flops / (ms_ref * 1e-3) / 1e12,
            "ours_same_api_ms": ms_ours, "ours_same_api_tflops": flops / (ms_ours * 1e-3) / 1e12,
            "speedup": ms_ref / ms_ours,
            "max_abs_diff": float(d.max()), "mean_abs_diff": float(d.mean()),
            "bit_identical_share": float((d == 0).float().mean()),
        }
        del o_ref, o_ours, d
    sp = out["patterns"].get("sptrans", {})
    out["ms"] = sp.get("triton_ms")
    out["ratio_ours_over_triton"] = sp.get("speedup")
    return out


def run_ours(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    pool = None
    if want_cpu:  # the oracle's process pool starts before the first CUDA call
        from oracle.cpu_sample import host_cores, make_pool

        cpu_cores = host_cores()
        pool = make_pool(cpu_cores)

    import torch
    import torch.distributed as dist

    from tilemix_b200.attention import tilemix as tmx
    from tilemix_b200.attention.precision_maps import make_precision_bitmask
    from tilemix_b200.attention.tilemix_varlen import tilemix_varlen_attention_from_host
    from tilemix_b200.sharding import unpack_units

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=_dt.timedelta(seconds=180), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    c = CFG
    B, T, HQ, HK, D = c["batch"], c["seq_len"], c["heads_q"], c["heads_k"], c["head_dim"]
    bm, bn, bnm = c["block_m"], c["block_n"], c["block_n_mask"]
    # The whole workload, identical on every rank; each rank computes only its shard.
    q_cpu, k_cpu, v_cpu = make_inputs(0)
    q, k, v = q_cpu.to(dev), k_cpu.to(dev), v_cpu.to(dev)
    cu = torch.arange(0, (B + 1) * T, T, device=dev, dtype=torch.int32)
    o = torch.empty_like(q)
    sm_scale = D ** -0.5
    thr = tmx.rescale_threshold()

    def pattern_words(pattern):
        params = {"percentage": c["percentage"]} if pattern not in ("zero", "one") else {}
        return make_precision_bitmask(T, bm, bnm, None, c["percentage"], pattern, params, bn, device=dev)

    words = pattern_words(c["pattern"])
    words_host = [int(x) for x in words.view(torch.int64).cpu().numpy().view("uint64")]
    share = int8_share(words_host, bm, bn, bnm, T)
    problems, shard_desc = make_problems(q, k, v, o, cu, words, rank, world)
    rank_flops = sum(problem_flops(p) for p in problems)
    total_flops = attention_flops()

    def make_step(probs, pm_key, mode_code):
        def step(evs=None):
            for i, p in enumerate(probs):
                k8 = sk16 = cuks = None
                vkw = {}
                if mode_code != tmx.ROUTING_MODE_FP16:
                    k8, sk16, cuks = tmx._quantize_k(p["k"], p["cu"], p["T"], 64, equal_len=p["T"])
                    if args.int8_v:  # the API default's V path: V quantised, its codes as fp16 values
                        v16, sv16, cuvs = tmx._quantize_v_f16(p["v"], p["cu"], p["T"], 64, equal_len=p["T"])
                        vkw = dict(v8_f16=v16, sv=sv16, cuvs=cuvs)
                if evs is not None:
                    evs[i][0].record()
                tmx._launch(p["q"], p["k"], p["v"], p["o"], p["cu"], p["cu"], p[pm_key], p["T"], p["T"], k8=k8,
                            sk=sk16, cuks=cuks, block_m=bm, block_n=bn, block_n_mask=bnm, BLKQ=128, BLKK=64,
                            causal=True, sm_scale=sm_scale, mode_code=mode_code, scalar_scales=True,
                            int8_use_fp16_v=not args.int8_v, threshold=thr, **vkw)
                if evs is not None:
                    evs[i][1].record()
        return step

    step = make_step(problems, "pm", tmx.ROUTING_MODE_MIXED)
    for _ in range(args.warmup):
        step()
    barrier()
    if tmx.device_error_code(dev) != 0:
        raise RuntimeError("attention kernel reported a device-side timeout during warm-up")

    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in problems]
           for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(gpu_id_for(local_rank))
    sampler.start()
    # The timed steps take milliseconds, less than the sampler's 100 ms period: the same steps
    # run back to back for about a second right before them, untimed, so that the clock
    # samples (window: this run-up and the timed region) see the GPU under this load.
    barrier()
    t_host0 = time.time()
    while time.time() - t_host0 < 1.0:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    barrier()
    start.record()
    for i in range(args.steps):
        step(evs[i])
    end.record()
    barrier()
    t_host1 = time.time()
    sampler.mark(t_host0, t_host1)
    clocks = sampler.stop()
    ms_step = max_over_ranks(start.elapsed_time(end) / args.steps)
    attn_ms = max_over_ranks(sum(a.elapsed_time(b) for row in evs for a, b in row) / args.steps)
    if tmx.device_error_code(dev) != 0:
        raise RuntimeError("attention kernel reported a device-side timeout in the timed region")

    # the output scatter of a packed shard (not needed for KV-head blocks: they write in place)
    scatter_ms = 0.0
    if any(p.get("packed") for p in problems):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for p in problems:
            unpack_units(p["o"], [i * T for i in range(B + 1)], p["units"], o)
        e1.record()
        barrier()
        scatter_ms = max_over_ranks(e0.elapsed_time(e1))

    # the same step with the all-FP16 and all-INT8 maps (BASELINE config 2's other patterns);
    # the routing mode is the one routing_mode="auto" selects for them
    pattern_lines = {"sptrans": {"ms_per_step": ms_step, "tflops": total_flops / (ms_step * 1e-3) / 1e12,
                                 "routing_mode": "mixed"}}
    pm_by_pattern = {"sptrans": (words.view(torch.int64).repeat(HK).view(torch.uint64), "mixed")}
    for pattern, mode in (("zero", "fp16"), ("one", "int8")):
        w_p = pattern_words(pattern)
        pm_by_pattern[pattern] = (w_p.view(torch.int64).repeat(HK).view(torch.uint64), mode)
        for p in problems:
            p["pm_" + pattern] = w_p.view(torch.int64).repeat(p["pm"].numel() // w_p.numel()).view(torch.uint64)
        st = make_step(problems, "pm_" + pattern, tmx._routing_mode_code(mode))
        for _ in range(args.warmup):
            st()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            st()
        e1.record()
        barrier()
        ms_p = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        pattern_lines[pattern] = {"ms_per_step": ms_p, "tflops": total_flops / (ms_p * 1e-3) / 1e12,
                                  "routing_mode": mode}
    if tmx.device_error_code(dev) != 0:
        raise RuntimeError("attention kernel reported a device-side timeout (patterns)")

    # end to end through the public API for host-resident data: this rank's shard of Q, K, V
    # in pinned host memory, its output back to pinned host memory, every byte crossing PCIe
    # inside the timed region (sequences are streamed, so copies in, attention and copies out
    # overlap)
    host = []
    for p in problems:
        host.append(dict(q=p["q"].cpu().contiguous().pin_memory(), k=p["k"].cpu().contiguous().pin_memory(),
                         v=p["v"].cpu().contiguous().pin_memory(),
                         o=torch.empty(tuple(p["q"].shape), dtype=torch.float16).pin_memory(), pm=p["pm"]))

    def e2e_step():
        for h in host:
            tilemix_varlen_attention_from_host(h["q"], h["k"], h["v"], h["o"], T, bm, bn, block_n_mask=bnm,
                                               causal=True, scale=sm_scale, precision_map_all=h["pm"], device=dev,
                                               chunk_seqs=1, ring=2)

    e2e_steps = max(3, min(args.steps, 30))
    for _ in range(max(3, min(args.warmup, 5))):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    h2d = sum((h["q"].numel() + h["k"].numel() + h["v"].numel()) * 2 for h in host)
    d2h = sum(h["o"].numel() * 2 for h in host)
    if world > 1:
        t = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        h2d, d2h = int(t[0].item()), int(t[1].item())
    del host

    value = total_flops / (ms_step * 1e-3) / 1e12
    peaks, peak_src = load_peaks()
    peak16 = float(peaks["bf16_tflops"])
    int8 = measure_int8_peak(dev)
    peak8 = -max_over_ranks(-int8["int8_tops"])  # the slowest GPU's
    achieved = rank_flops / (attn_ms * 1e-3) / 1e12
    t_star_ms = (rank_flops / 2 * (1 - share) / peak16 + rank_flops / 2 * share / peak8 + rank_flops / 2 / peak16) \
        / 1e12 * 1e3
    traffic = profiled_traffic("attn_fwd_paired_int8v_config2" if args.int8_v else "attn_fwd_paired_config2")
    if traffic is not None and world > 1:
        traffic = int(traffic * rank_flops / total_flops)

    map_line = map_builder_leg(dev) if world == 1 else None
    triton_line = None
    if world == 1 and not args.no_triton_reference:
        triton_line = triton_reference_leg(q, k, v, cu, pm_by_pattern, min(args.steps, 20), args.warmup)

    cpu_line = None
    if want_cpu:
        try:
            # Four whole (sequence, Q head) units per core: ~13 s of CPU work on the B200 host.
            tasks, cflops, sample = cpu_units(q_cpu.numpy(), k_cpu.numpy(), v_cpu.numpy(), oracle_map_words(),
                                              4 * cpu_cores, 8.0)
            t0 = time.perf_counter()
            pool.map(run_unit_proxy(), tasks, chunksize=1)
            dt = time.perf_counter() - t0
            cpu_line = {"value": cflops / dt / 1e12, "unit": UNIT, "cores": cpu_cores, "kind": "port",
                        "sample": sample, "seconds": dt, "interpreter_note": INTERPRETER_NOTE}
        finally:
            pool.close()
            pool.join()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16+int8", "data": "synthetic (seeded N(0,1) with outlier channels)",
            "config": {**config_dict(world, shard_desc),
                       "v_path": ("INT8-V (int8_use_fp16_v=False): the step also quantises V" if args.int8_v
                                  else "FP16 V for INT8 tiles (int8_use_fp16_v=True)")},
            "roofline": {
                "bound": "tensor", "kernel": "attn_fwd_paired", "achieved": achieved,
                "peak": rank_flops / t_star_ms / 1e9, "unit": "TFLOP/s", "frac": t_star_ms / attn_ms,
                "traffic": traffic,
                "peak_source": f"routed FP16/INT8 mix: bf16_tflops (burst) of {peak_src} for the FP16 share and "
                               "the INT8 GEMM peak measured in this run (torch._int_mm) for the INT8 share",
                "kernel_ms": attn_ms, "t_star_ms": t_star_ms, "flops_per_launch": rank_flops, "int8_share": share,
                "peak_fp16": peak16, "peak_int8": peak8, "int8_peak_measurement": int8["how"],
                "bf16_frac": achieved / peak16,
            },
            "patterns": pattern_lines,
            "map_builder": map_line,
            "triton_reference": triton_line,
            "cpu_baseline": cpu_line,
            "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "steps": e2e_steps,
                    "api": "tilemix_varlen_attention_from_host (pinned host q/k/v/out of each rank's shard, "
                           "1 sequence per chunk)"},
            "scatter_ms": scatter_ms,
            "clocks": clocks,
            "gpu_launches": (3 if args.int8_v else 2) * len(problems) * args.steps,
            "rescale_threshold": thr,
            "numerics": tmx.numerics_mode(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def run_prefill_components(args) -> None:
    """--component prefill: the Llama prefill companions at the workload's shapes (8 x 4096
    tokens of Llama-3.2-3B: hidden 3072, 24 / 8 heads of 128, MLP 8192), each timed with CUDA
    events over --steps launches after --warmup, against the measured HBM copy peak. One
    JSON line; the default bench line is unaffected."""
    import torch

    from tilemix_b200.models.tilemix_llama import rms_norm, rotary_token_major, rotary_token_major_quant_k, silu_mul

    dev = torch.device("cuda", 0)
    B, T, HQ, HK, D, HID, MLP = CFG["batch"], CFG["seq_len"], CFG["heads_q"], CFG["heads_k"], CFG["head_dim"], 3072, 8192
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn((B, T, (HQ + 2 * HK) * D), device=dev, generator=g).half()
    q = qkv[..., : HQ * D].view(B, T, HQ, D).transpose(1, 2)
    k = qkv[..., HQ * D:(HQ + HK) * D].view(B, T, HK, D).transpose(1, 2)
    cos = torch.randn((1, T, D), device=dev, generator=g).half()
    sin = torch.randn((1, T, D), device=dev, generator=g).half()
    gate = torch.randn((B, T, MLP), device=dev, generator=g).half()
    up = torch.randn((B, T, MLP), device=dev, generator=g).half()
    x = torch.randn((B, T, HID), device=dev, generator=g).half()
    w = torch.rand((HID,), device=dev, generator=g).half()
    peaks, src = load_peaks()
    tok = B * T
    rope_bytes = 2 * tok * (HQ + HK) * D * 2 + 2 * T * D * 2
    cases = [
        ("rotary_token_major", lambda: rotary_token_major(q, k, cos, sin), rope_bytes),
        ("rotary_token_major_quant_k", lambda: rotary_token_major_quant_k(q, k, cos, sin, 64),
         rope_bytes + tok * HK * D + tok // 64 * HK * 2),
        ("silu_mul", lambda: silu_mul(gate, up), 3 * tok * MLP * 2),
        ("rms_norm", lambda: rms_norm(x, w, 1e-5), 2 * tok * HID * 2 + HID * 2),
    ]
    out = []
    for name, fn, nbytes in cases:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        gbs = nbytes / (ms * 1e-3) / 1e9
        out.append({"kernel": name, "ms": ms, "algorithmic_bytes": nbytes, "achieved_gbs": gbs,
                    "peak_gbs": peaks["hbm_gbs"], "frac": gbs / peaks["hbm_gbs"]})
    print(json.dumps({"component": "prefill companions", "bound": "hbm", "peak_source": f"hbm_gbs of {src}",
                      "config": {"batch": B, "seq_len": T, "heads_q": HQ, "heads_k": HK, "head_dim": D,
                                 "hidden": HID, "mlp": MLP},
                      "steps": args.steps, "warmup": args.warmup, "kernels": out}), flush=True)


LLAMA_3B = dict(hidden_size=3072, intermediate_size=8192, num_hidden_layers=28, num_attention_heads=24,
                num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-5, rope_theta=500000.0, vocab_size=128256,
                tie_word_embeddings=True, max_position_embeddings=8192, initializer_range=0.02,
                hidden_act="silu")
QWEN2_7B = dict(hidden_size=3584, intermediate_size=18944, num_hidden_layers=28, num_attention_heads=28,
                num_key_value_heads=4, rms_norm_eps=1e-6, rope_theta=1000000.0, vocab_size=152064,
                tie_word_embeddings=False, max_position_embeddings=32768, initializer_range=0.02,
                hidden_act="silu")
# name: (config 3 / 4 of the headline benchmark) architecture, batch, tokens, patterns, A100 ms or None
MODEL_SPECS = {
    "llama3b": dict(label="Llama-3.2-3B", config=3, arch=LLAMA_3B, batch=8, seq_len=4096, patterns=("sptrans",),
                    a100_ms=1071.0,  # the reference paper's 30.59 K tok/s at B=8, L=4K on an A100 (derived)
                    a100_note="vs_baseline = ms / 1071 ms, the A100 40GB figure derived from the reference paper"),
    "qwen7b": dict(label="Qwen2-7B", config=4, arch=QWEN2_7B, batch=4, seq_len=16384, patterns=("band", "bigbird"),
                   a100_ms=None, a100_note="the reference publishes no Qwen2-7B number beyond 4K tokens"),
}


def run_model_prefill(args) -> None:
    """--component model: whole-model prefill through the public model API (config 3:
    Llama-3.2-3B, 8 x 4096 tokens, sptrans 50 %; ``--model qwen7b``, config 4: Qwen2-7B,
    4 x 16384 tokens, band and bigbird at 50 %): random-init weights (seed 0, std 0.02, fp16),
    TileMix attention injected and the routing pattern configured (Llama also
    prepare_llama_prefill), uniform token ids, PrefillCache and last-position logits. Under
    torchrun the layers are head-sharded across the N ranks (TP N, one NCCL all-reduce after
    each attention and MLP block). Each timed prefill is bracketed by a barrier and a
    synchronize; a line per pattern reports the median over prefills of the slowest rank's
    time, as the reference's prefill benchmark takes the median."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    import torch.distributed as dist

    from tilemix_b200.models.tensor_parallel import shard_model_for_tensor_parallel
    from tilemix_b200.models.tilemix_llama import PrefillCache

    spec = MODEL_SPECS[args.model]
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=_dt.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    if args.model == "llama3b":
        from transformers import LlamaConfig as Config, LlamaForCausalLM as Model

        from tilemix_b200.models.tilemix_llama import configure_tilemix_attention_pattern as configure
        from tilemix_b200.models.tilemix_llama import inject_tilemix_into_llama as inject
        from tilemix_b200.models.tilemix_llama import prepare_llama_prefill as prepare
    else:
        from transformers import Qwen2Config as Config, Qwen2ForCausalLM as Model

        from tilemix_b200.models.tilemix_qwen import configure_tilemix_attention_pattern as configure
        from tilemix_b200.models.tilemix_qwen import inject_tilemix_into_qwen as inject
        prepare = None
    B, T = spec["batch"], spec["seq_len"]
    cfg = Config(**spec["arch"])
    torch.manual_seed(0)
    with torch.device(dev):
        model = Model(cfg)
    model = model.half().eval()
    inject(model)
    if prepare is not None:
        prepare(model)
    if world > 1:
        shard_model_for_tensor_parallel(model, rank, world)
    torch.cuda.empty_cache()
    ids_host = torch.randint(0, cfg.vocab_size, (B, T), generator=torch.Generator().manual_seed(0)).pin_memory()
    logits_host = torch.empty((B, 1, cfg.vocab_size), dtype=torch.float16).pin_memory()

    def prefill(ids):
        with torch.inference_mode():
            return model(ids, past_key_values=PrefillCache(), use_cache=True, logits_to_keep=1).logits

    ids = ids_host.to(dev)
    steps, warmup = max(5, min(args.steps, 20)), max(3, min(args.warmup, 5))
    for pattern in spec["patterns"]:
        configure(model, pattern, percentage=0.5)
        for _ in range(warmup):
            prefill(ids)
        barrier()
        sampler = ClockSampler(gpu_id_for(local_rank))
        sampler.start()
        times, t_host0 = [], time.time()
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            e0.record()
            prefill(ids)
            e1.record()
            barrier()
            times.append(e0.elapsed_time(e1))
        # end to end: token ids from pinned host memory in, last-position logits back, per prefill
        e2e_times = []
        for _ in range(max(3, steps // 2)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            e0.record()
            logits_host.copy_(prefill(ids_host.to(dev, non_blocking=True)), non_blocking=True)
            e1.record()
            barrier()
            e2e_times.append(e0.elapsed_time(e1))
        t_host1 = time.time()
        sampler.mark(t_host0, t_host1)
        clocks = sampler.stop()
        if world > 1:
            t = torch.tensor([times, e2e_times + [0.0] * (len(times) - len(e2e_times))], dtype=torch.float64,
                             device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times = t[0].tolist()
            e2e_times = t[1, :len(e2e_times)].tolist()
        ms = statistics.median(times)
        e2e_ms = statistics.median(e2e_times)
        if rank == 0:
            a100 = spec["a100_ms"]
            print(json.dumps({
                "metric": f"{spec['label']} prefill ms (config {spec['config']})", "value": ms, "unit": "ms",
                "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": False,
                "scaling": "strong", "vs_baseline": (ms / a100) if a100 else None, "dtype": "fp16+int8",
                "data": "synthetic (random-init weights seed 0 std 0.02, uniform token ids seed 0)",
                "config": {"workload": f"config {spec['config']}: {spec['label']} architecture, prefill {B} x {T} "
                                       f"tokens with KV cache and last-position logits, {pattern} 50% INT8",
                           "model": f"{spec['label']} (random init)", "global_batch": B, "seq_len": T,
                           "pattern": pattern,
                           "parallelism": f"tp{world}" + (": heads and MLP columns sharded, NCCL all-reduce "
                                                          "after o_proj and down_proj" if world > 1 else ""),
                           "l2": "every prefill moves the full weights and activations, far above L2"},
                "tokens_per_s": B * T / (ms * 1e-3), "ms_all": times,
                "e2e": {"value": e2e_ms, "unit": "ms",
                        "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(),
                        "d2h_bytes_per_step": logits_host.numel() * logits_host.element_size()},
                "baseline_note": spec["a100_note"], "clocks": clocks,
            }), flush=True)
    del model
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


VARLEN = dict(sequences=8, min_len=8192, max_len=131072, heads_q=32, heads_k=8, head_dim=128)
# Config 5's grid: every percentage-driven pattern at INT8 shares 0 / 25 / 50 / 75 / 100 %, plus the
# all-FP16 and all-INT8 maps.
VARLEN_PCTS = (0.0, 0.25, 0.5, 0.75, 1.0)
VARLEN_CASES = tuple((p, pct) for p in ("sptrans", "band", "global", "row_rand", "align_sparse", "bigbird")
                     for pct in VARLEN_PCTS) + (("zero", None), ("one", None))


def run_varlen(args) -> None:
    """--component varlen: config 5, the long-context varlen attention op. 8 sequences of
    lengths uniform in [8K, 128K] (torch.randint, seed 1), 32 q / 8 kv heads, head_dim 128,
    fp16 N(0, 1), causal, tiles (128, 64) with the mask-group width the model picks for the
    longest sequence; one line per routing case (pattern, INT8 share). A step is K
    quantisation + the attention over the whole batch. Under torchrun the (sequence x KV-head)
    units are dealt to the ranks longest-processing-time first (tilemix_b200/sharding.py) and
    packed before the timed region, in groups that read the same routing words, so every
    rank's results equal the unsharded call's; value = all ranks' FLOPs / slowest rank's
    time (strong scaling)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    import torch.distributed as dist

    from tilemix_b200.attention import tilemix as tmx
    from tilemix_b200.attention.precision_maps import make_precision_bitmask
    from tilemix_b200.models._attention_base import pick_mask_block_n
    from tilemix_b200.sharding import map_rows, pack_units, plan_units, unpack_units

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=_dt.timedelta(seconds=300), device_id=dev)
    c = VARLEN
    lens = torch.randint(c["min_len"], c["max_len"] + 1, (c["sequences"],),
                         generator=torch.Generator().manual_seed(1)).tolist()
    cu_list = [0]
    for n in lens:
        cu_list.append(cu_list[-1] + n)
    T_max, HQ, HK, D = max(lens), c["heads_q"], c["heads_k"], c["head_dim"]
    group = HQ // HK
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn((cu_list[-1], HQ, D), device=dev, generator=g, dtype=torch.float16)
    k = torch.randn((cu_list[-1], HK, D), device=dev, generator=g, dtype=torch.float16)
    v = torch.randn((cu_list[-1], HK, D), device=dev, generator=g, dtype=torch.float16)
    bm, bn = 128, 64
    bnm = pick_mask_block_n(T_max, bn)
    flops = float(sum(4 * D * HQ * n * (n + 1) // 2 for n in lens))
    units = plan_units(lens, HK, world, group)[rank]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    results = []
    o_full = torch.empty_like(q) if world > 1 else None
    steps = max(3, min(args.steps, 5))
    for pattern, pct in VARLEN_CASES:
        words = make_precision_bitmask(T_max, bm, bnm, None, pct, pattern,
                                       {"percentage": pct} if pct is not None else {}, bn, device=dev)
        pm = words.view(torch.int64).repeat(HK).view(torch.uint64)
        pack_ms = 0.0
        if world == 1:
            cu = torch.tensor(cu_list, dtype=torch.int32, device=dev)
            problems = [(q, k, v, cu, T_max, pm, None)]
        else:
            # the rank's units packed into single-KV-head problems (a gather of its Q/K/V
            # rows), grouped by the routing words they read; timed, outside the step
            by_rows: dict = {}
            for u in units:
                off, _ = map_rows(pm, u, lens[u[0]], bm)
                by_rows.setdefault(off, []).append(u)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            problems = []
            for off, us in sorted(by_rows.items()):
                q_r, k_r, v_r, cu_r, mx = pack_units(q, k, v, cu_list, us)
                problems.append((q_r, k_r, v_r, cu_r, mx, pm[off:off + (mx + bm - 1) // bm].contiguous(), us))
            e1.record()
            torch.cuda.synchronize()
            pack_ms = e0.elapsed_time(e1)
        outs = [torch.empty_like(pr[0]) for pr in problems]

        def step():
            for (q_, k_, v_, cu_, mx_, pm_, _), o_ in zip(problems, outs):
                tmx._attention_forward(q_, k_, v_, cu_, cu_, mx_, mx_, pm_, block_m=bm, block_n=bn, block_n_mask=bnm,
                                       BLKQ=128, BLKK=64, causal=True, sm_scale=None, mode="mixed",
                                       scalar_scales=True, int8_use_fp16_v=True, o=o_)

        for _ in range(2):
            step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        barrier()
        ms = e0.elapsed_time(e1) / steps
        scatter_ms = 0.0
        if world > 1:
            # the rank's outputs scattered back into the [tokens, HQ, D] layout (timed, outside the step)
            e0.record()
            for (_, _, _, _, _, _, us), o_ in zip(problems, outs):
                unpack_units(o_, cu_list, us, o_full)
            e1.record()
            torch.cuda.synchronize()
            scatter_ms = e0.elapsed_time(e1)
            t = torch.tensor([ms, pack_ms, scatter_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, pack_ms, scatter_ms = (float(x) for x in t.tolist())
        if tmx.device_error_code(dev) != 0:
            raise RuntimeError("attention kernel reported a device-side timeout")
        results.append({"pattern": pattern, "int8_percentage": pct, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12,
                        "launches_per_step": len(problems), "pack_ms": pack_ms, "scatter_ms": scatter_ms,
                        "tflops_with_pack_and_scatter": flops / ((ms + pack_ms + scatter_ms) * 1e-3) / 1e12})
        del problems, outs
    if rank == 0:
        print(json.dumps({
            "component": "varlen attention (config 5)", "unit": "TFLOP/s", "n_gpus": world,
            "scaling": "strong", "dtype": "fp16+int8", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": "config 5: 8 packed sequences, lengths uniform in [8K, 128K] (seed 1), "
                                   "32 q / 8 kv heads, head_dim 128, causal", "lengths": lens,
                       "tokens": cu_list[-1], "block_m": bm, "block_n": bn, "block_n_mask": bnm,
                       "parallelism": f"shard{world}: (sequence x KV-head) units dealt longest first, no collective"},
            "flops_per_step": flops, "steps": steps, "warmup": 2, "cases": results,
            "pack_scatter_note": "at N > 1 each rank gathers its units' Q/K/V rows into packed problems and scatters "
                                 "its outputs back; both are timed per case outside the step (pack_ms, scatter_ms)",
        }), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the oracle timing on the host cores")
    ap.add_argument("--int8-v", action="store_true",
                    help="INT8-routed tiles take the INT8-V PV path (int8_use_fp16_v=False, the API's default): "
                         "the step also quantises V")
    ap.add_argument("--no-triton-reference", action="store_true",
                    help="skip timing the reference's Triton kernels on the GPU (N=1 line)")
    ap.add_argument("--batch", type=int, default=CFG["batch"],
                    help="sequences per GPU (default: the workload's 8; smaller only for profiling captures)")
    ap.add_argument("--model", choices=tuple(MODEL_SPECS), default="llama3b",
                    help="--component model: llama3b (config 3) or qwen7b (config 4)")
    ap.add_argument("--component", choices=("attention", "prefill", "model", "varlen"), default="attention",
                    help="prefill: time the Llama prefill companion kernels instead; model: Llama-3.2-3B prefill "
                         "ms through the model API (tensor-parallel over the ranks under torchrun); varlen: the "
                         "long-context varlen sweep (config 5)")
    args = ap.parse_args()
    CFG["batch"] = args.batch
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.component == "prefill":
        run_prefill_components(args)
    elif args.component == "model":
        run_model_prefill(args)
    elif args.component == "varlen":
        run_varlen(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
