"""CPU oracle for the routing-map builder — TEST INFRASTRUCTURE ONLY.

Restates ``make_precision_bitmask`` of the reference
(attention/precision_maps.py:404-636) for every path the model integration
uses: ``token_mask=None`` with a percentage for band / global / row_rand /
align_sparse / bigbird / sptrans, plus zero and one. It returns the packed
``uint64`` row words (bit j of row i = mask group j routed to INT8).

Random draws go through :mod:`oracle.mt19937`, a restatement of torch's CPU
generator and ``randperm``; unlike the reference, this module never touches
torch's global RNG. ``tests/golden/make_golden.py`` runs the reference itself
and ``tests/test_oracle_maps.py`` checks this module against those fixtures
bit for bit.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use
this module; the product path builds maps with the CUDA kernel
``tm_build_precision_map``.
"""
from __future__ import annotations

import numpy as np

from oracle.mt19937 import MT19937, randperm

PERCENT_PATTERNS = ("band", "global", "row_rand", "align_sparse", "bigbird", "sptrans")


def causal_compute_tile_weights(seq_len: int, block_m: int, block_n_mask: int, compute_block_n: int) -> np.ndarray:
    """Visited compute tiles per (query block, mask group) — precision_maps.py:238-270."""
    if block_n_mask % compute_block_n != 0:
        raise ValueError(f"block_n_mask ({block_n_mask}) must be a multiple of compute_block_n ({compute_block_n})")
    num_m = (seq_len + block_m - 1) // block_m
    num_mask_n = (seq_len + block_n_mask - 1) // block_n_mask
    num_compute_n = (seq_len + compute_block_n - 1) // compute_block_n
    group = block_n_mask // compute_block_n
    w = np.zeros((num_m, num_mask_n), dtype=np.int64)
    for row in range(num_m):
        tiles = min(num_compute_n, ((row + 1) * block_m + compute_block_n - 1) // compute_block_n)
        full, rem = divmod(tiles, group)
        if full:
            w[row, :full] = group
        if rem and full < num_mask_n:
            w[row, full] = rem
    return w


def retarget_weighted_int8_fraction(sparse: np.ndarray, weights: np.ndarray, percentage: float,
                                    seed: int = 42) -> np.ndarray:
    """Greedy walk to an exact weighted INT8 fraction — precision_maps.py:273-326."""
    if percentage < 0.0 or percentage > 1.0:
        raise ValueError(f"percentage must be in [0, 1], got {percentage}")
    visited = weights > 0
    result = sparse.astype(bool) & visited
    total = int(weights.sum())
    if total == 0:
        return result
    target = int(round(total * percentage))
    current = int((weights * result).sum())
    if current == target:
        return result
    add = current < target
    cand = np.argwhere(((~result) if add else result) & visited)  # row-major, like torch.nonzero
    order = randperm(len(cand), MT19937(seed))
    for pos in order.tolist():
        row, col = int(cand[pos][0]), int(cand[pos][1])
        w = int(weights[row, col])
        proposed = current + w if add else current - w
        if abs(target - proposed) <= abs(target - current):
            result[row, col] = add
            current = proposed
        if current == target:
            break
    max_w = int(weights.max())
    if abs(current - target) > max_w:
        raise RuntimeError(
            "unable to retarget executable INT8 fraction within one mask-bit "
            f"weight: target={target}, achieved={current}, max_weight={max_w}")
    return result


def sptrans_block_map(seq_len, block_m, block_n_mask, compute_block_n, percentage, params) -> np.ndarray:
    """precision_maps.py:329-385."""
    num_m = (seq_len + block_m - 1) // block_m
    num_n = (seq_len + block_n_mask - 1) // block_n_mask
    sparse = np.ones((num_m, num_n), dtype=bool)
    stride = params.get("stride", min(128, seq_len // 4))
    c = params.get("c", min(32, stride // 4))
    for row in range(num_m):
        qs = row * block_m
        qe = min(seq_len, (row + 1) * block_m)
        for qstride in range(qs // stride, (qe - 1) // stride + 1):
            ss = qstride * stride
            se = min((qstride + 1) * stride, qe)
            sb = ss // block_n_mask
            eb = min(num_n, (se + block_n_mask - 1) // block_n_mask)
            if sb < num_n:
                sparse[row, sb:eb] = False
            for prev in range(qstride):
                ps = prev * stride
                pe = (prev + 1) * stride
                ts = max(ps, pe - c)
                tsb = ts // block_n_mask
                teb = min(num_n, (pe + block_n_mask - 1) // block_n_mask)
                if tsb < num_n:
                    sparse[row, tsb:teb] = False
    w = causal_compute_tile_weights(seq_len, block_m, block_n_mask, compute_block_n)
    return retarget_weighted_int8_fraction(sparse, w, percentage, seed=42)


def pack_block_precision_map(sparse: np.ndarray) -> np.ndarray:
    """Bit j of each row word = column j — precision_maps.py:388-401."""
    if sparse.ndim != 2 or sparse.shape[1] > 64:
        raise ValueError(f"block_precision_map must be 2D with at most 64 columns, got {tuple(sparse.shape)}")
    out = np.zeros(sparse.shape[0], dtype=np.uint64)
    for j in range(sparse.shape[1]):
        out |= sparse[:, j].astype(np.uint64) << np.uint64(j)
    return out


def make_precision_bitmask(seq_len: int, BLOCK_M: int, BLOCK_N: int, token_mask=None, percentage: float = None,
                           pattern_type: str = None, pattern_params: dict = None,
                           COMPUTE_BLOCK_N: int = None) -> np.ndarray:
    """Packed routing words for the percentage-aware paths — precision_maps.py:404-636."""
    num_m = (seq_len + BLOCK_M - 1) // BLOCK_M
    num_n = (seq_len + BLOCK_N - 1) // BLOCK_N
    if COMPUTE_BLOCK_N is None:
        COMPUTE_BLOCK_N = BLOCK_N
    if BLOCK_N % COMPUTE_BLOCK_N != 0:
        raise ValueError(f"BLOCK_N(mask) ({BLOCK_N}) must be a multiple of COMPUTE_BLOCK_N ({COMPUTE_BLOCK_N})")
    if num_n > 64:
        raise ValueError(f"num_n_mask={num_n} > 64; BLOCK_N(mask) too small (seq_len={seq_len}, "
                         f"BLOCK_N(mask)={BLOCK_N})")
    if pattern_type in ("zero", "one"):
        w = causal_compute_tile_weights(seq_len, BLOCK_M, BLOCK_N, COMPUTE_BLOCK_N)
        sparse = np.zeros_like(w, dtype=bool) if pattern_type == "zero" else (w > 0)
        return pack_block_precision_map(sparse)
    if pattern_type == "sptrans" and percentage is not None and pattern_params is not None:
        return pack_block_precision_map(
            sptrans_block_map(seq_len, BLOCK_M, BLOCK_N, COMPUTE_BLOCK_N, percentage, pattern_params))
    direct = percentage is not None and pattern_type in PERCENT_PATTERNS and pattern_params is not None
    if token_mask is None and not direct:
        raise ValueError("token_mask may be None only for a percentage-aware block policy")
    if not direct:
        raise NotImplementedError("token-mask routing maps are outside the restated paths")
    p = float(percentage)
    if pattern_type == "band":
        tbb = int(round(num_n * (1.0 - p)))
        if tbb % 2 == 0:
            tbb = max(1, tbb - 1)
        tbb = max(1, min(tbb, num_n))
        sparse = np.ones((num_m, num_n), dtype=bool)
        for i in range(num_m):
            sparse[i, max(0, i - tbb // 2):min(num_n, i + tbb // 2 + 1)] = False
    elif pattern_type == "global":
        tgc = max(1, min(int(round(num_n * (1.0 - p))), num_n))
        key_pos = pattern_params.get("key_pos", list(range(min(4, seq_len))))
        cols = set()
        for pos in key_pos:
            if 0 <= pos < seq_len:
                bc = pos // BLOCK_N
                if bc < num_n:
                    cols.add(bc)
        while len(cols) < tgc and len(cols) < num_n:
            for col in range(num_n):
                if col not in cols:
                    cols.add(col)
                    break
        cols = sorted(cols)[:tgc]
        sparse = np.ones((num_m, num_n), dtype=bool)
        for col in cols:
            if 0 <= col < num_n:
                sparse[:, col] = False
    elif pattern_type == "row_rand":
        trb = max(1, min(int(round(num_n * (1.0 - p))), num_n))
        sparse = np.ones((num_m, num_n), dtype=bool)
        gen = MT19937(42)  # torch.manual_seed(42) on the global generator
        for i in range(num_m):
            sparse[i, randperm(num_n, gen)[:trb]] = False
    elif pattern_type == "align_sparse":
        tab = max(1, min(int(round(num_n * (1.0 - p))), num_n))
        sparse = np.ones((num_m, num_n), dtype=bool)
        sparse[:, max(0, num_n - tab):] = False
    elif pattern_type == "bigbird":
        thp = max(1, min(int(round(num_m * num_n * (1.0 - p))), num_m * num_n))
        sparse = np.ones((num_m, num_n), dtype=bool)
        n_global = pattern_params.get("num_global_block", 2)
        n_rand = pattern_params.get("num_rand_block", 3)
        tbr = max(1, min(int(round(num_n * (1.0 - p) * 0.5)), num_n))
        bw = tbr + 1 if tbr % 2 == 0 else tbr
        bw = min(bw, num_n)
        for i in range(num_m):
            center = min(i, num_n - 1)
            sparse[i, max(0, center - bw // 2):min(num_n, center + bw // 2 + 1)] = False
        for col in range(min(n_global, num_n)):
            sparse[:, col] = False
            if col < num_m:
                sparse[col, :] = False
        nrpr = min(n_rand, num_n)
        gen = MT19937(42)
        for i in range(num_m):
            sparse[i, randperm(num_n, gen)[:nrpr]] = False
        chp = int((~sparse).sum())
        if chp < thp:
            lpi = np.argwhere(sparse)
            k = thp - chp
            if k > 0 and len(lpi) > 0:
                for idx in randperm(len(lpi), gen)[:k].tolist():
                    sparse[lpi[idx][0], lpi[idx][1]] = False
        elif chp > thp:
            hpi = np.argwhere(~sparse)
            k = chp - thp
            if k > 0 and len(hpi) > 0:
                for idx in randperm(len(hpi), gen)[:k].tolist():
                    sparse[hpi[idx][0], hpi[idx][1]] = True
    else:
        raise ValueError(f"unsupported pattern {pattern_type!r}")
    w = causal_compute_tile_weights(seq_len, BLOCK_M, BLOCK_N, COMPUTE_BLOCK_N)
    sparse = retarget_weighted_int8_fraction(sparse, w, p, seed=42)
    return pack_block_precision_map(sparse)
