"""Input generators and comparison helpers shared by the test files."""
from __future__ import annotations

import numpy as np
import torch


def make_qkv(batch_lens, hq, hk, d, seed=0, outliers=0, outlier_scale=20.0):
    """Packed fp16 q, k, v ~ N(0,1) with optional fixed outlier channels per (tensor, head).

    Returns (q, k, v, cu) as CPU tensors; ``cu`` is int32 cu_seqlens.
    """
    g = torch.Generator().manual_seed(seed)
    total = int(sum(batch_lens))
    q = torch.randn((total, hq, d), generator=g).to(torch.float16)
    k = torch.randn((total, hk, d), generator=g).to(torch.float16)
    v = torch.randn((total, hk, d), generator=g).to(torch.float16)
    if outliers:
        for t, heads in ((q, hq), (k, hk)):
            for h in range(heads):
                ch = torch.randperm(d, generator=g)[:outliers]
                t[:, h, ch] = (t[:, h, ch].float() * outlier_scale).to(torch.float16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(batch_lens)]), dtype=torch.int32)
    return q, k, v, cu


def make_bias(n_seq, hq, T, seed, scale=2.0):
    """Seeded fp16 additive bias [n_seq, hq, T, T] ~ scale * N(0, 1) (CPU tensor)."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn((n_seq, hq, T, T), generator=g) * scale).to(torch.float16)


def random_bitmask(rows, seed=1):
    rng = np.random.default_rng(seed)
    words = rng.integers(0, 2**63, size=rows, dtype=np.int64).astype(np.uint64)
    words ^= rng.integers(0, 2, size=rows, dtype=np.int64).astype(np.uint64) << np.uint64(63)
    return torch.from_numpy(words.view(np.int64).copy()).view(torch.uint64)


def err_stats(out, ref, rows_valid=None):
    o = out.float().cpu().numpy() if isinstance(out, torch.Tensor) else np.asarray(out, dtype=np.float32)
    r = ref.float().cpu().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref, dtype=np.float32)
    d = np.abs(o.astype(np.float32) - r.astype(np.float32))
    return float(d.max()), float(d.mean())
