"""CPU tests of bench.py's strong-scaling partition: over the ranks of a world size, the
problems cover every (sequence x KV-head) unit of the workload exactly once, their FLOPs
add up to the workload's, and the KV-head-block views read the right heads in place."""
import pytest
import torch

import bench


@pytest.fixture
def small_cfg(monkeypatch):
    cfg = dict(bench.CFG, batch=3, seq_len=256, heads_q=6, heads_k=2, head_dim=64)
    monkeypatch.setattr(bench, "CFG", cfg)
    return cfg


def _inputs(c):
    g = torch.Generator().manual_seed(0)
    n = c["batch"] * c["seq_len"]
    q = torch.randn((n, c["heads_q"], c["head_dim"]), generator=g).to(torch.float16)
    k = torch.randn((n, c["heads_k"], c["head_dim"]), generator=g).to(torch.float16)
    v = torch.randn((n, c["heads_k"], c["head_dim"]), generator=g).to(torch.float16)
    o = torch.zeros_like(q)
    cu = torch.arange(0, (c["batch"] + 1) * c["seq_len"], c["seq_len"], dtype=torch.int32)
    words = torch.arange(1, c["seq_len"] // c["block_m"] + 1, dtype=torch.int64).view(torch.uint64)
    return q, k, v, o, cu, words


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_partition_covers_every_unit_once(small_cfg, world):
    c = small_cfg
    q, k, v, o, cu, words = _inputs(c)
    seen, flops = [], 0.0
    for rank in range(world):
        problems, desc = bench.make_problems(q, k, v, o, cu, words, rank, world)
        assert desc
        for p in problems:
            seen.extend(p["units"])
            flops += bench.problem_flops(p)
    assert sorted(seen) == [(b, h) for b in range(c["batch"]) for h in range(c["heads_k"])]
    assert flops == bench.attention_flops()


def test_head_block_views_read_in_place(small_cfg):
    """World 2 divides the 2 KV heads: rank r's views are heads of the full tensors, and the
    output view writes into the full output."""
    c = small_cfg
    q, k, v, o, cu, words = _inputs(c)
    g = c["heads_q"] // c["heads_k"]
    for rank in range(2):
        (p,), _ = bench.make_problems(q, k, v, o, cu, words, rank, 2)
        assert "packed" not in p
        assert torch.equal(p["k"], k[:, rank:rank + 1])
        assert torch.equal(p["q"], q[:, rank * g:(rank + 1) * g])
        assert p["o"].data_ptr() == o[:, rank * g:].data_ptr()
        assert p["pm"].numel() == c["seq_len"] // c["block_m"]
