"""CPU tests of the multi-GPU host logic: (sequence x KV-head) unit planning,
packing / unpacking, and a world_size-2 gloo run whose assembled output must
equal the unsharded computation bit for bit (the per-shard compute is the CPU
oracle, standing in for the CUDA kernel)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention_oracle as ora
from tests.helpers import make_qkv, random_bitmask
from tilemix_b200.sharding import (head_block_views, kv_head_block, pack_units, plan_units, sharded_attention,
                                   unit_cost, unpack_units)

LENS, HQ, HK, D, BM = [130, 64, 200, 17], 4, 2, 64, 64


def test_plan_covers_every_unit_once_and_balances():
    lens = [4096, 100, 2000, 8192, 513]
    for world in (1, 2, 3, 8):
        plan = plan_units(lens, 8, world, group=3)
        flat = sorted(u for p in plan for u in p)
        assert flat == [(b, h) for b in range(len(lens)) for h in range(8)]
        loads = [sum(unit_cost(lens[b], 3) for b, _ in p) for p in plan]
        assert max(loads) - min(loads) <= max(unit_cost(n, 3) for n in lens)
        assert plan == plan_units(lens, 8, world, group=3)  # deterministic


def test_pack_unpack_roundtrip():
    q, k, v, cu = make_qkv(LENS, HQ, HK, D, seed=3)
    units = [(2, 1), (0, 0), (3, 1)]
    q_r, k_r, v_r, cu_r, mx = pack_units(q, k, v, cu.tolist(), units)
    assert q_r.shape == (200 + 130 + 17, HQ // HK, D) and k_r.shape[1] == 1 and mx == 200
    assert cu_r.tolist() == [0, 200, 330, 347]
    out = torch.zeros_like(q)
    unpack_units(q_r, cu.tolist(), units, out)
    for b, h in units:
        s, e = int(cu[b]), int(cu[b + 1])
        assert torch.equal(out[s:e, 2 * h:2 * h + 2], q[s:e, 2 * h:2 * h + 2])


def _oracle_attn(q_r, k_r, v_r, cu_r, mx, rows):
    out = ora.tilemix_attention_with_quant(q_r.numpy(), k_r.numpy(), v_r.numpy(), cu_r.numpy(), cu_r.numpy(), mx, mx,
                                           rows.view(torch.int64).numpy().view(np.uint64), block_m=BM, block_n=64,
                                           block_n_mask=64, causal=True, routing_mode="mixed", scalar_scales=False,
                                           int8_use_fp16_v=True)
    return torch.from_numpy(out)


def _worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, cu = make_qkv(LENS, HQ, HK, D, seed=5, outliers=2)
        pm = random_bitmask(HK * ((max(LENS) + BM - 1) // BM), seed=9)
        out = sharded_attention(q, k, v, cu.tolist(), pm, BM, _oracle_attn, rank=rank, world_size=world)
        if rank == 0:
            torch.save(out, result_path)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_two_rank_gloo_matches_unsharded(tmp_path):
    path = str(tmp_path / "out.pt")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    got = torch.load(path)
    q, k, v, cu = make_qkv(LENS, HQ, HK, D, seed=5, outliers=2)
    pm = random_bitmask(HK * ((max(LENS) + BM - 1) // BM), seed=9)
    full = ora.tilemix_attention_with_quant(q.numpy(), k.numpy(), v.numpy(), cu.numpy(), cu.numpy(), max(LENS),
                                            max(LENS), pm.view(torch.int64).numpy().view(np.uint64), block_m=BM,
                                            block_n=64, block_n_mask=64, causal=True, routing_mode="mixed",
                                            scalar_scales=False, int8_use_fp16_v=True)
    assert np.array_equal(got.numpy().view(np.uint16), full.view(np.uint16))


def test_kv_head_blocks_partition_the_heads():
    for heads_k in (1, 2, 4, 8):
        for world in (1, 2, 4, 8):
            blocks = [kv_head_block(heads_k, world, r) for r in range(world)]
            if heads_k % world:
                assert all(b is None for b in blocks)
                continue
            assert blocks[0][0] == 0 and blocks[-1][1] == heads_k
            assert all(b[1] == n[0] for b, n in zip(blocks, blocks[1:]))
            assert len({b[1] - b[0] for b in blocks}) == 1


def test_head_block_views_assemble_the_unsharded_output():
    """Equal-length batch (the bench's and the model's): each KV-head block run on its views
    (the oracle standing in for the kernel) writes its slice of the full output in place;
    the union over the blocks equals the unsharded call bit for bit, with a map whose rows
    differ per KV head."""
    lens = [150, 150, 150]
    q, k, v, cu = make_qkv(lens, HQ, HK, D, seed=4, outliers=1)
    mb = (150 + BM - 1) // BM
    pm = random_bitmask(HK * mb, seed=2)
    full = _oracle_attn(q, k, v, cu, 150, pm)
    out = torch.zeros_like(q)
    for r in range(2):
        qv, kv, vv, ov, pmv = head_block_views(q, k, v, out, pm, mb, kv_head_block(HK, 2, r))
        ov.copy_(_oracle_attn(qv.contiguous(), kv.contiguous(), vv.contiguous(), cu, 150, pmv.contiguous()))
    assert torch.equal(out, full)
