"""CPU tests of the head-sharded tensor parallelism (tilemix_b200/models/tensor_parallel.py):
the head and column splits, and gloo runs (2 and 4 ranks) whose sharded Llama / Qwen2
forward must reproduce the unsharded model's logits. The attention inside these CPU runs is
HF's own (the TileMix kernel needs a GPU); the sharding, the local head bookkeeping and the
all-reduces are the same code the GPU prefill runs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tilemix_b200.models.tensor_parallel import column_split, head_split


def test_head_split_llama_3b_even():
    for world in (1, 2, 4, 8):
        splits = [head_split(24, 8, r, world) for r in range(world)]
        assert [s.num_q for s in splits] == [24 // world] * world
        assert [s.num_kv for s in splits] == [8 // world] * world
        assert splits[0].q_lo == 0 and splits[-1].q_hi == 24 and splits[-1].kv_hi == 8
        for s in splits:  # a rank's Q heads belong to its KV heads' groups
            assert s.q_lo // 3 == s.kv_lo and (s.q_hi - 1) // 3 == s.kv_hi - 1


def test_head_split_qwen_7b_replicated_kv():
    splits = [head_split(28, 4, r, 8) for r in range(8)]
    assert [(s.q_lo, s.q_hi) for s in splits] == [(0, 4), (4, 7), (7, 11), (11, 14), (14, 18), (18, 21),
                                                  (21, 25), (25, 28)]
    assert [s.kv_lo for s in splits] == [0, 0, 1, 1, 2, 2, 3, 3]
    assert all(s.num_kv == 1 for s in splits)
    assert [head_split(28, 4, r, 2).num_q for r in range(2)] == [14, 14]


def test_head_split_rejects_impossible_layouts():
    with pytest.raises(ValueError):
        head_split(24, 6, 0, 4)  # neither divides the other
    with pytest.raises(ValueError):
        head_split(4, 2, 0, 8)  # a KV head on 4 ranks with only 2 query heads
    with pytest.raises(ValueError):
        head_split(10, 4, 0, 2)  # query heads do not group


def test_column_split_covers_and_balances():
    for n, world in ((8192, 8), (18944, 8), (10, 4)):
        parts = [column_split(n, r, world) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        sizes = [hi - lo for lo, hi in parts]
        assert max(sizes) - min(sizes) <= 1


def _tiny(kind: str):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    if kind == "llama":
        cfg = LlamaConfig(hidden_size=128, intermediate_size=200, num_hidden_layers=2, num_attention_heads=8,
                          num_key_value_heads=4, vocab_size=300, max_position_embeddings=256)
        model = LlamaForCausalLM(cfg)
    else:
        cfg = Qwen2Config(hidden_size=96, intermediate_size=150, num_hidden_layers=2, num_attention_heads=6,
                          num_key_value_heads=2, vocab_size=300, max_position_embeddings=256)
        model = Qwen2ForCausalLM(cfg)
        with torch.no_grad():  # nonzero QKV biases, so their slicing is exercised
            for layer in model.model.layers:
                for proj in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj):
                    proj.bias.normal_(0, 0.1)
    return model.float().eval()


def _worker(rank, world, port, kind, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tilemix_b200.models.tensor_parallel import shard_model_for_tensor_parallel

        model = _tiny(kind)
        ids = torch.randint(0, 300, (2, 40), generator=torch.Generator().manual_seed(1))
        shard_model_for_tensor_parallel(model)
        with torch.no_grad():
            logits = model(ids).logits
        if rank == 0:
            torch.save(logits, result_path)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
@pytest.mark.parametrize("kind,world", [("llama", 2), ("qwen", 4)])
def test_sharded_forward_matches_unsharded(tmp_path, kind, world):
    """Llama at 2 ranks (KV heads split); Qwen2 at 4 ranks (each KV head on two ranks, its
    three query heads split 2 + 1, QKV biases sliced with them)."""
    path = str(tmp_path / "logits.pt")
    mp.spawn(_worker, args=(world, _free_port(), kind, path), nprocs=world, join=True)
    got = torch.load(path)
    model = _tiny(kind)
    ids = torch.randint(0, 300, (2, 40), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model(ids).logits
    assert torch.allclose(got, ref, atol=1e-5, rtol=1e-4), float((got - ref).abs().max())
