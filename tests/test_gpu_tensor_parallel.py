"""GPU test of the head-sharded tensor parallelism on 2 GPUs (skipped with fewer): a small
TileMix Llama prepared for prefill, sharded across two NCCL ranks, must give the last-position
logits of the same model on one GPU (the routed attention runs per rank on its own heads;
only the all-reduce summation order differs)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _model(dev):
    from transformers import LlamaConfig, LlamaForCausalLM

    from tilemix_b200.models.tilemix_llama import (configure_tilemix_attention_pattern, inject_tilemix_into_llama,
                                                   prepare_llama_prefill)

    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                      num_key_value_heads=2, vocab_size=1000, max_position_embeddings=8192, rope_theta=500000.0)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(dev, torch.float16).eval()
    inject_tilemix_into_llama(model)
    configure_tilemix_attention_pattern(model, "sptrans", percentage=0.5)
    prepare_llama_prefill(model)
    return model


def _logits(model, dev):
    from tilemix_b200.models.tilemix_llama import PrefillCache

    ids = torch.randint(0, 1000, (2, 1024), generator=torch.Generator().manual_seed(5)).to(dev)
    with torch.no_grad():
        return model(ids, past_key_values=PrefillCache(), use_cache=True, logits_to_keep=1).logits


def _worker(rank, world, port, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from tilemix_b200.attention.tilemix import device_error_code
        from tilemix_b200.models.tensor_parallel import shard_model_for_tensor_parallel

        model = shard_model_for_tensor_parallel(_model(dev))
        out = _logits(model, dev)
        torch.cuda.synchronize()
        assert device_error_code(dev) == 0
        if rank == 0:
            torch.save(out.cpu(), path)
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(600)
def test_two_gpu_tensor_parallel_prefill_matches_one_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    path = str(tmp_path / "tp.pt")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    got = torch.load(path).float()
    ref = _logits(_model(torch.device("cuda", 0)), torch.device("cuda", 0)).float().cpu()
    rel = float((got - ref).norm() / ref.norm())
    assert rel < 1e-2, rel
