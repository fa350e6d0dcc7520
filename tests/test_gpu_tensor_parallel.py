"""GPU tests of the head-sharded tensor parallelism (skipped on boxes with fewer GPUs than
ranks): a small TileMix model sharded across NCCL ranks must give the last-position logits
of the same model on one GPU (the routed attention runs per rank on its own heads; only the
all-reduce summation order differs). Llama on 2 ranks splits heads evenly; a Qwen2 layout
of 14 query / 2 KV heads on 4 ranks replicates each KV head on two ranks and splits its 7
query heads 4 + 3, the uneven split Qwen2-7B (28 / 4) takes at TP 8."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _model(dev, kind="llama"):
    if kind == "llama":
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
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from tilemix_b200.models.tilemix_qwen import configure_tilemix_attention_pattern, inject_tilemix_into_qwen

    cfg = Qwen2Config(hidden_size=896, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=14,
                      num_key_value_heads=2, vocab_size=1000, max_position_embeddings=8192)
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg).to(dev, torch.float16).eval()
    inject_tilemix_into_qwen(model)
    configure_tilemix_attention_pattern(model, "bigbird", percentage=0.5)
    return model


def _logits(model, dev):
    from tilemix_b200.models.tilemix_llama import PrefillCache

    ids = torch.randint(0, 1000, (2, 1024), generator=torch.Generator().manual_seed(5)).to(dev)
    with torch.no_grad():
        return model(ids, past_key_values=PrefillCache(), use_cache=True, logits_to_keep=1).logits


def _worker(rank, world, port, path, kind):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from tilemix_b200.attention.tilemix import device_error_code
        from tilemix_b200.models.tensor_parallel import shard_model_for_tensor_parallel

        model = shard_model_for_tensor_parallel(_model(dev, kind))
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
@pytest.mark.parametrize("kind,world", [("llama", 2), ("qwen", 4)])
def test_tensor_parallel_prefill_matches_one_gpu(tmp_path, kind, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path = str(tmp_path / "tp.pt")
    mp.spawn(_worker, args=(world, _free_port(), path, kind), nprocs=world, join=True)
    got = torch.load(path).float()
    ref = _logits(_model(torch.device("cuda", 0), kind), torch.device("cuda", 0)).float().cpu()
    rel = float((got - ref).norm() / ref.norm())
    assert rel < 1e-2, rel
