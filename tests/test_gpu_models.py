"""GPU tests of the model integration: a small random-init Llama / Qwen2 with
TileMix attention injected, prefilled through HF's forward. With the all-FP16
routing ("zero") the logits must track HF's own FP16 attention closely; with
mixed routing they must stay finite and close; the prefill path
(prepare_llama_prefill + PrefillCache) must give the same logits as the plain
injected model."""
import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM, Qwen2Config, Qwen2ForCausalLM

pytestmark = pytest.mark.gpu


def _llama(dev):
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=1000, max_position_embeddings=8192, rope_theta=500000.0)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(dev, torch.float16).eval()


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.mark.parametrize("T", [512, 4096])
def test_llama_prefill_tracks_hf(cuda_device, T):
    from tilemix_b200.models.tilemix_llama import configure_tilemix_attention_pattern, inject_tilemix_into_llama

    dev = cuda_device
    model = _llama(dev)
    ids = torch.randint(0, 1000, (2, T), generator=torch.Generator().manual_seed(1)).to(dev)
    with torch.no_grad():
        ref = model(ids).logits
        inject_tilemix_into_llama(model)
        configure_tilemix_attention_pattern(model, "zero")
        fp16 = model(ids).logits
        configure_tilemix_attention_pattern(model, "sptrans", percentage=0.5)
        mixed = model(ids).logits
    assert _rel(fp16, ref) < 1e-2
    assert torch.isfinite(mixed).all() and _rel(mixed, ref) < 5e-2


def test_llama_prefill_path_and_cache(cuda_device):
    from tilemix_b200.models.tilemix_llama import (PrefillCache, configure_tilemix_attention_pattern,
                                                   inject_tilemix_into_llama, prepare_llama_prefill)

    dev = cuda_device
    model = _llama(dev)
    ids = torch.randint(0, 1000, (2, 1024), generator=torch.Generator().manual_seed(2)).to(dev)
    inject_tilemix_into_llama(model)
    configure_tilemix_attention_pattern(model, "sptrans", percentage=0.5)
    with torch.no_grad():
        plain = model(ids).logits
        prepare_llama_prefill(model)
        cache = PrefillCache()
        fast = model(ids, past_key_values=cache, use_cache=True, logits_to_keep=1).logits
    assert _rel(fast[:, -1], plain[:, -1]) < 1e-2
    assert cache.get_seq_length() == 1024


def test_llama_prefill_fused_k_quantisation_is_exact(cuda_device):
    """K quantised inside the RoPE pass gives the same logits, bit for bit, as K quantised by
    the attention's own quantiser (the codes are identical)."""
    from tilemix_b200.models.tilemix_llama import (TileMixLlamaAttention, configure_tilemix_attention_pattern,
                                                   inject_tilemix_into_llama, prepare_llama_prefill)

    dev = cuda_device
    model = _llama(dev)
    ids = torch.randint(0, 1000, (2, 1024), generator=torch.Generator().manual_seed(4)).to(dev)
    inject_tilemix_into_llama(model)
    configure_tilemix_attention_pattern(model, "sptrans", percentage=0.5)
    prepare_llama_prefill(model)
    try:
        with torch.no_grad():
            TileMixLlamaAttention.fuse_k_quant = True
            fused = model(ids).logits
            TileMixLlamaAttention.fuse_k_quant = False
            separate = model(ids).logits
    finally:
        TileMixLlamaAttention.fuse_k_quant = True
    assert torch.equal(fused, separate)


def test_qwen_prefill_tracks_hf(cuda_device):
    from tilemix_b200.models.tilemix_qwen import configure_tilemix_attention_pattern, inject_tilemix_into_qwen

    dev = cuda_device
    cfg = Qwen2Config(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=1, vocab_size=1000, max_position_embeddings=8192)
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg).to(dev, torch.float16).eval()
    ids = torch.randint(0, 1000, (1, 2048), generator=torch.Generator().manual_seed(3)).to(dev)
    with torch.no_grad():
        ref = model(ids).logits
        inject_tilemix_into_qwen(model)
        configure_tilemix_attention_pattern(model, "zero")
        fp16 = model(ids).logits
        configure_tilemix_attention_pattern(model, "bigbird", percentage=0.5)
        mixed = model(ids).logits
    assert _rel(fp16, ref) < 1e-2
    assert torch.isfinite(mixed).all() and _rel(mixed, ref) < 5e-2
