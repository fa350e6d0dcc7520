"""CPU tests of the model-integration host logic (block policy, injection,
pattern configuration, Qwen map fix-up); the forward itself needs the GPU
(tests/test_gpu_models.py)."""
import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM, Qwen2Config, Qwen2ForCausalLM

from tilemix_b200.models._attention_base import block_config, pick_mask_block_n
from tilemix_b200.models.tilemix_llama import (
    TileMixLlamaAttention,
    configure_tilemix_attention_pattern,
    inject_tilemix_into_llama,
    prepare_llama_prefill,
)
from tilemix_b200.models.tilemix_qwen import TileMixqwenAttention, inject_tilemix_into_qwen


@pytest.mark.parametrize("seqlen,expected", [(17, (64, 64)), (512, (64, 64)), (4095, (64, 64)), (4096, (128, 64)),
                                             (16384, (128, 64)), (131072, (128, 64))])
def test_block_policy(seqlen, expected):
    cfg = block_config(seqlen)
    assert (cfg.block_m, cfg.block_n) == expected


def test_block_policy_forced(monkeypatch):
    monkeypatch.setenv("TILEMIX_FORCE_CONFIG", "128,64,4,1")
    assert (block_config(1024).block_m, block_config(1024).block_n) == (128, 64)
    monkeypatch.setenv("TILEMIX_FORCE_CONFIG", "64,200")
    assert (block_config(1024).block_m, block_config(1024).block_n) == (64, 256)


@pytest.mark.parametrize("T,bn,expected", [(512, 64, 64), (4096, 64, 64), (5000, 64, 128), (16384, 64, 256),
                                           (131072, 64, 2048), (100000, 64, 1600)])
def test_mask_block_n(T, bn, expected):
    assert pick_mask_block_n(T, bn) == expected


def _tiny_llama():
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
                      num_key_value_heads=1, vocab_size=128, max_position_embeddings=4096)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def test_inject_llama_copies_weights_and_configures():
    model = _tiny_llama()
    before = [layer.self_attn.q_proj.weight.clone() for layer in model.model.layers]
    inject_tilemix_into_llama(model)
    assert model.use_tilemix
    for layer, w in zip(model.model.layers, before):
        assert isinstance(layer.self_attn, TileMixLlamaAttention)
        assert torch.equal(layer.self_attn.q_proj.weight, w)
    configure_tilemix_attention_pattern(model, "sptrans", percentage=0.5)
    attn = model.model.layers[0].self_attn
    assert attn.default_pattern_type == "sptrans" and attn.default_pattern_params == {"percentage": 0.5}
    assert attn._get_pattern_config(4096) == ("sptrans", (("percentage", 0.5),))


def test_prepare_prefill_validates():
    model = _tiny_llama()
    with pytest.raises(ValueError):
        prepare_llama_prefill(model)  # not injected
    inject_tilemix_into_llama(model)
    with pytest.raises(ValueError):
        prepare_llama_prefill(model)  # fp32 weights


def test_qwen_inject_and_map_fixup():
    cfg = Qwen2Config(hidden_size=256, intermediate_size=512, num_hidden_layers=1, num_attention_heads=2,
                      num_key_value_heads=1, vocab_size=128)
    model = Qwen2ForCausalLM(cfg).eval()
    inject_tilemix_into_qwen(model)
    attn = model.model.layers[0].self_attn
    assert isinstance(attn, TileMixqwenAttention)
    # 512 tokens in 64-key groups -> 8 groups: stray high bits are cleared
    pm = torch.tensor([0xFFF, 0x1], dtype=torch.int64).view(torch.uint64)
    got = attn._fixup_precision_map(pm, 512, 64).view(torch.int64).tolist()
    assert got == [0xFF, 0x1]
    # every row holding only its highest group widens to all groups
    pm = torch.tensor([0x80, 0x80], dtype=torch.int64).view(torch.uint64)
    assert attn._fixup_precision_map(pm, 512, 64).view(torch.int64).tolist() == [0xFF, 0xFF]
