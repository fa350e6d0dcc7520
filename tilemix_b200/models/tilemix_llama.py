"""TileMix attention for HF Llama models (drop-in for the reference's
``models/tilemix_llama.py``).

Public API, same names and behaviour as the reference:
  TileMixLlamaAttention               models/tilemix_llama.py:52-646
  inject_tilemix_into_llama(model)    :657-688
  configure_tilemix_attention_pattern :691-700
  PrefillCache                        :703-715
  prepare_llama_prefill(model)        :883-895
Prefill sequences of 16 tokens or more run the routed FP16/INT8 attention through
``tilemix_varlen_attention`` (the sm_100a kernels); shorter ones (decode) use HF's
own attention, as in the reference.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor, nn
from transformers.cache_utils import Cache, DynamicLayer
from transformers.models.llama.modeling_llama import LlamaAttention, apply_rotary_pos_emb

from tilemix_b200.models._attention_base import (
    BucketConfig,
    TileMixAttentionMixin,
    configure_pattern,
    pick_block_n_for_64,
    pick_mask_block_n,
    prefill_past,
    replace_attention,
)

__all__ = [
    "BucketConfig", "TileMixLlamaAttention", "inject_tilemix_into_llama", "configure_tilemix_attention_pattern",
    "PrefillCache", "prepare_llama_prefill", "rotary_token_major", "silu_mul", "pick_block_n_for_64",
    "pick_mask_block_n",
]


class TileMixLlamaAttention(TileMixAttentionMixin, LlamaAttention):
    apply_rotary = staticmethod(apply_rotary_pos_emb)

    def __init__(self, config, layer_idx: int):
        super().__init__(config, layer_idx=layer_idx)
        self._init_tilemix(config)

    def forward(self, hidden_states: Tensor, attention_mask=None, position_ids=None, past_key_value=None,
                output_attentions: bool = False, use_cache: bool = False, cache_position=None,
                position_embeddings: Optional[Tuple[Tensor, Tensor]] = None, **kwargs):
        past_kv = prefill_past(past_key_value, kwargs)
        kwargs.pop("past_key_values", None)
        if not hidden_states.is_cuda:
            hidden_states = hidden_states.cuda()
        bsz, seqlen, _ = hidden_states.shape
        if seqlen < 16:  # decode: HF attention (models/tilemix_llama.py:526-536)
            return LlamaAttention.forward(self, hidden_states, position_embeddings=position_embeddings,
                                          attention_mask=attention_mask, past_key_values=past_kv,
                                          cache_position=cache_position, **kwargs)
        head_dim = self.config.hidden_size // self.nh
        dev = hidden_states.device
        q = self.q_proj(hidden_states).view(bsz, seqlen, self.nh, head_dim).transpose(1, 2)
        k = self.k_proj(hidden_states).view(bsz, seqlen, self.nkv, head_dim).transpose(1, 2)
        v = self.v_proj(hidden_states).view(bsz, seqlen, self.nkv, head_dim).transpose(1, 2)
        if position_embeddings is None:
            position_embeddings = self.rotary_emb(q, position_ids)
        cos, sin = (t.to(dev) for t in position_embeddings)
        q, k = self.apply_rotary(q, k, cos, sin)
        if past_kv is not None:
            k, v = past_kv.update(k, v, self.layer_idx,
                                  cache_kwargs={"sin": sin, "cos": cos, "cache_position": cache_position})
        out = self._tilemix_attention(q, k.to(q.dtype), v.to(q.dtype), seqlen)
        return self.o_proj(out.transpose(1, 2).reshape(bsz, seqlen, -1)), None


def inject_tilemix_into_llama(model):
    """Replace every decoder layer's self-attention with TileMixLlamaAttention (weights copied)."""
    replace_attention(model, TileMixLlamaAttention)
    return model


def configure_tilemix_attention_pattern(model, pattern_type: str = "one", **pattern_params):
    """Set the routing pattern (and its INT8 percentage) of every TileMix attention layer."""
    return configure_pattern(model, TileMixLlamaAttention, pattern_type, pattern_params)


class _PrefillDynamicLayer(DynamicLayer):
    """Stores the first update's tensors as they are (no concatenation copy)."""

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.dtype, self.device = key_states.dtype, key_states.device
            self.keys, self.values = key_states, value_states
            self.is_initialized = True
            return self.keys, self.values
        return super().update(key_states, value_states, *args, **kwargs)


class PrefillCache(Cache):
    def __init__(self):
        super().__init__(layer_class_to_replicate=_PrefillDynamicLayer)


def rotary_token_major(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor):
    """Split-half RoPE that writes token-major outputs ([B, T, H, D] storage, returned as
    [B, H, T, D] views) so the attention's packing is a no-op. Rounds like the reference's
    prefill rotary (models/tilemix_llama.py:797-822): fp16(x*cos) + fp16(rot(x)*sin) in fp32."""
    b, hq, t, d = q.shape
    hk = k.shape[1]
    if q.dtype != torch.float16 or any(x.dtype != q.dtype for x in (k, cos, sin)):
        raise ValueError("prefill rotary requires FP16 operands")
    if d % 2 or k.shape != (b, hk, t, d) or cos.shape[-2:] != (t, d) or sin.shape != cos.shape:
        raise ValueError("incompatible split-half rotary shapes")
    if cos.shape[0] not in (1, b):
        raise ValueError("rotary batch must be one or match the input")
    c = cos.float()[:, None]
    s = sin.float()[:, None]
    sign = torch.cat([-torch.ones(d // 2, device=q.device), torch.ones(d // 2, device=q.device)])

    def rot(x):
        xr = torch.cat([x[..., d // 2:], x[..., :d // 2]], dim=-1).float()
        a = (x.float() * c).half().float()
        bpart = (xr * sign * s).half().float()
        return (a + bpart).half().transpose(1, 2).contiguous().transpose(1, 2)

    return rot(q), rot(k)


def silu_mul(gate: Tensor, up: Tensor) -> Tensor:
    """fp16(silu(gate)) * up in fp32, rounded to fp16 (models/tilemix_llama.py:825-848)."""
    if gate.dtype != torch.float16 or up.dtype != gate.dtype or gate.shape != up.shape:
        raise ValueError("SiLU requires equally shaped FP16 operands")
    if not gate.is_contiguous() or not up.is_contiguous():
        raise ValueError("SiLU requires contiguous operands")
    g = gate.float()
    act = (g / (1.0 + torch.exp(-g))).half()
    return (act.float() * up.float()).half()


class PrefillMLP(nn.Module):
    def __init__(self, original):
        super().__init__()
        self.gate_proj = original.gate_proj
        self.up_proj = original.up_proj
        self.down_proj = original.down_proj
        self.train(original.training)

    def forward(self, x):
        return self.down_proj(silu_mul(self.gate_proj(x), self.up_proj(x)))


def prepare_llama_prefill(model):
    """Switch an injected, eval-mode FP16 SiLU Llama to the prefill path: token-major RoPE
    and the fused SiLU-multiply MLP (models/tilemix_llama.py:883-895). RMSNorm stays HF's."""
    if model.training or model.config.hidden_act != "silu":
        raise ValueError("prefill requires an eval-mode SiLU LLaMA")
    for layer in model.model.layers:
        if not isinstance(layer.self_attn, TileMixLlamaAttention):
            raise ValueError("inject TileMix attention before preparing prefill")
        if layer.mlp.gate_proj.weight.dtype != torch.float16:
            raise ValueError("prefill requires FP16 model weights")
    for layer in model.model.layers:
        layer.self_attn.apply_rotary = rotary_token_major
        layer.mlp = PrefillMLP(layer.mlp)
    return model
