"""TileMix attention for HF Qwen2 models (drop-in for the reference's
``models/tilemix_qwen.py``).

Public API, same names and behaviour as the reference:
  TileMixqwenAttention                models/tilemix_qwen.py:46-658
  inject_tilemix_into_qwen(model)     :661-693
  configure_tilemix_attention_pattern :696-708
Same block policy and routing-map cache as the Llama replacement, plus the
reference's Qwen map fix-up before the attention call (:626-636): bits beyond
the mask groups are cleared, and a map whose every row holds only its highest
group is widened to all groups.
"""
from __future__ import annotations

import torch
from torch import Tensor
from transformers.models.qwen2.modeling_qwen2 import Qwen2Attention, apply_rotary_pos_emb

from tilemix_b200.models._attention_base import (
    BucketConfig,
    TileMixAttentionMixin,
    configure_pattern,
    pick_block_n_for_64,
    pick_mask_block_n,
    prefill_past,
    replace_attention,
)

__all__ = ["BucketConfig", "TileMixqwenAttention", "TileMixQwenAttention", "inject_tilemix_into_qwen",
           "configure_tilemix_attention_pattern", "pick_block_n_for_64", "pick_mask_block_n"]


class TileMixqwenAttention(TileMixAttentionMixin, Qwen2Attention):
    def __init__(self, config, layer_idx: int):
        super().__init__(config, layer_idx=layer_idx)
        self._init_tilemix(config)

    def _fixup_precision_map(self, precision_map: Tensor, seqlen: int, block_n_mask: int) -> Tensor:
        num_n = (seqlen + block_n_mask - 1) // block_n_mask
        words = precision_map.view(torch.int64)
        valid = -1 if num_n >= 64 else (1 << num_n) - 1
        highest = -(1 << 63) if num_n == 64 else 1 << (num_n - 1)
        masked = words & valid
        if bool(torch.all(masked == highest)):
            masked = torch.full_like(words, valid)
        return masked.view(torch.uint64)

    def forward(self, hidden_states: Tensor, position_embeddings=None, attention_mask=None, past_key_values=None,
                cache_position=None, **kwargs):
        past_kv = prefill_past(past_key_values, kwargs)
        kwargs.pop("past_key_value", None)
        if not hidden_states.is_cuda:
            hidden_states = hidden_states.cuda()
        bsz, seqlen, _ = hidden_states.shape
        if seqlen < 16:
            return Qwen2Attention.forward(self, hidden_states, position_embeddings, attention_mask,
                                          past_key_values=past_kv, cache_position=cache_position, **kwargs)
        head_dim = self.head_dim
        dev = hidden_states.device
        q = self.q_proj(hidden_states).view(bsz, seqlen, self.nh, head_dim).transpose(1, 2)
        k = self.k_proj(hidden_states).view(bsz, seqlen, self.nkv, head_dim).transpose(1, 2)
        v = self.v_proj(hidden_states).view(bsz, seqlen, self.nkv, head_dim).transpose(1, 2)
        if position_embeddings is None:
            position_embeddings = self.rotary_emb(q, kwargs.get("position_ids", None))
        cos, sin = (t.to(dev) for t in position_embeddings)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        if past_kv is not None:
            k, v = past_kv.update(k, v, self.layer_idx,
                                  cache_kwargs={"sin": sin, "cos": cos, "cache_position": cache_position})
        out = self._tilemix_attention(q.contiguous(), k.to(q.dtype).contiguous(), v.to(q.dtype).contiguous(),
                                      seqlen)
        return self.o_proj(out.transpose(1, 2).reshape(bsz, seqlen, -1)), None


TileMixQwenAttention = TileMixqwenAttention


def inject_tilemix_into_qwen(model):
    """Replace every decoder layer's self-attention with TileMixqwenAttention (weights copied)."""
    replace_attention(model, TileMixqwenAttention)
    return model


def configure_tilemix_attention_pattern(model, pattern_type: str = "one", **pattern_params):
    """Set the routing pattern (and its INT8 percentage) of every TileMix attention layer."""
    return configure_pattern(model, TileMixqwenAttention, pattern_type, pattern_params)
