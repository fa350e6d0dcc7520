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
    "PrefillCache", "prepare_llama_prefill", "prepare_llama_norms", "PrefillRMSNorm", "rotary_token_major",
    "rotary_token_major_quant_k", "silu_mul", "rms_norm", "pick_block_n_for_64", "pick_mask_block_n",
]


class TileMixLlamaAttention(TileMixAttentionMixin, LlamaAttention):
    apply_rotary = staticmethod(apply_rotary_pos_emb)
    # With the prefill RoPE: quantise K for the attention in the RoPE pass (no counterpart in
    # the reference; the codes are bit-identical to the attention's own quantiser).
    fuse_k_quant = True

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
        head_dim = self.head_dim
        dev = hidden_states.device
        q = self.q_proj(hidden_states).view(bsz, seqlen, self.nh, head_dim).transpose(1, 2)
        k = self.k_proj(hidden_states).view(bsz, seqlen, self.nkv, head_dim).transpose(1, 2)
        v = self.v_proj(hidden_states).view(bsz, seqlen, self.nkv, head_dim).transpose(1, 2)
        if position_embeddings is None:
            position_embeddings = self.rotary_emb(q, position_ids)
        cos, sin = (t.to(dev) for t in position_embeddings)
        k_quant = None
        if self.apply_rotary is rotary_token_major and self.fuse_k_quant:
            # prefill path: the RoPE pass also quantises K for the attention
            q, k, k8, ks = rotary_token_major_quant_k(q, k, cos, sin, 64)
            k_quant = (k8, ks)
        else:
            q, k = self.apply_rotary(q, k, cos, sin)
        if past_kv is not None:
            k_rot = k
            k, v = past_kv.update(k, v, self.layer_idx,
                                  cache_kwargs={"sin": sin, "cos": cos, "cache_position": cache_position})
            if k is not k_rot:  # the cache returned other keys: quantise them in the attention
                k_quant = None
        out = self._tilemix_attention(q, k.to(q.dtype), v.to(q.dtype), seqlen, k_quant=k_quant)
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


def _stream(t: Tensor):
    import ctypes

    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _rotary_args(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor):
    b, hq, t, d = q.shape
    hk = k.shape[1]
    if q.dtype != torch.float16 or any(x.dtype != q.dtype for x in (k, cos, sin)):
        raise ValueError("prefill rotary requires FP16 operands")
    if d % 2 or k.shape != (b, hk, t, d) or cos.shape[-2:] != (t, d) or sin.shape != cos.shape:
        raise ValueError("incompatible split-half rotary shapes")
    if cos.shape[0] not in (1, b):
        raise ValueError("rotary batch must be one or match the input")
    if q.stride(-1) != 1 or k.stride(-1) != 1 or cos.stride(-1) != 1 or sin.stride(-1) != 1:
        raise ValueError("rotary operands must have contiguous head dimensions")
    if not q.is_cuda:
        raise RuntimeError("the prefill rotary is a CUDA kernel")
    return b, hq, hk, t, d


def _launch_rotary(q, k, cos, sin, oq, ok, k8=None, k_scale=None, blkk=64):
    import ctypes

    from tilemix_b200._lib import check, lib, numerics_code

    b, hq, hk, t, d = _rotary_args(q, k, cos, sin)
    cb = cos.stride(0) if cos.shape[0] > 1 else 0
    sb = sin.stride(0) if sin.shape[0] > 1 else 0
    ptr = lambda x: ctypes.c_void_p(x.data_ptr() if x is not None else 0)  # noqa: E731
    with torch.cuda.device(q.device):
        rc = lib().tm_rotary_token_major(ptr(q), q.stride(0), q.stride(1), q.stride(2), ptr(k), k.stride(0),
                                         k.stride(1), k.stride(2), ptr(cos), cb, cos.stride(1), ptr(sin), sb,
                                         sin.stride(1), b, hq, hk, t, d, ptr(oq), ptr(ok), ptr(k8), ptr(k_scale),
                                         ctypes.c_void_p(0), blkk, numerics_code(), _stream(q))
    check(rc, "tm_rotary_token_major")


def rotary_token_major(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor):
    """Split-half RoPE (models/tilemix_llama.py:797-822) by the library's CUDA kernel. Writes
    token-major outputs ([B, T, H, D] storage, returned as [B, H, T, D] views) so the
    attention's packing is a no-op; rounds as the reference: fp16(x*cos) + fp16(rot(x)*sin),
    the sum formed in fp32."""
    b, hq, hk, t, d = _rotary_args(q, k, cos, sin)
    oq = torch.empty((b, t, hq, d), device=q.device, dtype=q.dtype)
    ok = torch.empty((b, t, hk, d), device=k.device, dtype=k.dtype)
    _launch_rotary(q, k, cos, sin, oq, ok)
    return oq.transpose(1, 2), ok.transpose(1, 2)


def rotary_token_major_quant_k(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor, blkk: int = 64):
    """rotary_token_major that also quantises the rotated K per block of ``blkk`` tokens for the
    attention in the same pass (no counterpart in the reference, which re-reads K in its
    quantiser). Returns (q_rot, k_rot, k8 [B*T, HK, D] int8, k_scale [B*ceil(T/blkk), HK] fp16)."""
    b, hq, hk, t, d = _rotary_args(q, k, cos, sin)
    oq = torch.empty((b, t, hq, d), device=q.device, dtype=q.dtype)
    ok = torch.empty((b, t, hk, d), device=k.device, dtype=k.dtype)
    k8 = torch.empty((b * t, hk, d), device=k.device, dtype=torch.int8)
    ks = torch.empty((b * ((t + blkk - 1) // blkk), hk), device=k.device, dtype=torch.float16)
    _launch_rotary(q, k, cos, sin, oq, ok, k8, ks, blkk)
    return oq.transpose(1, 2), ok.transpose(1, 2), k8, ks


def silu_mul(gate: Tensor, up: Tensor) -> Tensor:
    """fp16(silu(gate)) * up in fp32, rounded to fp16 (models/tilemix_llama.py:825-848), by the
    library's CUDA kernel."""
    import ctypes

    from tilemix_b200._lib import check, lib

    if gate.dtype != torch.float16 or up.dtype != gate.dtype or gate.shape != up.shape:
        raise ValueError("SiLU requires equally shaped FP16 operands")
    if not gate.is_contiguous() or not up.is_contiguous():
        raise ValueError("SiLU requires contiguous operands")
    if not gate.is_cuda:
        raise RuntimeError("the prefill SiLU is a CUDA kernel")
    out = torch.empty_like(gate)
    with torch.cuda.device(gate.device):
        rc = lib().tm_silu_mul(ctypes.c_void_p(gate.data_ptr()), ctypes.c_void_p(up.data_ptr()),
                               ctypes.c_void_p(out.data_ptr()), gate.numel(), _stream(gate))
    check(rc, "tm_silu_mul")
    return out


def rms_norm(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    """fp16(weight * fp16(x * rsqrt(mean(x^2) + eps))) over the last dim, the mean in fp32
    (PrefillRMSNorm, models/tilemix_llama.py:718-771), by the library's CUDA kernel."""
    import ctypes

    from tilemix_b200._lib import check, lib

    if x.dtype != torch.float16 or weight.dtype != torch.float16 or weight.shape != x.shape[-1:]:
        raise ValueError("the prefill RMSNorm requires FP16 rows and a matching FP16 weight")
    if not x.is_cuda:
        raise RuntimeError("the prefill RMSNorm is a CUDA kernel")
    xc = x.contiguous()
    w = weight.contiguous()
    out = torch.empty_like(xc)
    with torch.cuda.device(x.device):
        rc = lib().tm_rms_norm(ctypes.c_void_p(xc.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                               ctypes.c_void_p(out.data_ptr()), xc.numel() // x.shape[-1], x.shape[-1],
                               ctypes.c_float(eps), _stream(x))
    check(rc, "tm_rms_norm")
    return out


class PrefillRMSNorm(nn.Module):
    """RMSNorm of the prefill path (models/tilemix_llama.py:757-771) on the CUDA kernel."""

    def __init__(self, original):
        super().__init__()
        self.weight = original.weight
        self.variance_epsilon = original.variance_epsilon
        self.train(original.training)

    def forward(self, hidden_states):
        return rms_norm(hidden_states, self.weight, self.variance_epsilon)


def prepare_llama_norms(model):
    """Replace every RMSNorm of the decoder with PrefillRMSNorm (models/tilemix_llama.py:774-778)."""
    for layer in model.model.layers:
        layer.input_layernorm = PrefillRMSNorm(layer.input_layernorm)
        layer.post_attention_layernorm = PrefillRMSNorm(layer.post_attention_layernorm)
    model.model.norm = PrefillRMSNorm(model.model.norm)


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
    """Switch an injected, eval-mode FP16 SiLU Llama to the prefill path: the CUDA RMSNorm,
    token-major RoPE and the fused SiLU-multiply MLP (models/tilemix_llama.py:883-895)."""
    if model.training or model.config.hidden_act != "silu":
        raise ValueError("prefill requires an eval-mode SiLU LLaMA")
    for layer in model.model.layers:
        if not isinstance(layer.self_attn, TileMixLlamaAttention):
            raise ValueError("inject TileMix attention before preparing prefill")
        if layer.mlp.gate_proj.weight.dtype != torch.float16:
            raise ValueError("prefill requires FP16 model weights")
    prepare_llama_norms(model)
    for layer in model.model.layers:
        layer.self_attn.apply_rotary = rotary_token_major
        layer.mlp = PrefillMLP(layer.mlp)
    return model
