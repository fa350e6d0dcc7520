"""Shared machinery of the TileMix attention replacements for HF Llama / Qwen2.

Mirrors the reference's model integration (models/tilemix_llama.py:33-646,
models/tilemix_qwen.py:27-658): the same block-size policy, routing-map cache
and attention call, with the map built by the CUDA kernel
``tm_build_precision_map`` and the attention run by ``tm_attn_fwd``.
"""
from __future__ import annotations

import hashlib
import math
import os
from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor

from tilemix_b200.attention.precision_maps import BLOCK_PERCENTAGE_PATTERNS, make_precision_bitmask
from tilemix_b200.attention.tilemix_varlen import tilemix_varlen_attention


@dataclass(frozen=True)
class BucketConfig:
    block_m: int
    block_n: int


def pick_block_n_for_64(seq_len: int, choices: list[int]) -> int:
    """Smallest block_n that keeps ceil(seq_len / block_n) <= 64 (models/tilemix_llama.py:38-42)."""
    for bn in sorted(choices):
        if math.ceil(seq_len / bn) <= 64:
            return bn
    return max(choices)


def pick_mask_block_n(seqlen: int, compute_block_n: int) -> int:
    """Mask-group width: at least ceil(seqlen / 64) keys, a multiple of the compute tile
    (models/tilemix_llama.py:45-49)."""
    need = max((seqlen + 63) // 64, compute_block_n)
    return ((need + compute_block_n - 1) // compute_block_n) * compute_block_n


# Every bucket of the reference uses 64 x 64 tiles (models/tilemix_llama.py:72-79);
# sequences of 4096 tokens and more move to block_m = 128 (:163-164).
_BUCKET_EDGES = ((128, "decode"), (2048, "short"), (8192, "medium"), (16384, "long"), (32768, "xl"))
_BUCKET_SIZES = {name: BucketConfig(64, 64) for name in ("decode", "short", "medium", "long", "xl", "xxl")}
_SUPPORTED_NS = (64, 128, 256)
AVAILABLE_BLOCK_SIZES = [(64, 64), (64, 128), (64, 256), (128, 64)]


def choose_bucket(seqlen: int) -> str:
    for edge, name in _BUCKET_EDGES:
        if seqlen <= edge:
            return name
    return "xxl"


def nearest_block_size(seqlen: int, block_m: int, block_n: int) -> tuple[int, int]:
    """Closest available (block_m, block_n) by the reference's weighted distance
    (models/tilemix_llama.py:122-140)."""
    best, best_d = None, float("inf")
    for m, n in AVAILABLE_BLOCK_SIZES:
        if n > seqlen:
            continue
        dist = abs(block_m - m) * 0.5 + abs(block_n - n) * 1.5
        if dist < best_d:
            best, best_d = (m, n), dist
    if best is None:
        return min((64, 128, 256, 512), key=lambda x: abs(x - block_m)), min(_SUPPORTED_NS, key=lambda x: abs(x - block_n))
    return best


def block_config(seqlen: int) -> BucketConfig:
    """Tile sizes for a prefill of `seqlen` tokens (models/tilemix_llama.py:143-175)."""
    forced = os.getenv("TILEMIX_FORCE_CONFIG")
    if forced:
        try:
            parts = [p.strip() for p in forced.split(",")]
            return BucketConfig(*nearest_block_size(seqlen, int(parts[0]), int(parts[1])))
        except (ValueError, IndexError):
            pass
    cfg = _BUCKET_SIZES[choose_bucket(seqlen)]
    bn = min(max(cfg.block_n, 64), max(_SUPPORTED_NS))
    bm = max(cfg.block_m, 128) if seqlen >= 4096 else cfg.block_m
    return BucketConfig(*nearest_block_size(seqlen, bm, bn))


class TileMixAttentionMixin:
    """Routing-map cache and the TileMix attention call, shared by the Llama and Qwen2
    replacements. The host class provides q/k/v/o projections, ``config`` and
    ``layer_idx`` (an HF attention module)."""

    def _init_tilemix(self, config) -> None:
        nh, nkv = config.num_attention_heads, config.num_key_value_heads
        if nh % nkv != 0:
            raise ValueError(f"num_attention_heads ({nh}) must be divisible by num_key_value_heads ({nkv})")
        self.nh, self.nkv = nh, nkv
        self.register_buffer("kv_head_mapping", torch.arange(nkv, dtype=torch.long).repeat_interleave(nh // nkv))
        self.available_block_sizes = list(AVAILABLE_BLOCK_SIZES)
        self._block_to_candidate = {bs: i for i, bs in enumerate(self.available_block_sizes)}
        self.precision_map_cache: dict[tuple, Tensor] = {}
        self.decode_precision_cache: dict[tuple, Tensor] = {}
        self.default_pattern_type = "one"
        self.default_pattern_params: dict = {}

    # -- pattern configuration (models/tilemix_llama.py:202-204, 395-399)
    def set_attention_pattern(self, pattern_type: str, **pattern_params) -> None:
        self.default_pattern_type = pattern_type
        self.default_pattern_params = pattern_params
        self.precision_map_cache.clear()
        self.decode_precision_cache.clear()

    def _get_pattern_config(self, seqlen: int):
        return self.default_pattern_type, tuple(sorted(self.default_pattern_params.items()))

    def _get_block_config(self, seqlen: int) -> BucketConfig:
        return block_config(seqlen)

    @staticmethod
    def _get_pattern_hash(pattern_type: str, pattern_params: dict) -> str:
        return hashlib.md5(f"{pattern_type}_{sorted(pattern_params.items())}".encode()).hexdigest()[:8]

    # -- routing map (models/tilemix_llama.py:317-460)
    def _get_or_create_precision_map(self, seqlen: int, block_m: int, block_n: int, block_n_mask: int,
                                     pattern_type: str, pattern_params: tuple, device: torch.device) -> Tensor:
        params = dict(pattern_params)
        percentage = None if pattern_type in ("one", "causal") else params.get("percentage", None)
        key = (seqlen, block_m, block_n, block_n_mask, self._get_pattern_hash(pattern_type, params), percentage)
        cached = self.precision_map_cache.get(key)
        if cached is not None:
            if cached.device != device:
                cached = cached.to(device)
                self.precision_map_cache[key] = cached
            return cached
        if not (pattern_type in ("zero", "one") or (percentage is not None and pattern_type in BLOCK_PERCENTAGE_PATTERNS)):
            raise NotImplementedError(
                f"routing pattern {pattern_type!r} without an INT8 percentage needs a token-mask map, which the GPU "
                "map builder does not construct; configure one of zero/one or a percentage-aware block pattern")
        words = make_precision_bitmask(seq_len=seqlen, BLOCK_M=block_m, BLOCK_N=block_n_mask, token_mask=None,
                                       percentage=percentage, pattern_type=pattern_type, pattern_params=params,
                                       COMPUTE_BLOCK_N=block_n, device=device)
        expected = (seqlen + block_m - 1) // block_m
        if words.numel() != expected:
            raise ValueError(f"Precision bitmask length mismatch: got {words.numel()}, expected {expected}")
        self.precision_map_cache[key] = words
        return words

    def _prepare_precision_map(self, seqlen: int, bucket: BucketConfig, block_n_mask: int, pattern_type: str,
                               pattern_params: tuple, device: torch.device) -> Tensor:
        m_blocks = (seqlen + bucket.block_m - 1) // bucket.block_m
        n_mask_blocks = (seqlen + block_n_mask - 1) // block_n_mask
        if n_mask_blocks > 64:
            raise ValueError(f"64-bit precision mask requires n_mask_blocks<=64, got n_mask_blocks={n_mask_blocks} "
                             f"(seqlen={seqlen}, block_n_mask={block_n_mask})")
        row = self._get_or_create_precision_map(seqlen, bucket.block_m, bucket.block_n, block_n_mask,
                                                pattern_type, pattern_params, device)
        if row.numel() != m_blocks:
            raise ValueError(f"Precision bitmask length {row.numel()} != expected {m_blocks}")
        key = (device, bucket, block_n_mask, self.nkv, seqlen, self._get_pattern_hash(pattern_type, dict(pattern_params)))
        flat = self.decode_precision_cache.get(key)
        if flat is None:
            flat = row.view(torch.int64).repeat(self.nkv).view(torch.uint64)
            self.decode_precision_cache[key] = flat
        return flat

    def _fixup_precision_map(self, precision_map: Tensor, seqlen: int, block_n_mask: int) -> Tensor:
        return precision_map

    # -- the attention call (models/tilemix_llama.py:505-646)
    def _tilemix_attention(self, q: Tensor, k: Tensor, v: Tensor, seqlen: int, k_quant=None) -> Tensor:
        """q [B, nh, T, D], k/v [B, nkv, T, D] -> attention output [B, nh, T, D]. ``k_quant``:
        K codes and block scales made with the RoPE (see tilemix_varlen_attention)."""
        head_dim = q.shape[-1]
        bucket = self._get_block_config(seqlen)
        block_n_mask = pick_mask_block_n(seqlen, bucket.block_n)
        pattern_type, pattern_params = self._get_pattern_config(seqlen)
        if (bucket.block_m, bucket.block_n) not in self._block_to_candidate:
            raise ValueError(f"Block size {(bucket.block_m, bucket.block_n)} is not in available_block_sizes "
                             f"{self.available_block_sizes}")
        pm = self._prepare_precision_map(seqlen, bucket, block_n_mask, pattern_type, pattern_params, q.device)
        pm = self._fixup_precision_map(pm, seqlen, block_n_mask)
        if not all(t.is_cuda for t in (q, k, v, pm)):
            raise RuntimeError(f"All tensors must be on CUDA: q={q.device}, k={k.device}, v={v.device}, "
                               f"precision_map={pm.device}")
        return tilemix_varlen_attention(q, k, v, bucket.block_m, bucket.block_n, block_n_mask=block_n_mask,
                                        causal=True, scale=head_dim ** -0.5, precision_map_all=pm,
                                        candidates=[(bucket.block_m, bucket.block_n)], flat_lengths=[pm.numel()],
                                        k_quant=k_quant)


def copy_attention_weights(orig, new) -> None:
    """Copy every parameter / buffer of the original attention module that the replacement has."""
    new_state = new.state_dict()
    with torch.no_grad():
        for name, value in orig.state_dict().items():
            if name in new_state and new_state[name].shape == value.shape:
                new_state[name].copy_(value)


def replace_attention(model, make_attention) -> None:
    root = model.model if hasattr(model, "model") else model
    for layer in root.layers:
        orig = layer.self_attn
        new_attn = make_attention(orig.config, orig.layer_idx)
        first = next(orig.parameters())
        new_attn = new_attn.to(device=first.device, dtype=first.dtype)
        copy_attention_weights(orig, new_attn)
        layer.self_attn = new_attn
    model.use_tilemix = True


def configure_pattern(model, attention_cls, pattern_type: str, pattern_params: dict):
    root = model.model if hasattr(model, "model") else model
    for layer in root.layers:
        if isinstance(layer.self_attn, attention_cls):
            layer.self_attn.set_attention_pattern(pattern_type, **pattern_params)
    return model


def prefill_past(past_key_value, kwargs) -> Optional[object]:
    return past_key_value if past_key_value is not None else kwargs.get("past_key_values")
