"""Head-sharded tensor parallelism for the Llama / Qwen2 prefill (Megatron layout).

One process per GPU. Every decoder layer is split across the ranks of a process
group: the Q/K/V projections by attention head and the gate/up projections by
intermediate column (column-parallel, no communication), the output and down
projections by input column (row-parallel), whose partial products are summed
with one NCCL all-reduce each. Embeddings, norms and the LM head stay
replicated, so every rank ends with the full logits. The TileMix attention of a
rank runs on its own heads with the unchanged kernel: the routing map is the
same for every head, and the GQA grouping of the local heads is whatever the
split leaves (possibly uneven across ranks).

Head split (``head_split``):
  * the world size divides the KV heads: each rank owns world-size-th of the KV
    heads and all Q heads of their groups (Llama-3.2-3B, 24 / 8 heads, at
    TP 2 / 4 / 8);
  * the KV heads divide the world size: each KV head is replicated on
    world / kv ranks, and its group's Q heads are split across them as evenly as
    possible, the first ranks taking one more (Qwen2-7B, 28 / 4 heads, at TP 8:
    4 + 3 Q heads per KV head).
Any other combination raises ValueError.

No counterpart in the reference, which runs the model on one GPU; this serves
the multi-GPU prefill configurations of the headline benchmark.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor, nn

__all__ = ["HeadSplit", "head_split", "column_split", "RowParallelLinear", "shard_model_for_tensor_parallel"]


@dataclass(frozen=True)
class HeadSplit:
    q_lo: int
    q_hi: int
    kv_lo: int
    kv_hi: int

    @property
    def num_q(self) -> int:
        return self.q_hi - self.q_lo

    @property
    def num_kv(self) -> int:
        return self.kv_hi - self.kv_lo


def head_split(num_heads: int, num_kv_heads: int, rank: int, world: int) -> HeadSplit:
    """The contiguous Q and KV head ranges of ``rank`` (see the module docstring)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if num_kv_heads <= 0 or num_heads % num_kv_heads:
        raise ValueError(f"{num_heads} query heads do not form groups over {num_kv_heads} KV heads")
    group = num_heads // num_kv_heads
    if num_kv_heads % world == 0:
        per = num_kv_heads // world
        kv_lo = rank * per
        return HeadSplit(kv_lo * group, (kv_lo + per) * group, kv_lo, kv_lo + per)
    if world % num_kv_heads == 0:
        reps = world // num_kv_heads
        if reps > group:
            raise ValueError(f"{world} ranks leave some of the {num_kv_heads} KV heads' ranks without a query head")
        kv = rank // reps
        j = rank % reps
        base, extra = divmod(group, reps)
        lo = j * base + min(j, extra)
        hi = lo + base + (1 if j < extra else 0)
        return HeadSplit(kv * group + lo, kv * group + hi, kv, kv + 1)
    raise ValueError(f"{num_kv_heads} KV heads cannot be split over {world} ranks")


def column_split(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous near-equal split of ``n`` columns: the first ``n % world`` ranks take one more."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class RowParallelLinear(nn.Module):
    """``y = all_reduce(x_shard @ W_shard^T) + b``: a linear layer whose input columns are split
    across the process group. The bias, if any, is added once after the sum."""

    def __init__(self, linear: nn.Linear, lo: int, hi: int, group=None):
        super().__init__()
        self.group = group
        self.in_features = hi - lo
        self.out_features = linear.out_features
        self.weight = nn.Parameter(linear.weight.detach()[:, lo:hi].contiguous(), requires_grad=False)
        self.bias = None if linear.bias is None else nn.Parameter(linear.bias.detach().clone(), requires_grad=False)

    def forward(self, x: Tensor) -> Tensor:
        y = torch.nn.functional.linear(x, self.weight)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias
        return y


def _slice_rows(linear: nn.Linear, lo: int, hi: int) -> None:
    """Keep output rows [lo, hi) of a column-parallel linear layer, in place."""
    linear.weight = nn.Parameter(linear.weight.detach()[lo:hi].contiguous(), requires_grad=False)
    if linear.bias is not None:
        linear.bias = nn.Parameter(linear.bias.detach()[lo:hi].contiguous(), requires_grad=False)
    linear.out_features = hi - lo


def shard_model_for_tensor_parallel(model, rank: Optional[int] = None, world_size: Optional[int] = None,
                                    group=None):
    """Split every decoder layer of an HF Llama / Qwen2 causal LM (plain, TileMix-injected or
    prepared for prefill) across the ranks of ``group`` (default: the world), in place.

    Call it on every rank with identical weights (same seed or checkpoint); afterwards the
    model's forward must run on all ranks together. Returns the model."""
    if world_size is None:
        world_size = dist.get_world_size(group) if dist.is_initialized() else 1
    if rank is None:
        rank = dist.get_rank(group) if dist.is_initialized() else 0
    cfg = model.config
    nh, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // nh
    hs = head_split(nh, nkv, rank, world_size)
    root = model.model if hasattr(model, "model") else model
    for layer in root.layers:
        attn = layer.self_attn
        _slice_rows(attn.q_proj, hs.q_lo * hd, hs.q_hi * hd)
        _slice_rows(attn.k_proj, hs.kv_lo * hd, hs.kv_hi * hd)
        _slice_rows(attn.v_proj, hs.kv_lo * hd, hs.kv_hi * hd)
        attn.o_proj = RowParallelLinear(attn.o_proj, hs.q_lo * hd, hs.q_hi * hd, group)
        attn.head_dim = hd
        attn.num_key_value_groups = hs.num_q // hs.num_kv
        if hasattr(attn, "nh"):  # TileMix attention: local head counts drive the map and the kernel
            attn.nh, attn.nkv = hs.num_q, hs.num_kv
            attn.kv_head_mapping = torch.arange(hs.num_kv, dtype=torch.long,
                                                device=attn.kv_head_mapping.device).repeat_interleave(
                                                    hs.num_q // hs.num_kv)
            attn.decode_precision_cache.clear()
        mlp = layer.mlp
        lo, hi = column_split(mlp.gate_proj.out_features, rank, world_size)
        _slice_rows(mlp.gate_proj, lo, hi)
        _slice_rows(mlp.up_proj, lo, hi)
        mlp.down_proj = RowParallelLinear(mlp.down_proj, lo, hi, group)
    model.tensor_parallel = (rank, world_size)
    return model
