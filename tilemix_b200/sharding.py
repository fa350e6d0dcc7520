"""Sharding of the attention work over ranks: independent (sequence x KV-head)
units, no data-path collective.

A unit is one sequence of the packed batch and one KV head with its group of
Q heads; its causal cost is group * T (T + 1) / 2 query-key pairs. Units are
assigned to ranks longest-processing-time first (each unit to the currently
least-loaded rank), which balances varlen batches of very different lengths.
A rank packs its units into varlen problems with a single KV head (each unit
becomes one "sequence"); its outputs are scattered back into the full
[tokens, HQ, D] layout.

The kernels read a sequence's routing word for query block m of KV head h at
h * m_blocks + m, with m_blocks counted from that sequence's own length
(attention/triton/tilemix.py:819-823); a shard groups its units by that
offset and passes each group the words it reads, so sharded and unsharded
results are identical.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch


def kv_head_block(heads_k: int, world_size: int, rank: int) -> Optional[tuple[int, int]]:
    """The contiguous KV heads [h0, h1) of ``rank`` when the world size divides the KV heads:
    the rank then owns the units (every sequence) x [h0, h1), an equal share of any batch,
    and its inputs and outputs are strided views of the full packed tensors (no packing, no
    scatter). None when the world size does not divide the KV heads (use ``plan_units``)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    if heads_k % world_size:
        return None
    per = heads_k // world_size
    return rank * per, (rank + 1) * per


def head_block_views(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                     precision_map: torch.Tensor, m_blocks: int, block: tuple[int, int]):
    """Views of one KV-head block [h0, h1) of packed [tokens, heads, D] q / k / v / out and
    its routing words (rows h * m_blocks + [0, m_blocks) for h in the block, contiguous).

    Exact for batches of equal sequence length m_blocks * block_m >= T > (m_blocks - 1) *
    block_m: the kernels index the words of KV head h with the sequence's own block count
    (attention/triton/tilemix.py:819-823), which is then m_blocks for every sequence. Varlen
    batches shard with ``plan_units`` / ``sharded_attention``, which group units by the words
    they read."""
    h0, h1 = block
    g = q.shape[1] // k.shape[1]
    return (q[:, h0 * g:h1 * g], k[:, h0:h1], v[:, h0:h1], out[:, h0 * g:h1 * g],
            precision_map[h0 * m_blocks:h1 * m_blocks])


def unit_cost(length: int, group: int, causal: bool = True) -> int:
    return group * (length * (length + 1) // 2 if causal else length * length)


def plan_units(lengths: Sequence[int], heads_k: int, world_size: int, group: int = 1,
               causal: bool = True) -> list[list[tuple[int, int]]]:
    """Per rank, the (sequence, KV head) units it computes (LPT assignment; ties go to
    the lower rank, units of equal cost keep sequence-major order)."""
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    units = [(b, h) for b in range(len(lengths)) for h in range(heads_k)]
    units.sort(key=lambda u: -unit_cost(int(lengths[u[0]]), group, causal))
    load = [0] * world_size
    plan: list[list[tuple[int, int]]] = [[] for _ in range(world_size)]
    for u in units:
        r = min(range(world_size), key=lambda i: (load[i], i))
        plan[r].append(u)
        load[r] += unit_cost(int(lengths[u[0]]), group, causal)
    for p in plan:
        p.sort()
    return plan


def pack_units(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: Sequence[int],
               units: Sequence[tuple[int, int]]):
    """Gather a rank's units into one varlen problem with one KV head.

    Returns (q_r [n, group, D], k_r [n, 1, D], v_r [n, 1, D], cu_r int32 [U+1], max_len)."""
    group = q.shape[1] // k.shape[1]
    qs, ks, vs, cu, mx = [], [], [], [0], 0
    for b, h in units:
        s, e = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        qs.append(q[s:e, h * group:(h + 1) * group])
        ks.append(k[s:e, h:h + 1])
        vs.append(v[s:e, h:h + 1])
        cu.append(cu[-1] + e - s)
        mx = max(mx, e - s)
    dev = q.device
    if not units:
        empty = q.new_empty((0, group, q.shape[2]))
        return empty, k.new_empty((0, 1, k.shape[2])), v.new_empty((0, 1, v.shape[2])), \
            torch.zeros(1, dtype=torch.int32, device=dev), 0
    return (torch.cat(qs).contiguous(), torch.cat(ks).contiguous(), torch.cat(vs).contiguous(),
            torch.tensor(cu, dtype=torch.int32, device=dev), mx)


def unpack_units(out_r: torch.Tensor, cu_seqlens: Sequence[int], units: Sequence[tuple[int, int]],
                 out: torch.Tensor) -> torch.Tensor:
    """Scatter a shard's [n, group, D] outputs into the full [tokens, HQ, D] tensor."""
    group = out_r.shape[1]
    pos = 0
    for b, h in units:
        s, e = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        out[s:e, h * group:(h + 1) * group] = out_r[pos:pos + e - s]
        pos += e - s
    return out


def map_rows(precision_map: torch.Tensor, unit: tuple[int, int], length: int, block_m: int) -> tuple[int, int]:
    """(offset, count) of the routing words unit (sequence, KV head h) reads in the full
    problem: rows h * m_blocks + [0, m_blocks) with m_blocks = ceil(length / block_m) of
    that sequence (attention/triton/tilemix.py:819-823 indexes with the sequence's own
    length)."""
    m_blocks = (length + block_m - 1) // block_m
    return unit[1] * m_blocks, m_blocks


def sharded_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: Sequence[int],
                      precision_map: torch.Tensor, block_m: int, attn_fn: Callable, *, rank: int,
                      world_size: int, gather: bool = True, process_group: Optional[object] = None) -> torch.Tensor:
    """Compute this rank's units and (optionally) assemble the full output on every rank.

    ``attn_fn(q_r, k_r, v_r, cu_r, max_len, rows)`` runs one packed problem with one KV
    head whose every sequence reads routing words ``rows``. Units are launched in groups
    that read the same words of ``precision_map`` in the full problem (one group for the
    model's equal-length batches), so the result equals the unsharded call's. The assembly
    is a sum all-reduce of disjoint outputs (exact)."""
    lengths = [int(cu_seqlens[i + 1]) - int(cu_seqlens[i]) for i in range(len(cu_seqlens) - 1)]
    group = q.shape[1] // k.shape[1]
    units = plan_units(lengths, k.shape[1], world_size, group)[rank]
    by_rows: dict[int, list[tuple[int, int]]] = {}
    for u in units:
        off, _ = map_rows(precision_map, u, lengths[u[0]], block_m)
        by_rows.setdefault(off, []).append(u)
    out = torch.zeros_like(q)
    for off, us in sorted(by_rows.items()):
        q_r, k_r, v_r, cu_r, mx = pack_units(q, k, v, cu_seqlens, us)
        rows = precision_map[off:off + (mx + block_m - 1) // block_m]
        out_r = attn_fn(q_r, k_r, v_r, cu_r, mx, rows)
        unpack_units(out_r, cu_seqlens, us, out)
    if gather and world_size > 1:
        import torch.distributed as dist

        if dist.get_backend(process_group) == "gloo" and out.dtype in (torch.float16, torch.bfloat16):
            acc = out.float()
            dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=process_group)
            out.copy_(acc)
        else:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=process_group)
    return out
