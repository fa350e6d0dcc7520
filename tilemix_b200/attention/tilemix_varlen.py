"""Batched-head entry point used by the model attention layers (drop-in for the
reference's ``attention/tilemix_varlen.py:17-96``).

``tilemix_varlen_attention`` takes ``[B, H, T, D]`` tensors, packs them
token-major (a no-op when they are permuted views of token-major data, as the
Llama/Qwen prefill produces), builds equal-length ``cu_seqlens`` and runs the
routed attention with the reference's fixed settings (``BLKQ=128``,
``BLKK=64``, ``scalar_scales = block_m == 128 and block_n == 64``, routing
mode from ``TILEMIX_BITMASK_ROUTING_MODE``, FP16 V from
``TILEMIX_SCORE_ONLY_PV``). Because every sequence has length T, the K scale
offsets are computed without a device-to-host read, so the call never
synchronises the host. ``tilemix_varlen_attention_from_host`` is the same attention
for packed inputs and output in pinned host memory, streamed through the GPU so
that the host-device copies of one chunk of sequences overlap the attention of
another.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
from torch import Tensor

from tilemix_b200.attention.tilemix import _attention_forward, _routing_mode_code, _validate


def _env_flag(name: str, default: str = "0") -> bool:
    return (os.getenv(name) or default).strip().lower() not in ("0", "false", "no", "")


def tilemix_varlen_attention(q: Tensor, k: Tensor, v: Tensor, block_m: int, block_n: int, *,
                             block_n_mask: Optional[int] = None, causal: bool, scale: float,
                             precision_map_all: Tensor, candidates: list[tuple[int, int]],
                             flat_lengths: list[int], bias: Optional[Tensor] = None,
                             k_quant: Optional[tuple[Tensor, Tensor]] = None) -> Tensor:
    """Routed FP16/INT8 attention of ``[B, H, T, D]`` q/k/v; returns ``[B, Hq, T, D]``.

    ``candidates`` and ``flat_lengths`` are accepted for signature parity and
    unused, as in the reference. ``k_quant`` (no counterpart in the reference):
    K already quantised per 64-token block, as ``(k8 [B*T, Hk, D] int8,
    scales [B*ceil(T/64), Hk] fp16)`` from the fused RoPE pass
    (``rotary_token_major_quant_k``), so K is not read again to quantise it.
    """
    B, Hq, Tq, D = q.shape
    _, Hk, Tk, Dk = k.shape
    _, Hv, Tv, Dv = v.shape
    assert Dk == D
    assert Dv == D
    assert Hk == Hv, "K and V must have the same number of heads (GQA support)"

    Q = q.permute(0, 2, 1, 3).reshape(B * Tq, Hq, D).contiguous()
    K = k.permute(0, 2, 1, 3).reshape(B * Tk, Hk, D).contiguous()
    V = v.permute(0, 2, 1, 3).reshape(B * Tk, Hv, D).contiguous()
    device = Q.device
    cu_q = torch.arange(0, (B + 1) * Tq, Tq, device=device, dtype=torch.int32)
    cu_k = torch.arange(0, (B + 1) * Tk, Tk, device=device, dtype=torch.int32)

    pm = precision_map_all
    assert pm.dtype == torch.uint64, f"precision_map dtype must be uint64, got {pm.dtype}"
    if block_n_mask is None:
        block_n_mask = block_n
    if block_n_mask % block_n != 0:
        raise ValueError(f"block_n_mask ({block_n_mask}) must be a multiple of block_n ({block_n})")
    if Tq != Tk:
        raise ValueError(f"Tq ({Tq}) != Tk ({Tk}). Bitmask was created assuming they're equal. "
                         f"This will cause incorrect indexing in the kernel.")
    m_blocks_total = (Tq + block_m - 1) // block_m
    n_mask_blocks_total = (Tk + block_n_mask - 1) // block_n_mask
    if n_mask_blocks_total > 64:
        raise ValueError(f"64-bit precision mask requires n_mask_blocks<=64, got n_mask_blocks={n_mask_blocks_total} "
                         f"(Tk={Tk}, block_n_mask={block_n_mask})")
    expected_pm_elems = Hk * m_blocks_total
    assert pm.numel() == expected_pm_elems, (
        f"precision_map length mismatch: got {pm.numel()}, expected {expected_pm_elems} "
        f"(Hk={Hk} KV heads × m_blocks={m_blocks_total}, n_mask_blocks={n_mask_blocks_total})")
    if bias is not None:
        bias = bias.to(device=device, dtype=q.dtype).contiguous()
        if bias.shape != (B, Hq, Tq, Tk):
            raise ValueError(f"Bias shape mismatch: got {bias.shape}, expected {(B, Hq, Tq, Tk)}")

    routing_mode = (os.getenv("TILEMIX_BITMASK_ROUTING_MODE") or "mixed").strip().lower()
    if routing_mode == "auto":
        from tilemix_b200.attention.tilemix import classify_bitmask_routing
        routing_mode = classify_bitmask_routing(pm, seqlen_q=Tq, seqlen_k=Tk, block_m=block_m, block_n=block_n,
                                                block_n_mask=block_n_mask, causal=causal)
    _routing_mode_code(routing_mode)
    scalar_scales = block_m == 128 and block_n == 64
    _validate(Q, K, V, Tq, Tk, pm, block_m, block_n, block_n_mask, 128, 64, scalar_scales)
    out = _attention_forward(Q, K, V, cu_q, cu_k, Tq, Tk, pm, block_m=block_m, block_n=block_n,
                             block_n_mask=block_n_mask, BLKQ=128, BLKK=64, causal=causal, sm_scale=scale,
                             mode=routing_mode, scalar_scales=scalar_scales,
                             int8_use_fp16_v=_env_flag("TILEMIX_SCORE_ONLY_PV", "1"), bias=bias, equal_len=Tq,
                             k_quant=k_quant)
    return out.view(B, Tq, Hq, D).permute(0, 2, 1, 3)


# The three streams of the host-resident entry point, one set per device and kept for the
# process: torch hands out a different pool stream for every new Stream(), and the caching
# allocator keeps freed blocks per stream, so fresh streams on every call would send each
# call's scratch allocations to cudaMalloc (which synchronises the device).
_HOST_STREAMS: dict = {}


def _host_streams(dev: torch.device):
    st = _HOST_STREAMS.get(dev.index)
    if st is None:
        st = _HOST_STREAMS[dev.index] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return st


@torch.no_grad()
def tilemix_varlen_attention_from_host(q: Tensor, k: Tensor, v: Tensor, out: Tensor, seq_len: int, block_m: int,
                                       block_n: int, *, block_n_mask: Optional[int] = None, causal: bool,
                                       scale: float, precision_map_all: Tensor,
                                       device: Optional[torch.device] = None, chunk_seqs: int = 1,
                                       ring: int = 2) -> Tensor:
    """``tilemix_varlen_attention`` for inputs and output in pinned host memory (no counterpart
    in the reference, whose entry points take device tensors).

    ``q`` ``[B*T, Hq, D]``, ``k`` / ``v`` ``[B*T, Hk, D]`` and ``out`` ``[B*T, Hq, D]`` are
    token-major packed fp16 CPU tensors in pinned memory, ``T = seq_len`` for every sequence.
    Sequences are streamed through the GPU ``chunk_seqs`` at a time: the copy of chunk c+1
    to the device, the attention of chunk c and the copy of chunk c-1 back to ``out`` run on
    three streams and overlap (PCIe moves both directions at once), with ``ring`` device
    buffers per tensor. Each chunk is an independent call of the same attention, so ``out``
    is bit-identical to the device call on the whole batch. Asynchronous on the current
    stream of ``device`` (default: the current CUDA device): work issued there afterwards
    (or an event recorded there) comes after the last copy back. Returns ``out``.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type != "cuda":
        raise ValueError("device must be a CUDA device")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.is_cuda or not t.is_pinned():
            raise ValueError(f"{name} must be a pinned host tensor")
        if t.dtype != torch.float16 or t.ndim != 3 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous fp16 [tokens, heads, dim] tensor")
    total, Hq, D = q.shape
    T = int(seq_len)
    if T <= 0 or total % T:
        raise ValueError("the token count must be a multiple of seq_len")
    B = total // T
    Hk = k.shape[1]
    if k.shape != (total, Hk, D) or v.shape != k.shape or out.shape != q.shape:
        raise ValueError("q / k / v / out shapes do not match")
    if chunk_seqs <= 0 or ring <= 0:
        raise ValueError("chunk_seqs and ring must be positive")
    if block_n_mask is None:
        block_n_mask = block_n
    routing_mode = (os.getenv("TILEMIX_BITMASK_ROUTING_MODE") or "mixed").strip().lower()
    if routing_mode == "auto":
        from tilemix_b200.attention.tilemix import classify_bitmask_routing
        routing_mode = classify_bitmask_routing(precision_map_all, seqlen_q=T, seqlen_k=T, block_m=block_m,
                                                block_n=block_n, block_n_mask=block_n_mask, causal=causal)
    _routing_mode_code(routing_mode)
    scalar_scales = block_m == 128 and block_n == 64
    pm = precision_map_all.to(device=dev, dtype=torch.uint64).contiguous()
    with torch.cuda.device(dev):
        main = torch.cuda.current_stream(dev)
        s_in, s_run, s_out = _host_streams(dev)
        for s in (s_in, s_run, s_out):
            s.wait_stream(main)  # the host buffers / map are ready as of the caller's stream
        cs = min(chunk_seqs, B)
        rows = cs * T
        slots = [dict(q=torch.empty((rows, Hq, D), device=dev, dtype=q.dtype),
                      k=torch.empty((rows, Hk, D), device=dev, dtype=k.dtype),
                      v=torch.empty((rows, Hk, D), device=dev, dtype=v.dtype),
                      o=torch.empty((rows, Hq, D), device=dev, dtype=q.dtype),
                      free_in=None, free_out=None) for _ in range(min(ring, (B + cs - 1) // cs))]
        fp16_v = _env_flag("TILEMIX_SCORE_ONLY_PV", "1")
        for c, b0 in enumerate(range(0, B, cs)):
            nb = min(cs, B - b0)
            r0, r1 = b0 * T, (b0 + nb) * T
            sl = slots[c % len(slots)]
            with torch.cuda.stream(s_in):
                if sl["free_in"] is not None:
                    s_in.wait_event(sl["free_in"])  # the previous chunk in this slot has been computed
                n = r1 - r0
                sl["q"][:n].copy_(q[r0:r1], non_blocking=True)
                sl["k"][:n].copy_(k[r0:r1], non_blocking=True)
                sl["v"][:n].copy_(v[r0:r1], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(s_in)
            with torch.cuda.stream(s_run):
                s_run.wait_event(ready)
                if sl["free_out"] is not None:
                    s_run.wait_event(sl["free_out"])  # the previous chunk's output has been copied out
                cu = torch.arange(0, (nb + 1) * T, T, device=dev, dtype=torch.int32)
                _attention_forward(sl["q"][:n], sl["k"][:n], sl["v"][:n], cu, cu, T, T, pm, block_m=block_m,
                                   block_n=block_n, block_n_mask=block_n_mask, BLKQ=128, BLKK=64, causal=causal,
                                   sm_scale=scale, mode=routing_mode, scalar_scales=scalar_scales,
                                   int8_use_fp16_v=fp16_v, equal_len=T, o=sl["o"][:n])
                done = torch.cuda.Event()
                done.record(s_run)
                sl["free_in"] = done
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                out[r0:r1].copy_(sl["o"][:n], non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(s_out)
                sl["free_out"] = copied
        for s in (s_in, s_run, s_out):
            main.wait_stream(s)
        # The ring buffers were allocated on the caller's stream, which now waits for all three
        # streams: their memory is reused only by work ordered after these copies.
    return out
