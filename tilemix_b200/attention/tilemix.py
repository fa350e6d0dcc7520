"""Host launch layer of the B200 TileMix attention (drop-in for the reference's
``attention/triton/tilemix.py`` host functions).

Public functions keep the reference's names, arguments, validation errors and
return values:

  quantize_qkv_for_tilemix   tilemix.py:45-107
  quantize_qk_for_tilemix    tilemix.py:110-156
  classify_bitmask_routing   tilemix.py:968-1014
  launch_prequantized        tilemix.py:1132-1336
  tilemix_attention_with_quant  tilemix.py:1340-1447

Underneath, every launch goes through the C ABI ``tm_attn_fwd_ex`` of
``libtilemix_b200.so`` (hand-written tcgen05/TMA kernel for sm_100a). There is
no Triton, no autotuner and no CPU fallback. Differences in mechanism, not in
results:
  * ``tilemix_attention_with_quant`` quantises Q inside the attention kernel
    (the 128-row CTA tile is exactly one BLKQ=128 block), so only K (and V for
    the INT8-V path) goes through the standalone quantiser;
  * ``run_length`` and ``int8_cache_ca`` only changed loop structure / cache
    hints in the reference and do not change results; they are accepted and
    have no effect;
  * the online softmax is updated per 64-key tile for any ``block_n`` that is a
    multiple of 64 (the reference updates once per ``block_n`` tile); keys the
    reference visits beyond the causal limit are fully masked either way.
Environment:
  * ``TILEMIX_B200_NUMERICS`` = ``gpu`` (default) / ``exact``: which execution of
    the reference's arithmetic the results reproduce, its kernels on the GPU or
    its algorithm in exact arithmetic (``tilemix_b200._lib.numerics_mode``);
  * ``TILEMIX_B200_RESCALE_THRESHOLD`` (log2 units, default 0, at most 15): 0 is
    the reference's softmax rule (the running max moves on every increase); with
    t > 0 it moves only when a tile max exceeds it by more than t, so P stays
    below 2^t and the output accumulator is rescaled less often, at the cost of
    P's fp16 rounding differing from the reference's where the max lags.
"""
from __future__ import annotations

import ctypes
import os
from typing import Literal, Optional

import torch

from tilemix_b200._lib import TmAttnParams, TmAttnTuning, check, lib, numerics_code, numerics_mode  # noqa: F401
from tilemix_b200.attention.quant_per_block_varlen import (
    _launch_quant,
    _scale_offsets,
    per_block_int8 as quant_per_block_int8,
    per_block_int8_single,
)

ROUTING_MODE_MIXED = 0
ROUTING_MODE_FP16 = 1
ROUTING_MODE_INT8 = 2
RoutingMode = Literal["auto", "mixed", "fp16", "int8"]

_ERROR_WORDS: dict[int, torch.Tensor] = {}


def _error_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _ERROR_WORDS.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERROR_WORDS[idx] = w
    return w


def device_error_code(device: Optional[torch.device] = None, reset: bool = True) -> int:
    """Read (and optionally clear) the device error word of the attention kernel.

    Non-zero means a bounded wait inside the kernel timed out (codes in
    csrc/common.cuh). Synchronises the device.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    w = _error_word(device)
    code = int(w.item())
    if reset and code:
        w.zero_()
    return code


def rescale_threshold() -> float:
    """Softmax rescale threshold (``TILEMIX_B200_RESCALE_THRESHOLD``, default 0: the reference's rule)."""
    return float(os.environ.get("TILEMIX_B200_RESCALE_THRESHOLD", "0"))


def _scale_dtype(dtype: torch.dtype) -> torch.dtype:
    if dtype == torch.float16:
        return torch.float16
    if dtype == torch.bfloat16:
        return torch.bfloat16
    return torch.float32


@torch.no_grad()
def quantize_qkv_for_tilemix(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ: int = 128,
                             BLKK: int = 64, sm_scale: float = None):
    """Quantise Q, K and V per block (tilemix.py:45-107)."""
    q8, q_scale_blocks, k8, k_scale_blocks, cu_q_scale, cu_k_scale = quant_per_block_int8(
        q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ=BLKQ, BLKK=BLKK, sm_scale=1.0)
    v8, v_scale_blocks, cu_v_scale = per_block_int8_single(v, cu_seqlens_k, max_seqlen_k, BLK=BLKK, sm_scale=1.0)
    sd = _scale_dtype(q.dtype)
    return (q8, q_scale_blocks.to(dtype=sd).contiguous(), cu_q_scale.to(dtype=torch.int32).contiguous(),
            k8, k_scale_blocks.to(dtype=sd).contiguous(), cu_k_scale.to(dtype=torch.int32).contiguous(),
            v8, v_scale_blocks.to(dtype=sd).contiguous(), cu_v_scale.to(dtype=torch.int32).contiguous())


@torch.no_grad()
def quantize_qk_for_tilemix(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ: int = 128,
                            BLKK: int = 64, sm_scale: float = None):
    """Quantise Q and K per block (tilemix.py:110-156)."""
    q8, q_scale_blocks, k8, k_scale_blocks, cu_q_scale, cu_k_scale = quant_per_block_int8(
        q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ=BLKQ, BLKK=BLKK, sm_scale=1.0)
    sd = _scale_dtype(q.dtype)
    return (q8.contiguous(), q_scale_blocks.to(dtype=sd).contiguous(), cu_q_scale.to(dtype=torch.int32).contiguous(),
            k8.contiguous(), k_scale_blocks.to(dtype=sd).contiguous(), cu_k_scale.to(dtype=torch.int32).contiguous())


def _routing_mode_code(mode: str) -> int:
    normalized = mode.strip().lower()
    codes = {"mixed": ROUTING_MODE_MIXED, "fp16": ROUTING_MODE_FP16, "int8": ROUTING_MODE_INT8}
    if normalized not in codes:
        raise ValueError(f"routing_mode must be one of {tuple(codes)}, got {mode!r}")
    return codes[normalized]


def classify_bitmask_routing(precision_bitmask: torch.Tensor, *, seqlen_q: int, seqlen_k: int, block_m: int,
                             block_n: int, block_n_mask: int, causal: bool) -> Literal["mixed", "fp16", "int8"]:
    """"fp16" / "int8" when every routing bit the kernel reads selects that format, else
    "mixed" (the contract of tilemix.py:968-1014).

    The bits a row reads are the mask groups its causal key range reaches; all rows are
    tested at once with tensor ops on the map's own device, and only the two verdicts
    cross to the host. The answer is remembered on the map tensor per argument set and
    reused while the tensor is not modified in place (its version counter is unchanged),
    so repeated ``routing_mode="auto"`` calls on a cached map cost no device sync.
    """
    if block_n_mask % block_n != 0:
        raise ValueError("block_n_mask must be a multiple of block_n")
    m_blocks = (seqlen_q + block_m - 1) // block_m
    n_rows = precision_bitmask.numel()
    if n_rows == 0 or m_blocks <= 0 or n_rows % m_blocks:
        raise ValueError("precision_bitmask has an invalid row count")
    key = (seqlen_q, seqlen_k, block_m, block_n, block_n_mask, bool(causal))
    memo = getattr(precision_bitmask, "_tilemix_routing", None)
    version = precision_bitmask._version
    if memo is not None and memo.get(key, (None, None))[0] == version:
        return memo[key][1]
    words = precision_bitmask.detach().reshape(-1)
    words = words.view(torch.int64) if words.dtype == torch.uint64 else words.to(torch.int64)
    compute_blocks = (seqlen_k + block_n - 1) // block_n
    group = block_n_mask // block_n
    if causal:
        query_block = torch.arange(n_rows, device=words.device, dtype=torch.int64) % m_blocks
        first_hidden = (query_block + 1) * block_m + (seqlen_k - seqlen_q)
        row_tiles = torch.div(first_hidden + block_n - 1, block_n, rounding_mode="floor").clamp(0, compute_blocks)
    else:
        row_tiles = torch.full((n_rows,), compute_blocks, device=words.device, dtype=torch.int64)
    groups = torch.div(row_tiles + group - 1, group, rounding_mode="floor")
    # Bits [0, groups) of each row; a row reaching past bit 63 can never be all-INT8.
    all_ones = torch.full_like(groups, -1)
    valid = torch.where(groups >= 64, all_ones, (torch.ones_like(groups) << groups.clamp(max=63)) - 1)
    routed = words & valid
    verdict = torch.stack([(routed == 0).all(), ((routed == valid) & (groups <= 64)).all()]).tolist()
    mode = "fp16" if verdict[0] else ("int8" if verdict[1] else "mixed")
    if memo is None:
        memo = {}
        try:
            precision_bitmask._tilemix_routing = memo
        except AttributeError:
            memo = None
    if memo is not None:
        memo[key] = (version, mode)
    return mode


def _ptr(t: Optional[torch.Tensor]) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _launch(q, k, v, o, cu_q, cu_k, bitmask, max_q, max_k, *, q8=None, sq=None, cuqs=None, k8=None, sk=None,
            cuks=None, v8=None, sv=None, cuvs=None, v8_f16=None, bias=None, block_m, block_n, block_n_mask, BLKQ,
            BLKK, causal,
            sm_scale, mode_code, scalar_scales, int8_use_fp16_v, threshold=None) -> None:
    p = TmAttnParams()
    p.q, p.k, p.v = _ptr(q), _ptr(k), _ptr(v)
    p.q_stride_tok, p.q_stride_head = q.stride(0), q.stride(1)
    p.k_stride_tok, p.k_stride_head = k.stride(0), k.stride(1)
    p.v_stride_tok, p.v_stride_head = v.stride(0), v.stride(1)
    p.q_tokens, p.k_tokens = q.shape[0], k.shape[0]
    p.out = _ptr(o)
    p.o_stride_tok, p.o_stride_head = o.stride(0), o.stride(1)
    if q8 is not None:
        p.q8 = _ptr(q8)
        p.q8_stride_tok, p.q8_stride_head = q8.stride(0), q8.stride(1)
        p.q_scale, p.cu_q_scale = _ptr(sq), _ptr(cuqs)
    if k8 is not None:
        p.k8 = _ptr(k8)
        p.k8_stride_tok, p.k8_stride_head = k8.stride(0), k8.stride(1)
        p.k_scale, p.cu_k_scale = _ptr(sk), _ptr(cuks)
    if v8 is not None:
        p.v8 = _ptr(v8)
        p.v8_stride_tok, p.v8_stride_head = v8.stride(0), v8.stride(1)
    if v8_f16 is not None:
        p.v8_f16 = _ptr(v8_f16)
        p.v8_f16_stride_tok, p.v8_f16_stride_head = v8_f16.stride(0), v8_f16.stride(1)
    if sv is not None:
        p.v_scale, p.cu_v_scale = _ptr(sv), _ptr(cuvs)
    if bias is not None:
        p.bias = _ptr(bias)
        for i in range(4):
            p.bias_stride[i] = bias.stride(i)
    p.cu_seqlens_q, p.cu_seqlens_k = _ptr(cu_q), _ptr(cu_k)
    p.precision_bitmask = _ptr(bitmask)
    p.batch = cu_q.numel() - 1
    p.heads_q, p.heads_k, p.head_dim = q.shape[1], k.shape[1], q.shape[2]
    p.max_seqlen_q, p.max_seqlen_k = int(max_q), int(max_k)
    p.block_m, p.block_n, p.block_n_mask = block_m, block_n, block_n_mask
    p.blkq, p.blkk = BLKQ, BLKK
    p.causal = int(bool(causal))
    p.routing_mode = mode_code
    p.scalar_scales = int(bool(scalar_scales))
    p.int8_use_fp16_v = int(bool(int8_use_fp16_v))
    p.sm_scale = float(sm_scale)
    p.error_flag = _ptr(_error_word(q.device))
    tune = TmAttnTuning()
    tune.rescale_threshold = rescale_threshold() if threshold is None else float(threshold)
    tune.force_general = 1 if _force_general() else 0
    tune.numerics = numerics_code()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib().tm_attn_fwd_ex(ctypes.byref(p), ctypes.byref(tune), ctypes.c_void_p(stream))
    check(rc, "tm_attn_fwd")


def _check_kernel_support(q, block_m, block_n, BLKK, int8_path: bool, int8_use_fp16_v: bool, bias,
                          max_q: int = 0, max_k: int = 0) -> None:
    if q.dtype != torch.float16:
        raise TypeError("the sm_100a TileMix kernel computes in fp16; q, k and v must be torch.float16")
    if q.shape[-1] not in (64, 128):
        raise ValueError("the sm_100a TileMix kernel supports head_dim 64 and 128")
    if block_m not in (64, 128) or block_n % 64 != 0:
        raise ValueError("the sm_100a TileMix kernel supports block_m in (64, 128) and block_n a multiple of 64")
    if int8_path and BLKK % 64 != 0:
        raise ValueError("the sm_100a TileMix kernel needs BLKK to be a multiple of 64")
    if bias is not None:
        # The kernel reads bias[0, hq, row, key] (the reference indexes it without a batch offset) and only
        # inside the tensor; the reference would read past a smaller bias.
        if bias.dtype != torch.float16:
            raise NotImplementedError("the sm_100a TileMix kernel takes an fp16 bias")
        if bias.device != q.device:
            raise ValueError("bias must be on q.device")
        if bias.ndim != 4 or bias.shape[1] < q.shape[1] or bias.shape[2] < max_q or bias.shape[3] < max_k:
            raise ValueError("bias must be [batch, heads_q, >= max_seqlen_q, >= max_seqlen_k]")


@torch.no_grad()
def launch_prequantized(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlens_q: int, max_seqlens_k: int,
                        precision_bitmask, *, q8, k8, v8, sQ_blocks, sK_blocks, sV_blocks, cu_q_scale, cu_k_scale,
                        cu_v_scale, block_m: int = 128, block_n: int = 64, block_n_mask: Optional[int] = None,
                        BLKQ: int = 128, BLKK: int = 64, causal: bool = False, sm_scale: Optional[float] = None,
                        bias: Optional[torch.Tensor] = None, o: Optional[torch.Tensor] = None,
                        routing_mode: RoutingMode = "auto", run_length: bool = False, scalar_scales: bool = True,
                        int8_cache_ca: bool = False, int8_use_fp16_v: bool = False):
    """Launch the attention kernel on prequantised Q/K(/V) (tilemix.py:1132-1336)."""
    if block_n_mask is None:
        block_n_mask = block_n
    # The reference's order: layout checks, routing classification, quantised tensors, then
    # the head-dimension limit.
    _validate(q, k, v, max_seqlens_q, max_seqlens_k, precision_bitmask, block_m, block_n, block_n_mask, BLKQ,
              BLKK, scalar_scales, head_dim_rule=False)
    normalized_mode = routing_mode.strip().lower()
    if normalized_mode == "auto":
        normalized_mode = classify_bitmask_routing(precision_bitmask, seqlen_q=max_seqlens_q,
                                                   seqlen_k=max_seqlens_k, block_m=block_m, block_n=block_n,
                                                   block_n_mask=block_n_mask, causal=causal)
    mode_code = _routing_mode_code(normalized_mode)
    quant_tensors = (q8, k8, v8, sQ_blocks, sK_blocks, sV_blocks, cu_q_scale, cu_k_scale, cu_v_scale)
    _raise_first((
        (lambda: any(t.device != q.device for t in quant_tensors),
         ValueError("all quantization tensors must share q.device")),
        (lambda: {q8.dtype, k8.dtype} != {torch.int8}, TypeError("q8 and k8 must be torch.int8")),
        (lambda: v8.dtype != torch.int8, TypeError("v8 must be torch.int8")),
        (lambda: q.shape[-1] > 128, ValueError("head dimension must be <= 128")),
    ))
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    if o is None:
        o = torch.empty_like(q)
    cu_seqlens_q = cu_seqlens_q.to(device=q.device, dtype=torch.int32).contiguous()
    cu_seqlens_k = cu_seqlens_k.to(device=q.device, dtype=torch.int32).contiguous()
    precision_bitmask = precision_bitmask.to(device=q.device, dtype=torch.uint64).contiguous()
    int8_path = mode_code != ROUTING_MODE_FP16
    _check_kernel_support(q, block_m, block_n, BLKK, int8_path, int8_use_fp16_v, bias, max_seqlens_q, max_seqlens_k)
    kw = {}
    if int8_path:
        kw = dict(q8=q8, sq=sQ_blocks.to(torch.float16).contiguous(), cuqs=cu_q_scale.to(torch.int32).contiguous(),
                  k8=k8, sk=sK_blocks.to(torch.float16).contiguous(), cuks=cu_k_scale.to(torch.int32).contiguous())
        if not int8_use_fp16_v:
            kw.update(v8=v8, sv=sV_blocks.to(torch.float16).contiguous(),
                      cuvs=cu_v_scale.to(torch.int32).contiguous())
    _launch(q, k, v, o, cu_seqlens_q, cu_seqlens_k, precision_bitmask, max_seqlens_q, max_seqlens_k,
            block_m=block_m, block_n=block_n, block_n_mask=block_n_mask, BLKQ=BLKQ, BLKK=BLKK, causal=causal,
            sm_scale=sm_scale, mode_code=mode_code, scalar_scales=scalar_scales,
            int8_use_fp16_v=int8_use_fp16_v, bias=bias, **kw)
    return o, normalized_mode


def _force_general() -> bool:
    return os.environ.get("TILEMIX_B200_KERNEL", "").strip().lower() == "general"


def _quantize_v_f16(v, cu_seqlens_k, max_seqlen_k, BLKK, equal_len: Optional[int] = None):
    """V codes as exact fp16 values + fp16 block scales + int32 block offsets (the
    quantiser of _quantize_k, writing the codes the paired kernel's INT8-V PV reads)."""
    batch = cu_seqlens_k.numel() - 1
    if equal_len is not None:
        nblk = (equal_len + BLKK - 1) // BLKK
        cu_scale_i32 = torch.arange(0, (batch + 1) * nblk, nblk, device=v.device, dtype=torch.int32)
        n_rows = batch * nblk
    else:
        _, cu_scale_i32 = _scale_offsets(cu_seqlens_k, BLKK, max_seqlen_k)
        n_rows = v.shape[0] // BLKK + batch
    if v.stride(-1) != 1:
        raise ValueError("the head dimension must be contiguous")
    v16 = torch.empty(v.shape, dtype=torch.float16, device=v.device)
    sv16 = torch.empty((n_rows, v.shape[1]), dtype=torch.float16, device=v.device)
    cu_i32 = cu_seqlens_k.to(device=v.device, dtype=torch.int32).contiguous()
    stream = torch.cuda.current_stream(v.device).cuda_stream
    with torch.cuda.device(v.device):
        rc = lib().tm_quant_per_block_int8_f16(
            ctypes.c_void_p(v.data_ptr()), v.stride(0), v.stride(1), ctypes.c_void_p(cu_i32.data_ptr()),
            ctypes.c_void_p(cu_scale_i32.data_ptr()), batch, v.shape[1], v.shape[2], BLKK, int(max_seqlen_k),
            ctypes.c_void_p(0), 0, 0, ctypes.c_void_p(v16.data_ptr()), v16.stride(0), v16.stride(1),
            ctypes.c_void_p(0), ctypes.c_void_p(sv16.data_ptr()), numerics_code(), ctypes.c_void_p(stream))
    check(rc, "tm_quant_per_block_int8_f16")
    return v16, sv16, cu_scale_i32


def _quantize_k(k, cu_seqlens_k, max_seqlen_k, BLKK, equal_len: Optional[int] = None):
    """K codes + fp16 block scales + int32 block offsets, without a host sync: for varlen
    batches the scale rows are allocated for the bound sum_b ceil(T_b / BLKK) <= tokens / BLKK
    + batch, and the offsets stay on the device."""
    batch = cu_seqlens_k.numel() - 1
    if equal_len is not None:
        nblk = (equal_len + BLKK - 1) // BLKK
        cu_scale_i32 = torch.arange(0, (batch + 1) * nblk, nblk, device=k.device, dtype=torch.int32)
        n_rows = batch * nblk
    else:
        _, cu_scale_i32 = _scale_offsets(cu_seqlens_k, BLKK, max_seqlen_k)
        n_rows = k.shape[0] // BLKK + batch
    k8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    sk16 = torch.empty((n_rows, k.shape[1]), dtype=torch.float16, device=k.device)
    cu_i32 = cu_seqlens_k.to(device=k.device, dtype=torch.int32).contiguous()
    _launch_quant(k, cu_i32, cu_scale_i32, max_seqlen_k, BLKK, 1.0, k8, None, sk16)
    return k8, sk16, cu_scale_i32


@torch.no_grad()
def _attention_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlens_q, max_seqlens_k, precision_bitmask, *,
                       block_m, block_n, block_n_mask, BLKQ, BLKK, causal, sm_scale, mode: str, scalar_scales,
                       int8_use_fp16_v, bias=None, equal_len: Optional[int] = None, o=None, threshold=None,
                       k_quant=None):
    mode_code = _routing_mode_code(mode)
    int8_path = mode_code != ROUTING_MODE_FP16
    _check_kernel_support(q, block_m, block_n, BLKK, int8_path, int8_use_fp16_v, bias, max_seqlens_q, max_seqlens_k)
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    if o is None:
        o = torch.empty_like(q)
    cu_q = cu_seqlens_q.to(device=q.device, dtype=torch.int32).contiguous()
    cu_k = cu_seqlens_k.to(device=q.device, dtype=torch.int32).contiguous()
    bm = precision_bitmask.to(device=q.device, dtype=torch.uint64).contiguous()
    kw = {}
    if int8_path:
        if k_quant is not None and equal_len is not None and BLKK == 64:
            # K codes and fp16 block scales already made (by the RoPE pass), blocks of 64 tokens
            # per equal-length sequence.
            k8, sk16 = k_quant
            nblk = (equal_len + BLKK - 1) // BLKK
            batch = cu_k.numel() - 1
            cuks = torch.arange(0, (batch + 1) * nblk, nblk, device=k.device, dtype=torch.int32)
        else:
            k8, sk16, cuks = _quantize_k(k, cu_k, max_seqlens_k, BLKK, equal_len)
        kw = dict(k8=k8, sk=sk16, cuks=cuks)
        if BLKQ != 128:
            q8, sq, cuq = per_block_int8_single(q, cu_q, max_seqlens_q, BLK=BLKQ, sm_scale=1.0)
            kw.update(q8=q8, sq=sq.to(torch.float16).contiguous(), cuqs=cuq.to(torch.int32).contiguous())
        if not int8_use_fp16_v:
            # V per BLKK block as K (tilemix.py:45-107): the INT8-V PV path of INT8-routed tiles.
            # The paired kernel (head_dim 128, block_m 128, Q quantised in kernel, no bias)
            # reads the codes as exact fp16 values; the general kernel reads the int8 codes.
            paired = (q.shape[-1] == 128 and block_m == 128 and BLKQ == 128 and bias is None
                      and BLKK in (64, 128) and not _force_general())
            if paired:
                v16, sv16, cuvs = _quantize_v_f16(v, cu_k, max_seqlens_k, BLKK, equal_len)
                kw.update(v8_f16=v16, sv=sv16, cuvs=cuvs)
            else:
                v8, sv16, cuvs = _quantize_k(v, cu_k, max_seqlens_k, BLKK, equal_len)
                kw.update(v8=v8, sv=sv16, cuvs=cuvs)
    _launch(q, k, v, o, cu_q, cu_k, bm, max_seqlens_q, max_seqlens_k, block_m=block_m, block_n=block_n,
            block_n_mask=block_n_mask, BLKQ=BLKQ, BLKK=BLKK, causal=causal, sm_scale=sm_scale,
            mode_code=mode_code, scalar_scales=scalar_scales, int8_use_fp16_v=int8_use_fp16_v,
            threshold=threshold, bias=bias, **kw)
    return o


@torch.no_grad()
def tilemix_attention_with_quant(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlens_q: int, max_seqlens_k: int,
                                 precision_bitmask, *, block_m: int = 128, block_n: int = 64,
                                 block_n_mask: Optional[int] = None, BLKQ: int = 128, BLKK: int = 64,
                                 causal: bool = False, sm_scale: Optional[float] = None,
                                 bias: Optional[torch.Tensor] = None, routing_mode: RoutingMode = "auto",
                                 run_length: bool = False, scalar_scales: bool = True, int8_cache_ca: bool = False,
                                 int8_use_fp16_v: bool = False):
    """Quantise and run the routed attention (tilemix.py:1340-1447). Returns (out, mode)."""
    if block_n_mask is None:
        block_n_mask = block_n
    normalized_mode = routing_mode.strip().lower()
    if normalized_mode == "auto":
        normalized_mode = classify_bitmask_routing(precision_bitmask, seqlen_q=max_seqlens_q,
                                                   seqlen_k=max_seqlens_k, block_m=block_m, block_n=block_n,
                                                   block_n_mask=block_n_mask, causal=causal)
    _validate(q, k, v, max_seqlens_q, max_seqlens_k, precision_bitmask, block_m, block_n, block_n_mask, BLKQ,
              BLKK, scalar_scales)
    _routing_mode_code(normalized_mode)
    o = _attention_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlens_q, max_seqlens_k, precision_bitmask,
                           block_m=block_m, block_n=block_n, block_n_mask=block_n_mask, BLKQ=BLKQ, BLKK=BLKK,
                           causal=causal, sm_scale=sm_scale, mode=normalized_mode, scalar_scales=scalar_scales,
                           int8_use_fp16_v=int8_use_fp16_v, bias=bias)
    return o, normalized_mode


def _raise_first(rules) -> None:
    """Raise the exception of the first rule whose predicate holds (rules in order)."""
    for failing, error in rules:
        if failing():
            raise error


def _validate(q, k, v, max_q, max_k, bitmask, block_m, block_n, block_n_mask, BLKQ, BLKK, scalar_scales,
              head_dim_rule: bool = True):
    """Argument checks of launch_prequantized (tilemix.py:1167-1201): the same exception types
    and messages, in the same order, so callers see the reference's first error. Each rule is
    a (predicate of a failing call, exception) pair evaluated lazily; later rules may assume
    the earlier ones held. ``head_dim_rule=False`` leaves the head-dimension limit to the
    caller (launch_prequantized checks it after its quantised tensors, as the reference)."""
    rows = k.shape[1] * ((max_q + block_m - 1) // block_m) if k.ndim == 3 else 0
    _raise_first((
        (lambda: not q.is_cuda, RuntimeError("TileMix is a CUDA-only kernel")),
        (lambda: 3 != q.ndim or 3 != k.ndim or 3 != v.ndim,
         ValueError("expected flattened [tokens, heads, dim] tensors")),
        (lambda: v.shape != k.shape or k.shape[-1] != q.shape[-1],
         ValueError("K/V shapes and Q/K/V head dimensions must match")),
        (lambda: q.shape[1] % k.shape[1], ValueError("Q heads must be divisible by KV heads")),
        (lambda: {k.device, v.device} != {q.device}, ValueError("q, k, and v must share one CUDA device")),
        (lambda: {k.dtype, v.dtype} != {q.dtype}, TypeError("q, k, and v must share one dtype")),
        (lambda: max_k != max_q, ValueError("packed routing currently requires equal Q/K lengths")),
        (lambda: block_n_mask % block_n, ValueError("block_n_mask must be a multiple of block_n")),
        (lambda: -(-max_k // block_n_mask) > 64, ValueError("packed routing exceeds 64 mask blocks")),
        (lambda: scalar_scales and (BLKQ, BLKK) != (block_m, block_n),
         ValueError("scalar_scales requires block_m == BLKQ and block_n == BLKK")),
        (lambda: bitmask.dtype != torch.uint64, TypeError("precision_bitmask must be torch.uint64")),
        (lambda: bitmask.numel() != rows,
         ValueError(f"precision_bitmask has {bitmask.numel()} rows, expected {rows}")),
        (lambda: head_dim_rule and q.shape[-1] > 128, ValueError("head dimension must be <= 128")),
    ))


