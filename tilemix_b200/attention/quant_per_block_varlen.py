"""Per-block INT8 quantisation on the B200 (drop-in for the reference's
``attention/triton/quant_per_block_varlen.py``).

Same functions, arguments and return values as the reference
(quant_per_block_varlen.py:48-106); the work runs in the sm_100a kernel
``tm_quant_per_block_int8_ex`` of ``libtilemix_b200.so``, in the numerics of
``tilemix_b200._lib.numerics_mode`` (by default the reference's GPU arithmetic, so
codes and scales equal those of its Triton quantiser run on the GPU).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from tilemix_b200._lib import check, lib, numerics_code


def _scale_offsets(cu_seqlens: torch.Tensor, BLK: int, max_seqlen: int):
    """cu_seqlens_scale (int64 like the reference's cumsum) and its int32 copy."""
    lens = cu_seqlens[1:] - cu_seqlens[:-1]
    nblk = (lens + BLK - 1) // BLK
    cu_scale = torch.nn.functional.pad(torch.cumsum(nblk, dim=0), (1, 0), value=0)
    return cu_scale, cu_scale.to(torch.int32).contiguous()


def _launch_quant(x: torch.Tensor, cu_seqlens_i32: torch.Tensor, cu_scale_i32: torch.Tensor, max_seqlen: int,
                  BLK: int, sm_scale: float, out: torch.Tensor, scale_f32: Optional[torch.Tensor],
                  scale_f16: Optional[torch.Tensor]) -> None:
    if x.dtype != torch.float16:
        raise TypeError("the sm_100a quantiser takes fp16 input")
    if x.stride(-1) != 1:
        raise ValueError("the head dimension must be contiguous")
    batch = cu_seqlens_i32.numel() - 1
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        rc = lib().tm_quant_per_block_int8_ex(
            ctypes.c_void_p(x.data_ptr()), x.stride(0), x.stride(1),
            ctypes.c_void_p(cu_seqlens_i32.data_ptr()), ctypes.c_void_p(cu_scale_i32.data_ptr()),
            batch, x.shape[1], x.shape[2], BLK, int(max_seqlen), float(sm_scale),
            ctypes.c_void_p(out.data_ptr()), out.stride(0), out.stride(1),
            ctypes.c_void_p(scale_f32.data_ptr() if scale_f32 is not None else 0),
            ctypes.c_void_p(scale_f16.data_ptr() if scale_f16 is not None else 0),
            numerics_code(), ctypes.c_void_p(stream))
    check(rc, "tm_quant_per_block_int8_ex")


def per_block_int8_single(x, cu_seqlens_x, max_seqlen_x, BLK=128, sm_scale=1.0):
    """Quantise one packed tensor; returns (x_int8, x_scale fp32, cu_seqlens_x_scale).

    Mirrors quant_per_block_varlen.py:48-75.
    """
    if not x.is_cuda:
        raise RuntimeError("tilemix_b200 quantisation runs on CUDA tensors only")
    x_int8 = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    cu_scale, cu_scale_i32 = _scale_offsets(cu_seqlens_x, BLK, max_seqlen_x)
    n_rows = int(cu_scale[-1].item())
    x_scale = torch.empty((n_rows, x.shape[1]), device=x.device, dtype=torch.float32)
    cu_i32 = cu_seqlens_x.to(device=x.device, dtype=torch.int32).contiguous()
    _launch_quant(x, cu_i32, cu_scale_i32, max_seqlen_x, BLK, sm_scale, x_int8, x_scale, None)
    return x_int8, x_scale, cu_scale


def per_block_int8(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ=128, BLKK=64,
                   sm_scale=None):
    """Quantise Q (BLKQ blocks) and K (BLKK blocks); mirrors quant_per_block_varlen.py:78-106."""
    head_dim = q.shape[-1]
    if sm_scale is None:
        sm_scale = head_dim ** -0.5
    if abs(sm_scale - 1.0) < 1e-6:
        q_sm_scale = 1.0
    else:
        q_sm_scale = sm_scale * 1.44269504
    q_int8, q_scale, cu_seqlens_q_scale = per_block_int8_single(q, cu_seqlens_q, max_seqlen_q, BLK=BLKQ,
                                                                sm_scale=q_sm_scale)
    k_int8, k_scale, cu_seqlens_k_scale = per_block_int8_single(k, cu_seqlens_k, max_seqlen_k, BLK=BLKK,
                                                                sm_scale=1.0)
    return q_int8, q_scale, k_int8, k_scale, cu_seqlens_q_scale, cu_seqlens_k_scale
