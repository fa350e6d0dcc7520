"""ctypes binding of the C-ABI library ``libtilemix_b200.so`` (include/tilemix_b200.h).

The product path has no fallback: if the shared library is missing or cannot
be loaded, :func:`lib` raises. Build it with ``python -m tilemix_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("TILEMIX_B200_LIB", _PKG / "libtilemix_b200.so"))

TM_OK = 0
TM_ROUTE_MIXED, TM_ROUTE_FP16, TM_ROUTE_INT8 = 0, 1, 2
TM_NUMERICS_GPU, TM_NUMERICS_EXACT = 0, 1


def numerics_mode() -> str:
    """The numerics every op of the package computes in (``TILEMIX_B200_NUMERICS``):

    ``"gpu"`` (default): the reference's Triton kernels as they execute on the GPU (FP16-route
    QK^T accumulated in fp16 by the tensor core, the quantiser's and the output's fp32
    divisions by the approximate ``div.full.f32`` that Triton emits for ``/``); outputs then
    match the reference run on the same GPU. ``"exact"``: the same algorithm in exact
    arithmetic (fp32 accumulation rounded once, IEEE divisions), as the reference's Triton
    interpreter runs it on the CPU.
    """
    mode = os.environ.get("TILEMIX_B200_NUMERICS", "gpu").strip().lower()
    if mode not in ("gpu", "exact"):
        raise ValueError(f"TILEMIX_B200_NUMERICS must be 'gpu' or 'exact', got {mode!r}")
    return mode


def numerics_code() -> int:
    """TM_NUMERICS_* value of :func:`numerics_mode`."""
    return TM_NUMERICS_GPU if numerics_mode() == "gpu" else TM_NUMERICS_EXACT

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_void_p = ctypes.c_void_p


class TmAttnParams(ctypes.Structure):
    """Mirror of ``tm_attn_params`` (include/tilemix_b200.h)."""

    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p),
        ("q_stride_tok", c_i64), ("q_stride_head", c_i64),
        ("k_stride_tok", c_i64), ("k_stride_head", c_i64),
        ("v_stride_tok", c_i64), ("v_stride_head", c_i64),
        ("q_tokens", c_i64), ("k_tokens", c_i64),
        ("out", c_void_p), ("o_stride_tok", c_i64), ("o_stride_head", c_i64),
        ("q8", c_void_p), ("q8_stride_tok", c_i64), ("q8_stride_head", c_i64),
        ("q_scale", c_void_p), ("cu_q_scale", c_void_p),
        ("k8", c_void_p), ("k8_stride_tok", c_i64), ("k8_stride_head", c_i64),
        ("k_scale", c_void_p), ("cu_k_scale", c_void_p),
        ("v8", c_void_p), ("v8_stride_tok", c_i64), ("v8_stride_head", c_i64),
        ("v_scale", c_void_p), ("cu_v_scale", c_void_p),
        ("v8_f16", c_void_p), ("v8_f16_stride_tok", c_i64), ("v8_f16_stride_head", c_i64),
        ("cu_seqlens_q", c_void_p), ("cu_seqlens_k", c_void_p),
        ("precision_bitmask", c_void_p),
        ("bias", c_void_p), ("bias_stride", c_i64 * 4),
        ("batch", c_int), ("heads_q", c_int), ("heads_k", c_int), ("head_dim", c_int),
        ("max_seqlen_q", c_int), ("max_seqlen_k", c_int),
        ("block_m", c_int), ("block_n", c_int), ("block_n_mask", c_int), ("blkq", c_int), ("blkk", c_int),
        ("causal", c_int), ("routing_mode", c_int), ("run_length", c_int), ("scalar_scales", c_int),
        ("int8_use_fp16_v", c_int),
        ("sm_scale", ctypes.c_float),
        ("error_flag", c_void_p),
    ]


class TmAttnTuning(ctypes.Structure):
    """Mirror of ``tm_attn_tuning`` (include/tilemix_b200.h)."""

    _fields_ = [("rescale_threshold", ctypes.c_float), ("force_general", c_int), ("numerics", c_int)]


class TmMapParams(ctypes.Structure):
    """Mirror of ``tm_map_params`` (include/tilemix_b200.h)."""

    _fields_ = [
        ("seq_len", c_int), ("block_m", c_int), ("block_n_mask", c_int), ("compute_block_n", c_int),
        ("pattern", c_int), ("percentage", ctypes.c_double), ("stride", c_int), ("c", c_int),
        ("key_pos", ctypes.POINTER(c_i64)), ("num_key_pos", c_int),
        ("num_global_block", c_int), ("num_rand_block", c_int),
    ]


# (name, restype, argtypes) of every exported entry point.
SIGNATURES = {
    "tm_quant_per_block_int8": (c_int, [c_void_p, c_i64, c_i64, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                        c_int, ctypes.c_float, c_void_p, c_i64, c_i64, c_void_p, c_void_p,
                                        c_void_p]),
    "tm_quant_per_block_int8_ex": (c_int, [c_void_p, c_i64, c_i64, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                           c_int, ctypes.c_float, c_void_p, c_i64, c_i64, c_void_p, c_void_p,
                                           c_int, c_void_p]),
    "tm_quant_per_block_int8_f16": (c_int, [c_void_p, c_i64, c_i64, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                            c_int, c_void_p, c_i64, c_i64, c_void_p, c_i64, c_i64, c_void_p,
                                            c_void_p, c_int, c_void_p]),
    "tm_attn_fwd": (c_int, [ctypes.POINTER(TmAttnParams), c_void_p]),
    "tm_attn_fwd_ex": (c_int, [ctypes.POINTER(TmAttnParams), ctypes.POINTER(TmAttnTuning), c_void_p]),
    "tm_attn_fwd_noalloc": (c_int, [ctypes.POINTER(TmAttnParams), ctypes.POINTER(TmAttnTuning), c_void_p]),
    "tm_build_precision_map": (c_int, [ctypes.POINTER(TmMapParams), c_void_p, c_void_p, c_void_p]),
    "tm_rotary_token_major": (c_int, [c_void_p, c_i64, c_i64, c_i64, c_void_p, c_i64, c_i64, c_i64,
                                      c_void_p, c_i64, c_i64, c_void_p, c_i64, c_i64, c_int, c_int, c_int,
                                      c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                      c_int, c_void_p]),
    "tm_silu_mul": (c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_void_p]),
    "tm_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_int, ctypes.c_float, c_void_p]),
    "tm_status_string": (ctypes.c_char_p, [c_int]),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raises if it is unavailable."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"tilemix_b200 native library not found at {LIB_PATH}; build it with "
                "`python -m tilemix_b200.build` (no CPU fallback exists)")
        handle = ctypes.CDLL(str(LIB_PATH))
        missing = [name for name in SIGNATURES if not hasattr(handle, name)]
        if missing:
            raise RuntimeError(f"{LIB_PATH} lacks {missing}; rebuild it with `python -m tilemix_b200.build --force`")
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(status: int, what: str) -> None:
    """Raise RuntimeError for a non-zero status returned by the library."""
    if status != TM_OK:
        msg = lib().tm_status_string(status).decode()
        raise RuntimeError(f"{what} failed with status {status}: {msg}")
