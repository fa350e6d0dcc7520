"""Routing maps built on the GPU (drop-in for the reference's
``attention/precision_maps.py`` entry point used by the model integration).

``make_precision_bitmask`` keeps the reference's signature, validation errors
and result (precision_maps.py:404-636): one ``torch.uint64`` word per query
block, bit j set = mask group j of that block runs the INT8 QK^T path. The map
is built by the CUDA kernel ``tm_build_precision_map`` in one launch, bit for
bit equal to the reference's, including its seeded random draws (torch's CPU
Mersenne Twister, seed 42). Differences, none in the words produced:

  * the result lives on a CUDA device (``device``, default the current one)
    instead of the CPU, ready for the attention launch;
  * torch's global random generator is left untouched (the reference reseeds
    it with ``torch.manual_seed(42)`` for row_rand and bigbird);
  * token-mask maps (``token_mask`` given, or patterns outside the
    percentage-aware block policy) are not built here: NotImplementedError.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from tilemix_b200._lib import TmMapParams, check, lib

PATTERN_CODES = {
    "zero": 0,
    "one": 1,
    "band": 2,
    "global": 3,
    "row_rand": 4,
    "align_sparse": 5,
    "bigbird": 6,
    "sptrans": 7,
}
BLOCK_PERCENTAGE_PATTERNS = ("band", "global", "row_rand", "align_sparse", "bigbird", "sptrans")


def make_precision_bitmask(seq_len: int, BLOCK_M: int, BLOCK_N: int, token_mask: Optional[torch.Tensor],
                           percentage: float = None, pattern_type: str = None, pattern_params: dict = None,
                           COMPUTE_BLOCK_N: int = None, *, device=None, check_retarget: bool = True) -> torch.Tensor:
    """Packed INT8/FP16 routing words of ``ceil(seq_len / BLOCK_M)`` query blocks.

    ``BLOCK_N`` is the mask-group width (``block_n_mask``), ``COMPUTE_BLOCK_N``
    the attention tile width. With ``check_retarget`` (default) the call waits
    for the kernel and raises RuntimeError where the reference does (the
    weighted retarget missing its target by more than one mask-group weight);
    without it the launch stays asynchronous.
    """
    num_m = (seq_len + BLOCK_M - 1) // BLOCK_M
    num_n = (seq_len + BLOCK_N - 1) // BLOCK_N
    if COMPUTE_BLOCK_N is None:
        COMPUTE_BLOCK_N = BLOCK_N
    if BLOCK_N % COMPUTE_BLOCK_N != 0:
        raise ValueError(f"BLOCK_N(mask) ({BLOCK_N}) must be a multiple of COMPUTE_BLOCK_N ({COMPUTE_BLOCK_N})")
    if num_n > 64:
        raise ValueError(f"num_n_mask={num_n} > 64; BLOCK_N(mask) too small "
                         f"(seq_len={seq_len}, BLOCK_N(mask)={BLOCK_N})")
    params = pattern_params or {}
    if pattern_type in ("zero", "one"):
        pass
    elif pattern_type == "sptrans" and percentage is not None and pattern_params is not None:
        pass
    else:
        direct = (percentage is not None and pattern_type in BLOCK_PERCENTAGE_PATTERNS
                  and pattern_params is not None)
        if token_mask is None and not direct:
            raise ValueError("token_mask may be None only for a percentage-aware block policy")
        if not direct:
            raise NotImplementedError("token-mask routing maps are built by the reference's host code; the GPU "
                                      "builder covers zero, one and the percentage-aware block patterns")
    if pattern_type not in ("zero", "one"):
        percentage = float(percentage)
        if percentage < 0.0 or percentage > 1.0 or percentage != percentage:
            raise ValueError(f"percentage must be in [0, 1], got {percentage}")

    p = TmMapParams()
    p.seq_len, p.block_m, p.block_n_mask, p.compute_block_n = int(seq_len), int(BLOCK_M), int(BLOCK_N), \
        int(COMPUTE_BLOCK_N)
    p.pattern = PATTERN_CODES[pattern_type]
    p.percentage = 0.0 if percentage is None else float(percentage)
    key_pos_buf = None
    if pattern_type == "sptrans":
        stride = int(params.get("stride", min(128, seq_len // 4)))
        c = int(params.get("c", min(32, stride // 4)))
        if stride == 0:
            raise ZeroDivisionError("integer division or modulo by zero")
        if stride < 0:
            raise ValueError(f"sptrans stride must be positive, got {stride}")
        p.stride, p.c = stride, c
    elif pattern_type == "global":
        key_pos = [int(x) for x in params.get("key_pos", list(range(min(4, seq_len))))]
        key_pos_buf = (ctypes.c_int64 * max(len(key_pos), 1))(*key_pos)
        p.key_pos = ctypes.cast(key_pos_buf, ctypes.POINTER(ctypes.c_int64))
        p.num_key_pos = len(key_pos)
    elif pattern_type == "bigbird":
        p.num_global_block = int(params.get("num_global_block", 2))
        p.num_rand_block = int(params.get("num_rand_block", 3))
        if p.num_global_block < 0 or p.num_rand_block < 0:
            raise ValueError("bigbird num_global_block and num_rand_block must be non-negative")

    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("the routing-map builder is a CUDA kernel; pass a CUDA device")
    out = torch.empty(num_m, dtype=torch.uint64, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        rc = lib().tm_build_precision_map(ctypes.byref(p), ctypes.c_void_p(out.data_ptr()),
                                          ctypes.c_void_p(err.data_ptr()), ctypes.c_void_p(stream))
    if rc == -4:  # TM_ERR_UNSUPPORTED: map larger than the single-CTA builder holds
        raise NotImplementedError(f"routing map of {num_m} x {num_n} cells exceeds the GPU builder's limit "
                                  "(4096 query blocks, 65536 cells)")
    check(rc, "tm_build_precision_map")
    if check_retarget and int(err.item()) != 0:
        raise RuntimeError("unable to retarget executable INT8 fraction within one mask-bit weight "
                           f"(seq_len={seq_len}, pattern={pattern_type}, percentage={percentage})")
    return out
