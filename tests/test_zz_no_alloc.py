"""tm_attn_fwd_noalloc (the attention entry point that takes its quantised-K
scratch from the library instead of the caller) against the regular path
(caller-owned K8 / scale buffers through tm_quant_per_block_int8 + tm_attn_fwd_ex):
identical outputs on consecutive calls with different shapes, and the size
limits enforced before anything is launched. Named to be collected last, so it
also runs after every other GPU test in the same process."""
import ctypes

import pytest
import torch

from tests.helpers import make_qkv, random_bitmask


def _params(q, k, v, o, cu, T, bm_words, block_m, mode=0, blkk=64):
    from tilemix_b200._lib import TmAttnParams

    p = TmAttnParams()
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    p.q, p.k, p.v, p.out = ptr(q), ptr(k), ptr(v), ptr(o)
    p.q_stride_tok, p.q_stride_head = q.stride(0), q.stride(1)
    p.k_stride_tok, p.k_stride_head = k.stride(0), k.stride(1)
    p.v_stride_tok, p.v_stride_head = v.stride(0), v.stride(1)
    p.o_stride_tok, p.o_stride_head = o.stride(0), o.stride(1)
    p.q_tokens, p.k_tokens = q.shape[0], k.shape[0]
    p.cu_seqlens_q = p.cu_seqlens_k = ptr(cu)
    p.precision_bitmask = ptr(bm_words)
    p.batch = cu.numel() - 1
    p.heads_q, p.heads_k, p.head_dim = q.shape[1], k.shape[1], q.shape[2]
    p.max_seqlen_q = p.max_seqlen_k = T
    p.block_m, p.block_n, p.block_n_mask, p.blkq, p.blkk = block_m, 64, 64, 128, blkk
    p.causal, p.routing_mode = 1, mode
    p.scalar_scales = int(block_m == 128)
    p.int8_use_fp16_v = 1
    p.sm_scale = q.shape[2] ** -0.5
    return p


# (lens, hq, hk, head_dim, block_m, routing mode, blkk): mixed routing with blocks of 64 keys, and all-INT8
# routing with blocks of 128 keys over an uneven varlen batch.
CASES = [([1024, 777], 6, 2, 128, 128, "mixed", 64), ([512, 300], 4, 4, 64, 64, "mixed", 64),
         ([1000, 129, 513], 6, 2, 128, 128, "int8", 128)]
MODES = {"mixed": 0, "fp16": 1, "int8": 2}


@pytest.mark.gpu
def test_noalloc_matches_caller_buffers_on_consecutive_calls(cuda_device):
    from tilemix_b200._lib import TmAttnTuning, check, lib, numerics_code
    from tilemix_b200.attention.tilemix import _attention_forward, device_error_code

    dev = cuda_device
    tune = TmAttnTuning()
    tune.rescale_threshold = 0.0
    tune.numerics = numerics_code()
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for call, (lens, hq, hk, d, block_m, mode, blkk) in enumerate(CASES + CASES[:1]):
        q, k, v, cu = make_qkv(lens, hq, hk, d, seed=20 + call, outliers=2)
        q, k, v, cu = q.to(dev), k.to(dev), v.to(dev), cu.to(dev)
        T = max(lens)
        words = random_bitmask(hk * ((T + block_m - 1) // block_m), seed=call).to(dev)
        ref = _attention_forward(q, k, v, cu, cu, T, T, words, block_m=block_m, block_n=64, block_n_mask=64,
                                 BLKQ=128, BLKK=blkk, causal=True, sm_scale=None, mode=mode,
                                 scalar_scales=block_m == 128 and blkk == 64, int8_use_fp16_v=True, threshold=0.0)
        out = torch.full_like(q, float("nan"))
        p = _params(q, k, v, out, cu, T, words, block_m, mode=MODES[mode], blkk=blkk)
        p.scalar_scales = int(block_m == 128 and blkk == 64)
        with torch.cuda.device(dev):
            check(lib().tm_attn_fwd_noalloc(ctypes.byref(p), ctypes.byref(tune), stream), "tm_attn_fwd_noalloc")
        torch.cuda.synchronize(dev)
        assert device_error_code(dev) == 0
        assert torch.equal(out, ref), call


def test_noalloc_rejects_oversize_and_caller_scratch():
    from tilemix_b200._lib import TmAttnTuning, lib

    q = torch.zeros(16, 8, 128, dtype=torch.float16)
    cu = torch.tensor([0, 16], dtype=torch.int32)
    words = torch.zeros(8, dtype=torch.uint64)
    p = _params(q, q, q, q, cu, 16, words, 128)
    tune = TmAttnTuning()
    p.k_tokens = 16385  # 16385 * 8 * 128 codes > 16 MiB of scratch
    assert lib().tm_attn_fwd_noalloc(ctypes.byref(p), ctypes.byref(tune), None) == -4
    p.k_tokens = 16
    p.k8 = ctypes.c_void_p(q.data_ptr())  # the K operand must come from the library
    assert lib().tm_attn_fwd_noalloc(ctypes.byref(p), ctypes.byref(tune), None) == -4
    p.k8 = None
    p.blkk = 192  # scale blocks of 64 or 128 keys only
    assert lib().tm_attn_fwd_noalloc(ctypes.byref(p), ctypes.byref(tune), None) == -4


def test_noalloc_rejects_one_scale_row_over_the_limit():
    """(k_tokens / blkk + batch) * heads_k scale rows may not exceed 262,144: 65,536 tokens of
    4 KV heads at head_dim 64 fill the 16 MiB of codes exactly, and a batch of 64,513
    sequences then needs 262,148 scale rows. Rejected before any CUDA call."""
    from tilemix_b200._lib import TmAttnTuning, lib

    q = torch.zeros(16, 4, 64, dtype=torch.float16)
    cu = torch.tensor([0, 16], dtype=torch.int32)
    words = torch.zeros(8, dtype=torch.uint64)
    p = _params(q, q, q, q, cu, 16, words, 128)
    p.k_tokens, p.batch = 65536, 64513
    assert lib().tm_attn_fwd_noalloc(ctypes.byref(p), ctypes.byref(TmAttnTuning()), None) == -4
