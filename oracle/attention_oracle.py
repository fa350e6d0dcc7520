"""CPU oracle for the TileMix attention hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference's Triton
kernels so that the sm_100a CUDA path can be checked against it. It is used
only by ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py``; the product path never imports it.

Pinning: every operation mirrors what the Triton interpreter
(``TRITON_INTERPRET=1``) executes for the reference source, op for op, so the
results are bit-identical to the reference run on the CPU:
  * ``tl.dot(fp16, fp16, out_dtype=fp16)`` is ``np.matmul(a, b, dtype=float16)``
    (float32 accumulation, one rounding), int8 dots are exact int32 matmuls,
    fp16 x fp16 -> fp32 dots are ``np.matmul(..., dtype=float32)``;
  * fp16 op fp32 promotes to fp32; ``tl.sum``/``tl.max`` are ``np.sum``/``np.max``;
    ``tl.math.exp2`` is ``np.exp2`` on float32.
``tests/golden/make_golden.py`` runs the reference itself under the
interpreter and ``tests/test_oracle.py`` checks this oracle against those
fixtures bit for bit.

References (paths inside the reference project):
  quantiser          attention/triton/quant_per_block_varlen.py:6-106
  softmax update     attention/triton/tilemix.py:179-207
  FP16 tile update   attention/triton/tilemix.py:210-300
  INT8 tile update   attention/triton/tilemix.py:303-500
  attn_fwd           attention/triton/tilemix.py:503-951
  host wrappers      attention/triton/tilemix.py:45-156, 954-1447
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634
ROUTING_MODE_MIXED, ROUTING_MODE_FP16, ROUTING_MODE_INT8 = 0, 1, 2

f16 = np.float16
f32 = np.float32


# ---------------------------------------------------------------------------
# Per-block INT8 quantiser (quant_per_block_varlen.py:6-45, :48-106)
# ---------------------------------------------------------------------------
def per_block_int8_single(x: np.ndarray, cu_seqlens: np.ndarray, max_seqlen: int, BLK: int = 128,
                          sm_scale: float = 1.0):
    """Quantise packed fp16 x [tokens, H, D] in blocks of BLK tokens per head.

    Returns (x_int8 [tokens,H,D] int8, scale [sum blocks, H] fp32, cu_seqlens_scale int32).
    Follows quant_per_block_varlen.py:6-45 (kernel) and :48-75 (launcher).
    """
    x = np.asarray(x)
    tokens, H, D = x.shape
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    lens = cu[1:] - cu[:-1]
    nblk = (lens + BLK - 1) // BLK
    cu_scale = np.concatenate([[0], np.cumsum(nblk)]).astype(np.int32)
    out = np.zeros((tokens, H, D), dtype=np.int8)
    scale = np.zeros((int(cu_scale[-1]), H), dtype=f32)
    sm = f32(sm_scale)
    for b in range(len(lens)):
        L = int(lens[b])
        for blk in range(int(nblk[b])):
            r0 = int(cu[b]) + blk * BLK
            r1 = int(cu[b]) + min(L, (blk + 1) * BLK)
            xb = x[r0:r1].astype(f32) * sm                      # :35-36
            s = (np.abs(xb).max(axis=(0, 2)) / f32(127.0)).astype(f32)   # :37 (per head)
            with np.errstate(divide="ignore", invalid="ignore"):
                y = (xb / s[None, :, None]).astype(f32)          # :38
            y = (y + f32(0.5) * np.where(y >= 0, f32(1), f32(-1))).astype(f32)  # :39
            with np.errstate(invalid="ignore"):
                q = np.where(np.isnan(y), 0, np.trunc(y)).astype(np.int64)
            out[r0:r1] = np.clip(q, -128, 127).astype(np.int8)   # :40 (.to(tl.int8))
            scale[int(cu_scale[b]) + blk] = s
    return out, scale, cu_scale


def per_block_int8(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ=128, BLKK=64,
                   sm_scale=None):
    """quant_per_block_varlen.py:78-106 (Q scaled by sm_scale*1.44269504 unless sm_scale == 1)."""
    head_dim = q.shape[-1]
    if sm_scale is None:
        sm_scale = head_dim ** -0.5
    q_sm_scale = 1.0 if abs(sm_scale - 1.0) < 1e-6 else sm_scale * 1.44269504
    q8, sq, cuqs = per_block_int8_single(q, cu_seqlens_q, max_seqlen_q, BLK=BLKQ, sm_scale=q_sm_scale)
    k8, sk, cuks = per_block_int8_single(k, cu_seqlens_k, max_seqlen_k, BLK=BLKK, sm_scale=1.0)
    return q8, sq, k8, sk, cuqs, cuks


# ---------------------------------------------------------------------------
# attn_fwd (tilemix.py:503-951)
# ---------------------------------------------------------------------------
def _softmax_prefix_update(qk16, m_i, l_i, acc):
    """tilemix.py:179-207."""
    with np.errstate(invalid="ignore", over="ignore"):
        qk_max = qk16.astype(f32).max(axis=1)
        has = qk_max != -np.inf
        m_next = np.maximum(m_i, qk_max)
        m_next = np.where(has, m_next, m_i).astype(f32)
        shifted = np.where(has[:, None], qk16.astype(f32) - m_next[:, None], f32(-np.inf)).astype(f32)
        p = np.exp2(shifted.astype(f32)).astype(f16)
        l_tile = np.sum(p.astype(f32), axis=1).astype(f32)
        alpha = np.where(has, np.exp2((m_i - m_next).astype(f32)), f32(1.0)).astype(f32)
    acc = (acc * alpha[:, None]).astype(f32)
    l_i = (l_i * alpha + l_tile).astype(f32)
    return p, m_next, l_i, acc


def attn_fwd(q, k, v, cu_q, cu_k, bitmask, *, q8=None, sq=None, cu_qs=None, k8=None, sk=None, cu_ks=None,
             v8=None, sv=None, cu_vs=None, max_seqlen_q, max_seqlen_k, block_m=128, block_n=64,
             block_n_mask=None, BLKQ=128, BLKK=64, causal=False, sm_scale=None, routing_mode=ROUTING_MODE_MIXED,
             scalar_scales=True, int8_use_fp16_v=False, bias=None, heads=None, q_blocks=None):
    """Reference attention forward on packed [tokens, heads, D] fp16 arrays.

    ``heads`` and ``q_blocks`` optionally restrict the computed Q heads and
    query blocks (others stay zero), for bounded CPU samples. Returns fp16
    [tokens, HQ, D].
    """
    q = np.asarray(q, dtype=f16)
    k = np.asarray(k, dtype=f16)
    v = np.asarray(v, dtype=f16)
    HQ, D = q.shape[1], q.shape[2]
    HK = k.shape[1]
    group = HQ // HK
    if block_n_mask is None:
        block_n_mask = block_n
    mask_group = block_n_mask // block_n
    if sm_scale is None:
        sm_scale = D ** -0.5
    qk_scale = f32(f32(sm_scale) * f32(LOG2E))                     # :639
    cu_q = np.asarray(cu_q, dtype=np.int64)
    cu_k = np.asarray(cu_k, dtype=np.int64)
    out = np.zeros_like(q)
    bm = None if bitmask is None else np.asarray(bitmask, dtype=np.uint64)
    n_m = (max_seqlen_q + block_m - 1) // block_m
    head_list = range(HQ) if heads is None else heads
    for z in range(len(cu_q) - 1):
        q0, k0 = int(cu_q[z]), int(cu_k[z])
        Tq, Tk = int(cu_q[z + 1]) - q0, int(cu_k[z + 1]) - k0
        for hq in head_list:
            hk = hq // group if group != 1 else hq                    # :588-592
            for start_m in (range(n_m) if q_blocks is None else q_blocks):
                if start_m * block_m >= Tq:                           # :600
                    continue
                n_blocks = (Tk + block_n - 1) // block_n              # :603
                if causal:
                    num = (start_m + 1) * block_m + Tk - Tq + block_n - 1
                    cb = int(np.trunc(num / block_n)) if num < 0 else num // block_n
                    n_blocks = min(n_blocks, cb)
                offs_m = start_m * block_m + np.arange(block_m)
                q_valid = offs_m < Tq
                rows = np.clip(offs_m, 0, max(Tq - 1, 0))
                qt = np.where(q_valid[:, None], q[q0 + rows, hq, :], f16(0)).astype(f16)
                q_fp16 = (qt.astype(f32) * qk_scale).astype(f16) if routing_mode != ROUTING_MODE_INT8 else None
                if routing_mode != ROUTING_MODE_FP16:
                    q8t = np.where(q_valid[:, None], q8[q0 + rows, hq, :], 0).astype(np.int8)
                    qs_base, qs_end = int(cu_qs[z]), int(cu_qs[z + 1])
                    if scalar_scales:
                        idx = min(qs_base + start_m * block_m // BLKQ, qs_end - 1)
                        sq_s = f16(sq[idx, hq]) if qs_end > qs_base else f16(1.0)
                        sq_v = np.full(block_m, sq_s, dtype=f16)
                    else:
                        idx = np.minimum(qs_base + offs_m // BLKQ, qs_end - 1)
                        sq_v = np.where(q_valid, sq[np.clip(idx, 0, None), hq], f16(1.0)).astype(f16)
                    ks_base, ks_end = int(cu_ks[z]), int(cu_ks[z + 1])
                    if not int8_use_fp16_v:
                        vs_base, vs_end = int(cu_vs[z]), int(cu_vs[z + 1])
                m_i = np.full(block_m, -np.inf, dtype=f32)
                l_i = np.ones(block_m, dtype=f32)                      # :728
                acc = np.zeros((block_m, D), dtype=f32)
                row_word = 0
                if routing_mode == ROUTING_MODE_MIXED:
                    m_blocks = (Tq + block_m - 1) // block_m          # :819
                    row_word = int(bm[hk * m_blocks + start_m])        # :820-823
                for nb in range(max(n_blocks, 0)):
                    if routing_mode == ROUTING_MODE_FP16:
                        use_int8 = False
                    elif routing_mode == ROUTING_MODE_INT8:
                        use_int8 = True
                    else:
                        use_int8 = bool((row_word >> (nb // mask_group)) & 1)   # :828-831
                    start_n = nb * block_n
                    keys = start_n + np.arange(block_n)
                    key_valid = keys < Tk
                    kidx = np.clip(keys, 0, max(Tk - 1, 0))
                    valid = np.broadcast_to(key_valid[None, :], (block_m, block_n))
                    if causal:
                        valid = valid & (offs_m[:, None] >= (keys + (Tq - Tk))[None, :])   # :257-261
                    if not use_int8:
                        kt = np.where(key_valid[:, None], k[k0 + kidx, hk, :], f16(0)).astype(f16)
                        qk = np.matmul(q_fp16, kt.T, dtype=f16)        # :254
                    else:
                        k8t = np.where(key_valid[:, None], k8[k0 + kidx, hk, :], 0).astype(np.int8)
                        if scalar_scales:
                            kidx_s = min(ks_base + start_n // BLKK, ks_end - 1)
                            sk_s = f16(sk[kidx_s, hk]) if ks_end > ks_base else f16(1.0)
                            ss = (f32(f16(sq_v[0] * sk_s)) * qk_scale).astype(f16)
                            score_scale = np.full((block_m, block_n), ss, dtype=f16)
                        else:
                            kidx_v = np.minimum(ks_base + keys // BLKK, ks_end - 1)
                            sk_v = np.where(key_valid, sk[np.clip(kidx_v, 0, None), hk], f16(1.0)).astype(f16)
                            prod = (sq_v[:, None] * sk_v[None, :]).astype(f16)
                            score_scale = (prod.astype(f32) * qk_scale).astype(f16)
                        qk_i32 = np.matmul(q8t.astype(np.int32), k8t.T.astype(np.int32))  # :401
                        qk = (qk_i32.astype(f32) * score_scale.astype(f32)).astype(f16)   # :402-404
                    qk = np.where(valid, qk, f16(-np.inf)).astype(f16)
                    if bias is not None:
                        # the reference indexes bias without a batch offset (:265-270)
                        braw = bias[0, hq, offs_m[:, None].clip(0, bias.shape[2] - 1),
                                    keys[None, :].clip(0, bias.shape[3] - 1)]
                        b = np.where(valid, braw, f16(0)).astype(f16)
                        qk = (qk + (b * f16(LOG2E)).astype(f16)).astype(f16)
                    p, m_i, l_i, acc = _softmax_prefix_update(qk, m_i, l_i, acc)
                    if (not use_int8) or int8_use_fp16_v:
                        vt = np.where(key_valid[:, None], v[k0 + kidx, hk, :], f16(0)).astype(f16)
                        pv = np.matmul(p.astype(f16), vt, dtype=f32)   # :299 / :448
                    else:
                        v8t = np.where(key_valid[:, None], v8[k0 + kidx, hk, :], 0).astype(np.int8)
                        if scalar_scales:
                            vidx = min(vs_base + start_n // BLKK, vs_end - 1)
                            sv_s = f16(sv[vidx, hk]) if vs_end > vs_base else f16(1.0)
                            p_scaled = (p * sv_s).astype(f16)
                        else:
                            vidx_v = np.minimum(vs_base + keys // BLKK, vs_end - 1)
                            sv_v = np.where(key_valid, sv[np.clip(vidx_v, 0, None), hk], f16(1.0)).astype(f16)
                            p_scaled = (p * sv_v[None, :]).astype(f16)
                        pv = np.matmul(p_scaled, v8t.astype(f16), dtype=f32)  # :497
                    acc = (acc + pv).astype(f32)
                with np.errstate(invalid="ignore", divide="ignore"):
                    o = (acc / l_i[:, None]).astype(f32).astype(f16)    # :935-936
                sel = np.nonzero(q_valid)[0]
                out[q0 + offs_m[sel], hq, :] = o[sel]
    return out


def quantize_qk_for_tilemix(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ=128, BLKK=64):
    """tilemix.py:110-156: quantise Q and K with sm_scale=1.0, cast scales to fp16."""
    q8, sq, k8, sk, cuqs, cuks = per_block_int8(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                                BLKQ=BLKQ, BLKK=BLKK, sm_scale=1.0)
    return q8, sq.astype(f16), cuqs, k8, sk.astype(f16), cuks


def quantize_qkv_for_tilemix(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, BLKQ=128, BLKK=64):
    """tilemix.py:45-107."""
    q8, sq, cuqs, k8, sk, cuks = quantize_qk_for_tilemix(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                                         max_seqlen_k, BLKQ, BLKK)
    v8, sv, cuvs = per_block_int8_single(v, cu_seqlens_k, max_seqlen_k, BLK=BLKK, sm_scale=1.0)
    return q8, sq, cuqs, k8, sk, cuks, v8, sv.astype(f16), cuvs


def tilemix_attention_with_quant(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlens_q, max_seqlens_k,
                                 precision_bitmask, *, block_m=128, block_n=64, block_n_mask=None, BLKQ=128,
                                 BLKK=64, causal=False, sm_scale=None, routing_mode="mixed", scalar_scales=True,
                                 int8_use_fp16_v=False, bias=None, heads=None, q_blocks=None):
    """tilemix.py:1340-1447 for an explicit routing mode ("mixed" / "fp16" / "int8")."""
    mode = {"mixed": ROUTING_MODE_MIXED, "fp16": ROUTING_MODE_FP16, "int8": ROUTING_MODE_INT8}[routing_mode]
    kw = {}
    if mode != ROUTING_MODE_FP16:
        if int8_use_fp16_v:
            q8, sq, cuqs, k8, sk, cuks = quantize_qk_for_tilemix(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlens_q,
                                                                 max_seqlens_k, BLKQ, BLKK)
            kw = dict(q8=q8, sq=sq, cu_qs=cuqs, k8=k8, sk=sk, cu_ks=cuks)
        else:
            q8, sq, cuqs, k8, sk, cuks, v8, sv, cuvs = quantize_qkv_for_tilemix(
                q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlens_q, max_seqlens_k, BLKQ, BLKK)
            kw = dict(q8=q8, sq=sq, cu_qs=cuqs, k8=k8, sk=sk, cu_ks=cuks, v8=v8, sv=sv, cu_vs=cuvs)
    return attn_fwd(q, k, v, cu_seqlens_q, cu_seqlens_k, precision_bitmask, max_seqlen_q=max_seqlens_q,
                    max_seqlen_k=max_seqlens_k, block_m=block_m, block_n=block_n, block_n_mask=block_n_mask,
                    BLKQ=BLKQ, BLKK=BLKK, causal=causal, sm_scale=sm_scale, routing_mode=mode,
                    scalar_scales=scalar_scales, int8_use_fp16_v=int8_use_fp16_v, bias=bias, heads=heads,
                    q_blocks=q_blocks, **kw)


def attention_flops(cu_seqlens_q, heads_q: int, head_dim: int, causal: bool = True) -> float:
    """Algorithmic FLOPs of one call: 4*D*HQ*sum_b T_b(T_b+1)/2 causal (T_b^2 dense)."""
    cu = np.asarray(cu_seqlens_q, dtype=np.int64)
    lens = cu[1:] - cu[:-1]
    pairs = (lens * (lens + 1) // 2) if causal else lens * lens
    return float(4 * head_dim * heads_q * int(pairs.sum()))
