"""CPU restatement of the reference's Llama prefill companions (test infrastructure).

Only ``tests/`` and ``__graft_entry__.smoke()`` use this module, as the checker
of the CUDA kernels in ``tilemix_b200/csrc/prefill.cu``; the library never
calls it.

* ``rotary_token_major`` follows ``_rotary`` / ``rotary_token_major``
  (models/tilemix_llama.py:797-822): per element, ``fp16(x * cos)`` plus
  ``fp16(x[(d + D/2) % D] * sign * sin)`` (sign -1 on the first half), the sum
  formed in fp32 and stored as fp16, token-major ``[B, T, H, D]``. Pinned bit
  for bit against the reference kernel run by the Triton interpreter
  (``tests/golden/interp_rotary_*.npz``).
* ``silu_mul`` follows ``_silu_mul`` (:851-857): ``fp16(gate / (1 + exp(-gate)))``
  with a correctly rounded fp32 division, times ``up`` in fp32, stored as fp16.
  The reference's ``libdevice.exp`` cannot run in the Triton interpreter, so
  this restatement (numpy's float32 exp) is parity unpinned: the tests bound the
  CUDA kernel by one fp16 ulp against it.
* ``rms_norm`` follows ``PrefillRMSNorm`` (:757-771, the tail :757-760): fp32
  mean of x^2 over the row, ``fp16(x * rsqrt(var + eps))``, times the fp16
  weight rounded to fp16. The reference's squared-mean is a CUDA-only extension
  (its fp32 reduction order is torch's); parity unpinned, bounded by one fp16
  ulp in the tests.
* ``quant_rotated_k`` is the per-block INT8 quantisation of the rotated K
  (quant_per_block_varlen.py:6-45 with sm_scale 1) that the fused rotary kernel
  performs, by the attention oracle's pinned quantiser.
"""
from __future__ import annotations

import numpy as np

f16 = np.float16
f32 = np.float32


def rotary_token_major(q, k, cos, sin):
    """q [B, HQ, T, D], k [B, HK, T, D], cos/sin [1 or B, T, D] (fp16 numpy) ->
    (oq [B, T, HQ, D], ok [B, T, HK, D]) fp16."""
    D = q.shape[-1]
    half = D // 2
    sign = np.where(np.arange(D) < half, f32(-1.0), f32(1.0))

    def rot(x):
        c = cos.astype(f32)[:, None]  # [1|B, 1, T, D]
        s = sin.astype(f32)[:, None]
        xr = np.concatenate([x[..., half:], x[..., :half]], axis=-1)
        a = (x.astype(f32) * c).astype(f16)
        b = ((xr.astype(f32) * sign) * s).astype(f16)
        return (a.astype(f32) + b.astype(f32)).astype(f16).transpose(0, 2, 1, 3)

    return rot(q), rot(k)


def silu_mul(gate, up):
    g = gate.astype(f32)
    with np.errstate(over="ignore"):
        act = (g / (f32(1.0) + np.exp(-g))).astype(f16)
    return (act.astype(f32) * up.astype(f32)).astype(f16)


def rms_norm(x, weight, eps):
    x32 = x.astype(f32)
    var = (x32.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(f32)
    h = (x32 * (f32(1.0) / np.sqrt(var + f32(eps)))).astype(f16)
    return (weight.astype(f32) * h.astype(f32)).astype(f16)


def quant_rotated_k(ok, blk=64):
    """ok [B, T, HK, D] fp16 (equal-length sequences) -> (k8 [B*T, HK, D] int8,
    scale [B * ceil(T/blk), HK] fp32): the pinned per-block quantiser of the
    attention oracle applied to the packed rotated K."""
    from oracle.attention_oracle import per_block_int8_single

    B, T, HK, D = ok.shape
    cu = np.arange(0, (B + 1) * T, T, dtype=np.int32)
    k8, scale, _ = per_block_int8_single(ok.reshape(B * T, HK, D), cu, T, BLK=blk, sm_scale=1.0)
    return k8, scale
