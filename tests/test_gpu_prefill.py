"""GPU parity of the Llama prefill companions (tilemix_b200/csrc/prefill.cu) against the
CPU oracle (oracle/prefill_oracle.py): the RoPE bit for bit (its oracle is pinned to the
reference's own kernel), the RoPE-fused K quantisation bit for bit against the pinned
quantiser and against the library's own quantiser kernel, SiLU-multiply and RMSNorm within
one fp16 ulp (their reference arithmetic, libdevice exp and torch's reduction order, cannot
be reproduced bit for bit on the CPU)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import prefill_oracle as po

# Compared with the CPU oracle / interpreter fixtures: exact numerics.
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_numerics")]

GOLDEN = Path(__file__).resolve().parent / "golden"


def _ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in fp16 units in the last place (monotonic integer view)."""
    def key(x):
        i = x.view(np.uint16).astype(np.int32)
        return np.where(i & 0x8000, 0x8000 - (i & 0x7FFF), 0x8000 + i)
    return np.abs(key(a) - key(b))


@pytest.mark.parametrize("name", ["d64", "d128_b2"])
def test_rotary_matches_reference_fixture(cuda_device, name):
    from tilemix_b200.models.tilemix_llama import rotary_token_major

    f = np.load(GOLDEN / f"interp_rotary_{name}.npz")
    dev = cuda_device
    oq, ok = rotary_token_major(*(torch.from_numpy(f[x]).to(dev) for x in ("q", "k", "cos", "sin")))
    torch.cuda.synchronize()
    assert np.array_equal(oq.transpose(1, 2).cpu().numpy().view(np.uint16), f["oq"].view(np.uint16))
    assert np.array_equal(ok.transpose(1, 2).cpu().numpy().view(np.uint16), f["ok"].view(np.uint16))


@pytest.mark.parametrize("b,hq,hk,t,d,cos_b", [(2, 24, 8, 300, 128, 1), (3, 4, 2, 129, 64, 3)])
def test_rotary_strided_inputs_match_oracle(cuda_device, b, hq, hk, t, d, cos_b):
    """q / k as the attention module produces them: views of one QKV projection output."""
    from tilemix_b200.models.tilemix_llama import rotary_token_major

    g = torch.Generator().manual_seed(7)
    qkv = (torch.randn(b, t, (hq + 2 * hk) * d, generator=g) * 4).half()
    q = qkv[..., : hq * d].view(b, t, hq, d).transpose(1, 2)
    k = qkv[..., hq * d:(hq + hk) * d].view(b, t, hk, d).transpose(1, 2)
    cos = torch.randn(cos_b, t, d, generator=g).half()
    sin = torch.randn(cos_b, t, d, generator=g).half()
    rq, rk = po.rotary_token_major(q.numpy(), k.numpy(), cos.numpy(), sin.numpy())
    dev = cuda_device
    qkv_d = qkv.to(dev)
    qd = qkv_d[..., : hq * d].view(b, t, hq, d).transpose(1, 2)
    kd = qkv_d[..., hq * d:(hq + hk) * d].view(b, t, hk, d).transpose(1, 2)
    oq, ok = rotary_token_major(qd, kd, cos.to(dev), sin.to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(oq.transpose(1, 2).cpu().numpy().view(np.uint16), rq.view(np.uint16))
    assert np.array_equal(ok.transpose(1, 2).cpu().numpy().view(np.uint16), rk.view(np.uint16))


@pytest.mark.parametrize("t,d,blkk", [(300, 128, 64), (257, 64, 128), (64, 128, 64)])
def test_rotary_fused_k_quantisation(cuda_device, t, d, blkk):
    """K8 / scales of the fused pass equal the pinned quantiser on the rotated K and the
    library's own quantiser kernel run on it; the rotated Q / K equal the plain pass."""
    from tilemix_b200.attention.quant_per_block_varlen import per_block_int8_single
    from tilemix_b200.models.tilemix_llama import rotary_token_major, rotary_token_major_quant_k

    b, hq, hk = 2, 6, 2
    g = torch.Generator().manual_seed(11)
    q = (torch.randn(b, hq, t, d, generator=g) * 3).half()
    k = (torch.randn(b, hk, t, d, generator=g) * 3).half()
    k[:, 1, :, 5] *= 40  # an outlier channel in one head
    cos = torch.randn(1, t, d, generator=g).half()
    sin = torch.randn(1, t, d, generator=g).half()
    dev = cuda_device
    args = [x.to(dev) for x in (q, k, cos, sin)]
    oq0, ok0 = rotary_token_major(*args)
    oq, ok, k8, ks = rotary_token_major_quant_k(*args, blkk=blkk)
    torch.cuda.synchronize()
    assert torch.equal(oq0, oq) and torch.equal(ok0, ok)
    ok_np = ok.transpose(1, 2).contiguous().cpu().numpy()
    rk8, rsc = po.quant_rotated_k(ok_np, blk=blkk)
    assert np.array_equal(k8.cpu().numpy(), rk8)
    assert np.array_equal(ks.cpu().numpy().view(np.uint16), rsc.astype(np.float16).view(np.uint16))
    cu = torch.arange(0, (b + 1) * t, t, dtype=torch.int32, device=dev)
    lib8, libsc, _ = per_block_int8_single(ok.transpose(1, 2).reshape(b * t, hk, d), cu, t, BLK=blkk, sm_scale=1.0)
    assert torch.equal(lib8, k8)
    assert np.array_equal(libsc.cpu().numpy().astype(np.float16).view(np.uint16), ks.cpu().numpy().view(np.uint16))


@pytest.mark.parametrize("n", [4096 * 8, 1000 * 3 + 5])
def test_silu_mul_within_one_ulp(cuda_device, n):
    from tilemix_b200.models.tilemix_llama import silu_mul

    g = torch.Generator().manual_seed(3)
    gate = (torch.randn(n, generator=g) * 6).half()
    gate[:4] = torch.tensor([-30.0, 30.0, 0.0, -0.0]).half()
    up = (torch.randn(n, generator=g) * 2).half()
    ref = po.silu_mul(gate.numpy(), up.numpy())
    out = silu_mul(gate.to(cuda_device), up.to(cuda_device))
    torch.cuda.synchronize()
    u = _ulps(out.cpu().numpy(), ref)
    assert u.max() <= 1, int(u.max())
    assert (u > 0).mean() < 1e-3, float((u > 0).mean())


@pytest.mark.parametrize("rows,cols", [(64, 3072), (37, 1000), (5, 4100)])
def test_rms_norm_within_one_ulp(cuda_device, rows, cols):
    from tilemix_b200.models.tilemix_llama import rms_norm

    g = torch.Generator().manual_seed(5)
    x = (torch.randn(rows, cols, generator=g) * 3).half()
    w = (torch.rand(cols, generator=g) * 2).half()
    ref = po.rms_norm(x.numpy(), w.numpy(), 1e-5)
    out = rms_norm(x.to(cuda_device), w.to(cuda_device), 1e-5)
    torch.cuda.synchronize()
    u = _ulps(out.cpu().numpy(), ref)
    assert u.max() <= 1, int(u.max())
