"""GPU parity of the sm_100a per-block INT8 quantiser: bit-exact codes and scales."""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from tests.helpers import make_qkv

# Compared with the CPU oracle / interpreter fixtures: exact numerics.
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_numerics")]


@pytest.mark.parametrize("lens,h,d,blk", [([512], 4, 64, 128), ([4096, 1000, 1], 8, 128, 64),
                                          ([300, 129], 3, 128, 128), ([64], 1, 64, 256),
                                          ([300, 0, 129], 3, 128, 64)])
def test_quant_bit_exact(cuda_device, lens, h, d, blk):
    from tilemix_b200.attention.quant_per_block_varlen import per_block_int8_single

    q, _, _, cu = make_qkv(lens, h, 1, d, seed=3, outliers=2)
    x8, xs, cus = per_block_int8_single(q.to(cuda_device), cu.to(cuda_device), max(lens), BLK=blk)
    torch.cuda.synchronize()
    r8, rs, rcu = ora.per_block_int8_single(q.numpy(), cu.numpy(), max(lens), BLK=blk)
    assert np.array_equal(cus.cpu().numpy(), rcu)
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(x8.cpu().numpy(), r8)


def test_quant_all_zero_block(cuda_device):
    from tilemix_b200.attention.quant_per_block_varlen import per_block_int8_single

    x = torch.zeros((128, 2, 64), dtype=torch.float16)
    x[:, 1] = 1.0
    cu = torch.tensor([0, 128], dtype=torch.int32)
    x8, xs, _ = per_block_int8_single(x.to(cuda_device), cu.to(cuda_device), 128, BLK=128)
    assert float(xs[0, 0]) == 0.0 and int(x8[:, 0].abs().max()) == 0
    assert int(x8[:, 1].min()) == 127


@pytest.mark.parametrize("blk,sm_scale", [(64, 1.0), (128, 1.0), (64, 0.5), (256, 1.0)])
def test_quant_special_values(cuda_device, blk, sm_scale):
    """A block holding inf quantises to zeros (x / inf is 0, or NaN which truncates to 0), on
    the unit-scale fast path (64 / 128-token blocks) and on the generic kernel (other scales /
    blocks). (NaN inputs are left out: the oracle follows the Triton interpreter, whose numpy
    max propagates NaN into the scale, while GPU max instructions, the reference's included,
    skip it.)"""
    from tilemix_b200.attention.quant_per_block_varlen import per_block_int8_single

    q, _, _, cu = make_qkv([300, 200], 2, 1, 128, seed=9, outliers=1)
    q[70, 1, 3] = float("inf")
    q[210, 0, 9] = -float("inf")
    x8, xs, cus = per_block_int8_single(q.to(cuda_device), cu.to(cuda_device), 300, BLK=blk, sm_scale=sm_scale)
    torch.cuda.synchronize()
    r8, rs, rcu = ora.per_block_int8_single(q.numpy(), cu.numpy(), 300, BLK=blk, sm_scale=sm_scale)
    assert np.array_equal(cus.cpu().numpy(), rcu)
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(x8.cpu().numpy(), r8)


@pytest.mark.parametrize("lens,h,d,blk", [([4096, 1000, 1], 8, 128, 64), ([300, 129], 3, 128, 128),
                                          ([512], 4, 64, 64)])
def test_quant_fp16_codes_equal_int8_codes(cuda_device, lens, h, d, blk):
    """tm_quant_per_block_int8_f16 (the V operand of the paired kernel's INT8-V path): the
    same scales as the int8 quantiser, and codes whose fp16 values equal the int8 codes; the
    int8 output written alongside is unchanged."""
    from tilemix_b200.attention.quant_per_block_varlen import per_block_int8_single
    from tilemix_b200.attention.tilemix import _quantize_k, _quantize_v_f16

    x, _, _, cu = make_qkv(lens, h, 1, d, seed=11, outliers=2)
    x, cu = x.to(cuda_device), cu.to(cuda_device)
    k8, ks, cuks = _quantize_k(x, cu, max(lens), blk)
    v16, vs, cuvs = _quantize_v_f16(x, cu, max(lens), blk)
    torch.cuda.synchronize()
    rows = int(cuks[-1])
    assert torch.equal(cuks, cuvs)
    assert torch.equal(ks[:rows].view(torch.int16), vs[:rows].view(torch.int16))
    assert v16.dtype == torch.float16
    assert torch.equal(v16.float(), k8.float())
    x8, _, _ = per_block_int8_single(x, cu, max(lens), BLK=blk)
    assert torch.equal(x8, k8)
