"""GPU parity at the full headline configuration (8 x 4096 tokens, 24 q / 8 kv
heads, head_dim 128, causal, tiles 128/64/64): long key loops are where the
multi-warp pipelines of the sm_100a kernels run furthest ahead of each other,
so these cases check the device error word (no bounded wait expired) and the
output against the CPU oracle on a sample of heads and query blocks.

These cases run in exact numerics (the oracle's arithmetic). With N(0, 1)
inputs the north-star bound (max-abs 2e-3, mean-abs 2e-4) holds everywhere.
With the benchmark's outlier channels (4 per head scaled x20 on Q and K)
scores reach ~30-60 in log2 units, where one fp16 step is 1/32-1/16: an
FP16-routed score whose exact value lies within float32 rounding error of an
fp16 rounding midpoint rounds differently under the oracle's summation order
(numpy, sequential float32) than under the tensor core's, and a softmax
weight near an fp16 midpoint rounds differently under the hardware exp2 than
under numpy's; when such a key dominates its row the output moves by up to
~1e-2. (Worked case: a score whose exact value is 32.484373 lies 2e-6 below
the fp16 midpoint 32.484375; sequential float32 summation lands above it and
rounds to 32.5, the tensor core to the correctly rounded 32.46875.) The
reference's own Triton kernels run on a B200 depart from the same oracle far
more on these rows (measured on this exact sample: max 8.7e-2, mean 7.8e-4,
10.5 % of elements over 2e-3), because their FP16 QK^T accumulates in fp16;
the default numerics reproduce that run and are checked against it directly
(tests/test_gpu_reference_triton.py). For these inputs this test bounds the
mean error by 2e-4, the share of elements over 2e-3 by 0.05 % and the largest
error by 3e-2.
"""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from oracle.precision_maps_oracle import make_precision_bitmask as oracle_map
from tests.helpers import make_qkv

# Compared with the CPU oracle / interpreter fixtures: exact numerics.
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_numerics")]

MAX_ABS = 2e-3
MEAN_ABS = 2e-4
B, T, HQ, HK, D = 8, 4096, 24, 8, 128
HEADS, BLOCKS = [0, 13, 23], [0, 7, 30, 31]


def _run(dev, pattern, outliers):
    from tilemix_b200.attention.precision_maps import make_precision_bitmask
    from tilemix_b200.attention.tilemix import device_error_code, tilemix_attention_with_quant

    q, k, v, cu = make_qkv([T] * B, HQ, HK, D, seed=0, outliers=outliers)
    words = make_precision_bitmask(T, 128, 64, None, 0.5, pattern, {"percentage": 0.5}, 64, device=dev)
    ref_words = oracle_map(T, 128, 64, None, 0.5, pattern, {"percentage": 0.5}, 64)
    assert np.array_equal(words.view(torch.int64).cpu().numpy().view(np.uint64), ref_words)
    pm = words.view(torch.int64).repeat(HK).view(torch.uint64)
    out, _ = tilemix_attention_with_quant(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), cu.to(dev), T, T, pm,
                                          block_m=128, block_n=64, block_n_mask=64, causal=True,
                                          routing_mode="mixed", scalar_scales=True, int8_use_fp16_v=True)
    torch.cuda.synchronize()
    assert device_error_code(dev) == 0
    ref = ora.tilemix_attention_with_quant(q.numpy(), k.numpy(), v.numpy(), cu.numpy(), cu.numpy(), T, T,
                                           np.tile(ref_words, HK), block_m=128, block_n=64, block_n_mask=64,
                                           causal=True, routing_mode="mixed", scalar_scales=True,
                                           int8_use_fp16_v=True, heads=HEADS, q_blocks=BLOCKS)
    rows = np.concatenate([np.arange(b * T + m * 128, b * T + (m + 1) * 128) for b in range(B) for m in BLOCKS])
    got = out.float().cpu().numpy()[rows][:, HEADS]
    diff = np.abs(got - ref[rows][:, HEADS].astype(np.float32))
    return q.numpy(), k.numpy(), ref_words, rows, diff


@pytest.mark.parametrize("pattern", ["sptrans", "zero", "one"])
def test_headline_config_within_bound(cuda_device, pattern):
    _, _, _, _, diff = _run(cuda_device, pattern, outliers=0)
    assert diff.max() <= MAX_ABS and diff.mean() <= MEAN_ABS, (float(diff.max()), float(diff.mean()))


def test_headline_config_with_outliers(cuda_device):
    q, k, words, rows, diff = _run(cuda_device, "sptrans", outliers=4)
    assert diff.mean() <= MEAN_ABS, float(diff.mean())
    assert diff.max() <= 3e-2, float(diff.max())
    over = int((diff > MAX_ABS).sum())
    assert over <= 5e-4 * diff.size, (over, diff.size)


def test_long_sequence_chunked_item_order(cuda_device):
    """One 25,600-token sequence with GQA group 3 gives each (sequence, KV head) unit 300
    work-item levels, enough for the paired kernel to deal one unit's levels per round of the
    grid (chunked order); sampled query blocks of all heads match the CPU oracle within the
    north-star bound. The mask groups are 7 key tiles wide at this length."""
    from tilemix_b200.attention.precision_maps import make_precision_bitmask
    from tilemix_b200.attention.tilemix import device_error_code, tilemix_attention_with_quant
    from tilemix_b200.models._attention_base import pick_mask_block_n

    dev = cuda_device
    T, hq, hk = 25600, 3, 1
    bnm = pick_mask_block_n(T, 64)
    q, k, v, cu = make_qkv([T], hq, hk, D, seed=11)
    words = make_precision_bitmask(T, 128, bnm, None, 0.5, "sptrans", {"percentage": 0.5}, 64, device=dev)
    out, _ = tilemix_attention_with_quant(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), cu.to(dev), T, T, words,
                                          block_m=128, block_n=64, block_n_mask=bnm, causal=True,
                                          routing_mode="mixed", scalar_scales=True, int8_use_fp16_v=True)
    torch.cuda.synchronize()
    assert device_error_code(dev) == 0
    blocks = [0, 1, 99, 198, 199]
    ref = ora.tilemix_attention_with_quant(q.numpy(), k.numpy(), v.numpy(), cu.numpy(), cu.numpy(), T, T,
                                           words.view(torch.int64).cpu().numpy().view(np.uint64), block_m=128,
                                           block_n=64, block_n_mask=bnm, causal=True, routing_mode="mixed",
                                           scalar_scales=True, int8_use_fp16_v=True, heads=list(range(hq)),
                                           q_blocks=blocks)
    rows = np.concatenate([np.arange(m * 128, (m + 1) * 128) for m in blocks])
    diff = np.abs(out.float().cpu().numpy()[rows] - ref[rows].astype(np.float32))
    assert diff.max() <= MAX_ABS and diff.mean() <= MEAN_ABS, (float(diff.max()), float(diff.mean()))
