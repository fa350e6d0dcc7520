"""GPU parity of the sm_100a attention kernel against the CPU oracle.

Tolerance: max-abs 2e-3 and mean-abs 2e-4 on fp16
outputs, per case. The kernel is driven through the reference-facing host API
(which calls the C ABI ``tm_attn_fwd_ex``).
"""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from tests.helpers import err_stats, make_bias, make_qkv, random_bitmask

# Compared with the CPU oracle / interpreter fixtures: exact numerics.
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_numerics")]

MAX_ABS = 2e-3
MEAN_ABS = 2e-4


def _run_case(lens, hq, hk, d, block_m, block_n=64, block_n_mask=64, mode="mixed", causal=True, seed=0,
              outliers=0, threshold=0.0, bits_seed=1, fp16_v=True, bias_seed=None, return_diff=False, blkk=64):
    from tilemix_b200.attention import tilemix as tmx

    q, k, v, cu = make_qkv(lens, hq, hk, d, seed=seed, outliers=outliers)
    T = max(lens)
    rows = hk * ((T + block_m - 1) // block_m)
    bm = random_bitmask(rows, seed=bits_seed)
    scalar = block_m == 128 and block_n == blkk
    bias = None if bias_seed is None else make_bias(len(lens), hq, T, bias_seed)
    ref = ora.tilemix_attention_with_quant(
        q.numpy(), k.numpy(), v.numpy(), cu.numpy(), cu.numpy(), T, T, bm.numpy().view(np.uint64),
        block_m=block_m, block_n=block_n, block_n_mask=block_n_mask, BLKK=blkk, causal=causal, routing_mode=mode,
        scalar_scales=scalar, int8_use_fp16_v=fp16_v, bias=None if bias is None else bias.numpy())
    dev = torch.device("cuda", 0)
    out = tmx._attention_forward(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), cu.to(dev), T, T, bm.to(dev),
                                 block_m=block_m, block_n=block_n, block_n_mask=block_n_mask, BLKQ=128, BLKK=blkk,
                                 causal=causal, sm_scale=None, mode=mode, scalar_scales=scalar,
                                 int8_use_fp16_v=fp16_v, threshold=threshold,
                                 bias=None if bias is None else bias.to(dev))
    torch.cuda.synchronize()
    assert tmx.device_error_code(dev) == 0
    if return_diff:
        return np.abs(out.float().cpu().numpy() - np.asarray(ref, dtype=np.float32))
    return err_stats(out, ref)


CASES = [
    # (lens, hq, hk, d, block_m, block_n_mask, mode)
    ([512], 4, 4, 64, 64, 64, "mixed"),          # BASELINE config 1 shapes
    ([512], 4, 4, 64, 64, 64, "fp16"),
    ([512], 4, 4, 64, 64, 64, "int8"),
    ([1024, 1024], 6, 2, 128, 128, 64, "mixed"),  # GQA, config-2 head shapes
    ([1024], 3, 1, 128, 128, 64, "fp16"),
    ([1024], 3, 1, 128, 128, 64, "int8"),
    ([300, 700, 129], 4, 2, 128, 128, 128, "mixed"),  # varlen, mask group of 2 tiles
    ([777, 64, 513], 2, 1, 64, 64, 64, "mixed"),
    ([896, 333], 3, 1, 128, 128, 64, "mixed"),    # GQA group 3, 21 tiles: one item holds a single tile
    ([640, 200], 5, 5, 128, 128, 64, "mixed"),    # MHA (group 1): items of consecutive query blocks
    ([520], 8, 2, 128, 128, 64, "mixed"),         # group 4: two head pairs per query block
]


@pytest.mark.parametrize("lens,hq,hk,d,block_m,bnm,mode", CASES)
@pytest.mark.parametrize("threshold", [0.0, 8.0, 15.0])
def test_attention_matches_oracle(cuda_device, lens, hq, hk, d, block_m, bnm, mode, threshold):
    mx, mean = _run_case(lens, hq, hk, d, block_m, 64, bnm, mode, threshold=threshold)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_attention_outlier_channels(cuda_device):
    """Config-2 style inputs: 4 fixed outlier channels per head scaled x20. Rows dominated by
    a key whose score lies at an fp16 rounding midpoint can move by ~1e-2 against the oracle
    (test_gpu_attention_large.py explains the two rounding cases; the reference's own GPU run
    departs from the oracle further), so the bound is the mean, the share of elements over
    2e-3 and the largest error."""
    diff = _run_case([1024], 3, 1, 128, 128, mode="mixed", outliers=4, threshold=0.0, return_diff=True)
    assert diff.mean() <= MEAN_ABS, float(diff.mean())
    assert diff.max() <= 3e-2, float(diff.max())
    assert int((diff > MAX_ABS).sum()) <= 5e-4 * diff.size


def test_attention_non_causal(cuda_device):
    mx, mean = _run_case([640], 4, 2, 128, 128, mode="mixed", causal=False)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


# The INT8-V PV path (int8_use_fp16_v=False, the API's default): INT8-routed
# tiles multiply fp16(p * sv) by the int8 V codes. block_m 64 with a random map
# routes the two 64-row halves of a 128-row tile differently (two PVs).
# Head_dim 128 / block_m 128 calls run on the paired kernel, whose V producer
# loads V and / or the fp16 V codes per key tile as the item's two tiles route it.
V8_CASES = [
    ([1024, 640], 6, 2, 128, 128, 64, "mixed"),
    ([1024], 3, 1, 128, 128, 64, "int8"),
    ([896, 333], 3, 1, 128, 128, 64, "mixed"),       # group 3: cross-block pairs route key tiles differently
    ([300, 700, 129], 4, 2, 128, 128, 128, "mixed"),  # varlen, mask group of 2 tiles
    ([640, 200], 5, 5, 128, 128, 64, "mixed"),       # MHA: items of consecutive query blocks
    ([777, 64, 513], 2, 1, 64, 64, 64, "mixed"),
    ([512], 4, 4, 64, 64, 128, "mixed"),
]


@pytest.mark.parametrize("lens,hq,hk,d,block_m,bnm,mode", V8_CASES)
@pytest.mark.parametrize("threshold", [0.0, 8.0, 15.0])
def test_attention_int8_v_path_matches_oracle(cuda_device, lens, hq, hk, d, block_m, bnm, mode, threshold):
    mx, mean = _run_case(lens, hq, hk, d, block_m, 64, bnm, mode, threshold=threshold, fp16_v=False, seed=3)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.parametrize("fp16_v", [True, False])
def test_attention_blkk_128_matches_oracle(cuda_device, fp16_v):
    """K (and V) scale blocks of 128 keys: two 64-key tiles per scale row, tracked by the
    paired kernel's step loop (per-key scale vectors in the reference, scalar_scales off)."""
    mx, mean = _run_case([1024, 640], 6, 2, 128, 128, 64, 64, "mixed", fp16_v=fp16_v, seed=4, blkk=128)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_attention_int8_v_general_kernel_matches_oracle(cuda_device, monkeypatch):
    """The general kernel's INT8-V path (int8 V codes) at the paired kernel's shape."""
    monkeypatch.setenv("TILEMIX_B200_KERNEL", "general")
    mx, mean = _run_case([1024, 640], 6, 2, 128, 128, 64, 64, "mixed", fp16_v=False, seed=3)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


BIAS_CASES = [
    # (lens, hq, hk, d, block_m, mode, fp16_v)
    ([512, 300], 4, 2, 128, 128, "mixed", True),
    ([640], 3, 1, 128, 128, "fp16", True),
    ([300, 257], 4, 4, 64, 64, "mixed", False),
]


@pytest.mark.parametrize("lens,hq,hk,d,block_m,mode,fp16_v", BIAS_CASES)
def test_attention_bias_matches_oracle(cuda_device, lens, hq, hk, d, block_m, mode, fp16_v):
    """A bias of 2 * N(0, 1) widens the logits, so softmax rows are peaked, and
    a score whose exact value sits within float32 summation error of an fp16
    midpoint can round to either side. Worked case (lens [640], head 1, row 26,
    key 17): exact score 3.954101833, midpoint 3.9541015625 (2.7e-7 apart, one
    fp32 ulp); the CPU's sum rounds up to 3.955078, the tensor core's down to
    3.953125; adding the bias term 4.12890625 then gives 8.0859 against a tie
    at 8.08203 that rounds to even (8.0781), one fp16 ulp of the logit, and the
    row (three near-equal top weights) moves by 3.8e-3. The bound is therefore
    the statistical one of the outlier-channel tests: mean <= 2e-4, at most
    0.05 % of the elements over 2e-3, none over 3e-2."""
    diff = _run_case(lens, hq, hk, d, block_m, 64, 64, mode, fp16_v=fp16_v, bias_seed=5, seed=2, return_diff=True)
    assert diff.mean() <= MEAN_ABS, float(diff.mean())
    assert diff.max() <= 3e-2, float(diff.max())
    assert int((diff > MAX_ABS).sum()) <= 5e-4 * diff.size, (int((diff > MAX_ABS).sum()), diff.size)


@pytest.mark.parametrize("chunk,ring", [(1, 2), (2, 3), (4, 2)])
def test_from_host_entry_point_matches_device_call(cuda_device, chunk, ring):
    """Streaming sequences from pinned host memory gives the device call's output bit for bit."""
    from tilemix_b200.attention.precision_maps import make_precision_bitmask
    from tilemix_b200.attention.tilemix_varlen import tilemix_varlen_attention, tilemix_varlen_attention_from_host

    B, T, hq, hk, d = 3, 1024, 6, 2, 128
    q, k, v, _ = make_qkv([T] * B, hq, hk, d, seed=8, outliers=2)
    dev = cuda_device
    words = make_precision_bitmask(T, 128, 64, None, 0.5, "sptrans", {"percentage": 0.5}, 64, device=dev)
    pm = words.view(torch.int64).repeat(hk).view(torch.uint64)
    ref = tilemix_varlen_attention(*(x.to(dev).view(B, T, -1, d).permute(0, 2, 1, 3) for x in (q, k, v)), 128, 64,
                                   block_n_mask=64, causal=True, scale=d ** -0.5, precision_map_all=pm,
                                   candidates=[], flat_lengths=[])
    out = torch.empty((B * T, hq, d), dtype=torch.float16).pin_memory()
    tilemix_varlen_attention_from_host(q.pin_memory(), k.pin_memory(), v.pin_memory(), out, T, 128, 64,
                                       block_n_mask=64, causal=True, scale=d ** -0.5, precision_map_all=pm,
                                       device=dev, chunk_seqs=chunk, ring=ring)
    torch.cuda.synchronize()
    assert torch.equal(out, ref.permute(0, 2, 1, 3).reshape(B * T, hq, d).cpu())


@pytest.mark.parametrize("fp16_v,mode", [(True, "mixed"), (False, "mixed"), (False, "auto")])
def test_launch_prequantized_matches_oracle(cuda_device, fp16_v, mode):
    """launch_prequantized (tilemix.py:1132-1336) on codes from quantize_qkv_for_tilemix: the
    general kernel's prequantised-Q path, INT8-V from the int8 V codes, and the routing mode
    returned as the reference does ("auto" classifies the map)."""
    from tilemix_b200.attention.tilemix import launch_prequantized, quantize_qkv_for_tilemix

    lens, hq, hk, d = [640, 300, 512], 4, 2, 128
    T = max(lens)
    q, k, v, cu = make_qkv(lens, hq, hk, d, seed=6)
    bm = random_bitmask(hk * ((T + 127) // 128), seed=3)
    ref = ora.tilemix_attention_with_quant(
        q.numpy(), k.numpy(), v.numpy(), cu.numpy(), cu.numpy(), T, T, bm.numpy().view(np.uint64), block_m=128,
        block_n=64, block_n_mask=64, causal=True, routing_mode="mixed", scalar_scales=False,
        int8_use_fp16_v=fp16_v)
    dev = cuda_device
    qd, kd, vd, cud = q.to(dev), k.to(dev), v.to(dev), cu.to(dev)
    q8, sq, cuq, k8, sk, cuk, v8, sv, cuv = quantize_qkv_for_tilemix(qd, kd, vd, cud, cud, T, T, BLKQ=128, BLKK=64)
    out, got_mode = launch_prequantized(qd, kd, vd, cud, cud, T, T, bm.to(dev), q8=q8, k8=k8, v8=v8, sQ_blocks=sq,
                                        sK_blocks=sk, sV_blocks=sv, cu_q_scale=cuq, cu_k_scale=cuk, cu_v_scale=cuv,
                                        block_m=128, block_n=64, block_n_mask=64, BLKQ=128, BLKK=64, causal=True,
                                        routing_mode=mode, scalar_scales=False, int8_use_fp16_v=fp16_v)
    torch.cuda.synchronize()
    assert got_mode == "mixed"
    mx, mean = err_stats(out, ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.parametrize("lens,d,block_m,fp16_v", [
    ([512, 0, 300], 128, 128, True),      # paired kernel: the empty sequence's units are skipped
    ([512, 0, 300], 128, 128, False),     # paired kernel, INT8-V
    ([200, 0, 0, 130], 64, 64, False),    # general kernel
])
def test_zero_length_sequences_match_oracle(cuda_device, lens, d, block_m, fp16_v):
    """Empty sequences inside a varlen batch (cu_seqlens with equal neighbours): no rows,
    no K scale blocks, and the other sequences' outputs as the oracle's."""
    mx, mean = _run_case(lens, 4, 2, d, block_m, 64, 64, "mixed", fp16_v=fp16_v, seed=2)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
