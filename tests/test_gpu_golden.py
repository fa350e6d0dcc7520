"""GPU parity against the reference's own outputs: the fixtures of tests/golden/
were produced by running the reference's Triton kernels (interpreter mode) on
seeded inputs; the CUDA path runs the same inputs through the reference-facing
API and must agree within the north-star tolerance (max-abs 2e-3, mean-abs
2e-4 on fp16 outputs)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.helpers import make_bias, make_qkv

# Compared with the CPU oracle / interpreter fixtures: exact numerics.
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_numerics")]

GOLDEN = Path(__file__).resolve().parent / "golden"
MAX_ABS = 2e-3
MEAN_ABS = 2e-4
NAMES = ["cfg1_sptrans", "cfg1_zero", "cfg1_one", "gqa128_sptrans", "gqa128_bigbird_varlen",
         "cfg1_sptrans_v8", "gqa128_sptrans_v8", "gqa128_sptrans_bias", "cfg1_one_bias_v8"]


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("threshold", ["0", "8", "15"])
def test_attention_matches_reference_fixture(cuda_device, monkeypatch, name, threshold):
    from tilemix_b200.attention.tilemix import device_error_code, tilemix_attention_with_quant

    monkeypatch.setenv("TILEMIX_B200_RESCALE_THRESHOLD", threshold)
    f = np.load(GOLDEN / f"interp_attn_{name}.npz")
    lens = [int(x) for x in f["lens"]]
    hq, hk, d = int(f["hq"]), int(f["hk"]), int(f["d"])
    bm, bn, bnm = int(f["block_m"]), int(f["block_n"]), int(f["block_n_mask"])
    q, k, v, cu = make_qkv(lens, hq, hk, d, seed=int(f["seed"]), outliers=int(f["outliers"]))
    fp16_v = bool(f["int8_use_fp16_v"]) if "int8_use_fp16_v" in f.files else True
    bias_seed = int(f["bias_seed"]) if "bias_seed" in f.files else -1
    T = max(lens)
    pm = torch.from_numpy(f["bitmask"].copy()).view(torch.uint64).to(cuda_device)
    dev = cuda_device
    bias = None if bias_seed < 0 else make_bias(len(lens), hq, T, bias_seed).to(dev)
    out, mode = tilemix_attention_with_quant(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), cu.to(dev), T, T, pm,
                                             block_m=bm, block_n=bn, block_n_mask=bnm, causal=True,
                                             sm_scale=d ** -0.5, routing_mode="mixed",
                                             scalar_scales=(bm == 128 and bn == 64), int8_use_fp16_v=fp16_v,
                                             bias=bias)
    torch.cuda.synchronize()
    assert device_error_code(dev) == 0
    diff = np.abs(out.float().cpu().numpy() - f["out"].astype(np.float32))
    assert diff.max() <= MAX_ABS and diff.mean() <= MEAN_ABS, (float(diff.max()), float(diff.mean()))


def test_varlen_entry_point_matches_packed_call(cuda_device):
    """tilemix_varlen_attention ([B, H, T, D]) equals the packed call on the same data."""
    from tilemix_b200.attention.precision_maps import make_precision_bitmask
    from tilemix_b200.attention.tilemix import tilemix_attention_with_quant
    from tilemix_b200.attention.tilemix_varlen import tilemix_varlen_attention

    B, T, hq, hk, d = 2, 1024, 6, 2, 128
    q, k, v, cu = make_qkv([T] * B, hq, hk, d, seed=4, outliers=4)
    dev = cuda_device
    words = make_precision_bitmask(T, 128, 64, None, 0.5, "sptrans", {"percentage": 0.5}, 64, device=dev)
    pm = words.view(torch.int64).repeat(hk).view(torch.uint64)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    ref, _ = tilemix_attention_with_quant(qd, kd, vd, cu.to(dev), cu.to(dev), T, T, pm, block_m=128, block_n=64,
                                          block_n_mask=64, causal=True, sm_scale=d ** -0.5, routing_mode="mixed",
                                          scalar_scales=True, int8_use_fp16_v=True)
    out = tilemix_varlen_attention(qd.view(B, T, hq, d).permute(0, 2, 1, 3), kd.view(B, T, hk, d).permute(0, 2, 1, 3),
                                   vd.view(B, T, hk, d).permute(0, 2, 1, 3), 128, 64, block_n_mask=64, causal=True,
                                   scale=d ** -0.5, precision_map_all=pm, candidates=[], flat_lengths=[])
    assert out.shape == (B, hq, T, d)
    assert torch.equal(out.permute(0, 2, 1, 3).reshape(B * T, hq, d), ref)
