"""CPU tests: the oracle against the reference's golden fixtures (tests/golden/).

The fixtures were produced by running the reference itself (see
tests/golden/make_golden.py); these tests pin the oracle bit for bit, so the
GPU parity tests that compare the CUDA path with the oracle are comparisons
with the reference.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from oracle.mt19937 import MT19937, randperm
from oracle.precision_maps_oracle import make_precision_bitmask
from tests.helpers import make_bias, make_qkv

GOLDEN = Path(__file__).resolve().parent / "golden"


def _maps():
    return json.loads((GOLDEN / "maps.json").read_text())["cases"]


@pytest.mark.parametrize("seed", [0, 42, 12345])
def test_randperm_matches_torch(seed):
    torch.manual_seed(seed)
    gen = MT19937(seed)
    for n in [1, 2, 3, 17, 64, 528, 4096, 65536]:
        assert np.array_equal(torch.randperm(n).numpy(), randperm(n, gen)), n


def test_map_oracle_matches_reference_fixtures():
    cases = _maps()
    assert len(cases) > 400
    for c in cases:
        if "error" in c:
            with pytest.raises(Exception):
                make_precision_bitmask(c["T"], c["bm"], c["bnm"], None, c["pct"], c["pattern"], c["params"], c["cbn"])
            continue
        words = make_precision_bitmask(c["T"], c["bm"], c["bnm"], None, c["pct"], c["pattern"], c["params"], c["cbn"])
        got = " ".join(format(int(x), "x") for x in words.tolist())
        assert got == c["words"], (c["T"], c["pattern"], c["pct"], c["params"])


def test_map_oracle_validation_errors():
    with pytest.raises(ValueError):
        make_precision_bitmask(8192, 128, 64, None, 0.5, "sptrans", {"percentage": 0.5}, 64)  # 128 mask groups
    with pytest.raises(ValueError):
        make_precision_bitmask(4096, 128, 96, None, 0.5, "band", {"percentage": 0.5}, 64)  # 96 % 64
    with pytest.raises(ValueError):
        make_precision_bitmask(4096, 128, 64, None, 0.5, "band", None, 64)  # needs params or token mask


@pytest.mark.parametrize("name,blk", [("q128", 128), ("k64", 64)])
def test_quant_oracle_matches_interpreter(name, blk):
    f = np.load(GOLDEN / f"interp_quant_{name}.npz")
    q, k, _, cu = make_qkv([512, 300, 129], 3, 2, 128, seed=11, outliers=2)
    x = (q if name.startswith("q") else k).numpy()
    x8, xs, cus = ora.per_block_int8_single(x, cu.numpy(), 512, BLK=blk)
    assert np.array_equal(x8, f["x8"])
    assert np.array_equal(xs.view(np.uint32), f["scale"].view(np.uint32))
    assert np.array_equal(cus, f["cu_scale"])


ATTN_FIXTURES = ["cfg1_sptrans", "cfg1_zero", "cfg1_one", "gqa128_sptrans", "gqa128_bigbird_varlen",
                 "cfg1_sptrans_v8", "gqa128_sptrans_v8", "gqa128_sptrans_bias", "cfg1_one_bias_v8"]


def fixture_options(f):
    """(int8_use_fp16_v, bias seed or None) of an attention fixture (older fixtures: FP16 V, no bias)."""
    fp16_v = bool(f["int8_use_fp16_v"]) if "int8_use_fp16_v" in f.files else True
    bias_seed = int(f["bias_seed"]) if "bias_seed" in f.files else -1
    return fp16_v, (None if bias_seed < 0 else bias_seed)


@pytest.mark.parametrize("name", ATTN_FIXTURES)
def test_attention_oracle_matches_interpreter(name):
    f = np.load(GOLDEN / f"interp_attn_{name}.npz")
    lens = [int(x) for x in f["lens"]]
    hq, hk, d = int(f["hq"]), int(f["hk"]), int(f["d"])
    bm, bn, bnm = int(f["block_m"]), int(f["block_n"]), int(f["block_n_mask"])
    q, k, v, cu = make_qkv(lens, hq, hk, d, seed=int(f["seed"]), outliers=int(f["outliers"]))
    fp16_v, bias_seed = fixture_options(f)
    T = max(lens)
    bias = None if bias_seed is None else make_bias(len(lens), hq, T, bias_seed).numpy()
    out = ora.tilemix_attention_with_quant(
        q.numpy(), k.numpy(), v.numpy(), cu.numpy(), cu.numpy(), T, T, f["bitmask"].view(np.uint64),
        block_m=bm, block_n=bn, block_n_mask=bnm, causal=True, sm_scale=d ** -0.5, routing_mode="mixed",
        scalar_scales=(bm == 128 and bn == 64), int8_use_fp16_v=fp16_v, bias=bias)
    assert np.array_equal(out.view(np.uint16), f["out"].view(np.uint16))


def test_attention_flops_formula():
    cu = np.array([0, 4096] + [4096 * i for i in range(2, 9)])
    assert ora.attention_flops(cu, 24, 128) == pytest.approx(8.248e11, rel=1e-3)


@pytest.mark.parametrize("name", ["d64", "d128_b2"])
def test_rotary_oracle_matches_reference(name):
    """The prefill RoPE restatement equals the reference's Triton kernel (interpreter run)."""
    from oracle import prefill_oracle as po

    f = np.load(GOLDEN / f"interp_rotary_{name}.npz")
    oq, ok = po.rotary_token_major(f["q"], f["k"], f["cos"], f["sin"])
    assert np.array_equal(oq.view(np.uint16), f["oq"].view(np.uint16))
    assert np.array_equal(ok.view(np.uint16), f["ok"].view(np.uint16))
