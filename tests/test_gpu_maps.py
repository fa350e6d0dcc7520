"""GPU parity of the routing-map kernel ``tm_build_precision_map``: bit-exact
words against the reference's own outputs (tests/golden/maps.json, made by
running the reference's make_precision_bitmask) and against the CPU oracle on
cases outside the fixture grid."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.precision_maps_oracle import make_precision_bitmask as oracle_map

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _words(t: torch.Tensor) -> str:
    return " ".join(format(int(x), "x") for x in t.cpu().view(torch.int64).numpy().view(np.uint64).tolist())


def test_maps_match_reference_fixtures(cuda_device):
    from tilemix_b200.attention.precision_maps import make_precision_bitmask

    cases = json.loads((GOLDEN / "maps.json").read_text())["cases"]
    bad = []
    for c in cases:
        got = make_precision_bitmask(c["T"], c["bm"], c["bnm"], None, c["pct"], c["pattern"], c["params"], c["cbn"],
                                     device=cuda_device)
        if _words(got) != c["words"]:
            bad.append((c["T"], c["bm"], c["bnm"], c["pattern"], c["pct"], c["params"]))
    assert not bad, f"{len(bad)} of {len(cases)} maps differ, first: {bad[:5]}"


@pytest.mark.parametrize("T,bm,bnm,cbn", [(3000, 64, 64, 64), (12345, 128, 256, 64), (777, 64, 128, 128),
                                          (40000, 128, 640, 64)])
@pytest.mark.parametrize("pattern", ["band", "global", "row_rand", "align_sparse", "bigbird", "sptrans"])
def test_maps_match_oracle_off_grid(cuda_device, T, bm, bnm, cbn, pattern):
    from tilemix_b200.attention.precision_maps import make_precision_bitmask

    for pct in (0.1, 0.37, 0.5, 0.9):
        params = {"percentage": pct}
        if pattern == "bigbird":
            params.update(num_global_block=1, num_rand_block=4)
        if pattern == "global":
            params.update(key_pos=[5, T // 2, T - 1, 10 * T])
        got = make_precision_bitmask(T, bm, bnm, None, pct, pattern, params, cbn, device=cuda_device)
        ref = oracle_map(T, bm, bnm, None, pct, pattern, params, cbn)
        assert np.array_equal(got.cpu().view(torch.int64).numpy().view(np.uint64), ref), (pct, params)


def test_map_is_asynchronous_and_leaves_global_rng(cuda_device):
    from tilemix_b200.attention.precision_maps import make_precision_bitmask

    torch.manual_seed(7)
    before = torch.get_rng_state()
    words = make_precision_bitmask(4096, 128, 64, None, 0.5, "row_rand", {"percentage": 0.5}, 64,
                                   device=cuda_device, check_retarget=False)
    torch.cuda.synchronize()
    assert torch.equal(before, torch.get_rng_state())
    assert words.dtype == torch.uint64 and words.device.type == "cuda" and words.numel() == 32
