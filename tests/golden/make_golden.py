"""Generate the golden fixtures of tests/golden/ by running the reference itself.

Run in the build container, where the reference sources are mounted:

    python tests/golden/make_golden.py /path/to/reference

* ``maps.json``   — exact ``uint64`` row words of the reference's
  ``make_precision_bitmask`` (attention/precision_maps.py:404-636) over a grid
  of sequence lengths, block sizes, patterns and INT8 percentages, using the
  block-size policy of the model integration (models/tilemix_llama.py:46-49,
  :143-175). Cases where the reference raises record the exception type.
* ``interp_*.npz`` — outputs of the reference's Triton kernels run by the
  Triton interpreter (``TRITON_INTERPRET=1``) on the CPU: the per-block INT8
  quantiser (attention/triton/quant_per_block_varlen.py) and
  ``tilemix_attention_with_quant`` (attention/triton/tilemix.py:1340). The two
  CUDA-only host guards of the reference (``q.is_cuda`` at tilemix.py:1167 and
  ``torch.cuda.get_device_capability`` at :1277) are bypassed in this process
  only, and one autotune configuration is forced, so the kernels run
  unmodified on the CPU. Inputs are regenerated from their seeds by the tests;
  each fixture stores a checksum of its inputs.

The tests never import the reference; they read these files.
"""
from __future__ import annotations

import hashlib
import inspect
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.helpers import make_bias, make_qkv  # noqa: E402

PATTERNS = ["zero", "one", "band", "global", "row_rand", "align_sparse", "bigbird", "sptrans"]
PERCENTS = [0.0, 0.25, 0.5, 0.75, 1.0]


def pick_mask_block_n(seqlen: int, compute_block_n: int) -> int:
    min_mask_bn = (seqlen + 63) // 64
    return ((max(min_mask_bn, compute_block_n) + compute_block_n - 1) // compute_block_n) * compute_block_n


def map_cases():
    cases = []
    for T in [17, 100, 512, 1000, 2048, 4095, 4096, 5000, 8192, 16384, 32768, 65536]:
        bm = 128 if T >= 4096 else 64
        bn = 64
        bnm = pick_mask_block_n(T, bn)
        for pat in PATTERNS:
            for pct in (PERCENTS if T <= 16384 else [0.5]):
                cases.append(dict(T=T, bm=bm, bnm=bnm, cbn=bn, pattern=pat, pct=pct, params={"percentage": pct}))
    # explicit pattern parameters and other block shapes
    extra = [
        dict(T=4096, bm=128, bnm=64, cbn=64, pattern="sptrans", pct=0.5,
             params={"percentage": 0.5, "stride": 128, "c": 32}),
        dict(T=4096, bm=128, bnm=128, cbn=64, pattern="sptrans", pct=0.5, params={"percentage": 0.5, "stride": 256}),
        dict(T=2048, bm=64, bnm=128, cbn=128, pattern="bigbird", pct=0.5,
             params={"percentage": 0.5, "num_global_block": 3, "num_rand_block": 2}),
        dict(T=2048, bm=64, bnm=64, cbn=64, pattern="global", pct=0.4,
             params={"percentage": 0.4, "key_pos": [0, 700, 1500, 5000]}),
        dict(T=131072, bm=128, bnm=2048, cbn=64, pattern="sptrans", pct=0.5, params={"percentage": 0.5}),
        dict(T=131072, bm=128, bnm=2048, cbn=64, pattern="bigbird", pct=0.25, params={"percentage": 0.25}),
        dict(T=131072, bm=128, bnm=2048, cbn=64, pattern="row_rand", pct=0.75, params={"percentage": 0.75}),
        dict(T=100000, bm=128, bnm=1600, cbn=64, pattern="band", pct=0.5, params={"percentage": 0.5}),
    ]
    return cases + extra


def make_maps(ref_root: str):
    sys.path.insert(0, ref_root)
    import torch
    from attention.precision_maps import make_precision_bitmask
    out = []
    for c in map_cases():
        rec = dict(c)
        try:
            words = make_precision_bitmask(c["T"], c["bm"], c["bnm"], None, percentage=c["pct"],
                                           pattern_type=c["pattern"], pattern_params=c["params"],
                                           COMPUTE_BLOCK_N=c["cbn"])
            rec["words"] = " ".join(format(int(x) & (2**64 - 1), "x") for x in words.tolist())
        except Exception as e:  # the reference's own errors are part of its behaviour
            rec["error"] = type(e).__name__
        out.append(rec)
        print(c["T"], c["pattern"], c["pct"], "error" if "error" in rec else len(rec["words"]), flush=True)
    meta = dict(torch=torch.__version__, generator="tests/golden/make_golden.py")
    (HERE / "maps.json").write_text(json.dumps(dict(meta=meta, cases=out), separators=(",", ":")))


def checksum(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def make_interp(ref_root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    import attention.triton.tilemix as tmx
    from attention.precision_maps import make_precision_bitmask
    from attention.triton.quant_per_block_varlen import per_block_int8_single

    # Bypass the two CUDA-only guards (this process only).
    torch.cuda.get_device_capability = lambda *a, **k: (10, 0)
    src = inspect.getsource(tmx.launch_prequantized).replace("if not q.is_cuda:", "if False:")
    ns = dict(tmx.__dict__)
    exec(src.replace("@torch.no_grad()\n", ""), ns)
    tmx.launch_prequantized = ns["launch_prequantized"]

    # quantiser fixtures
    q, k, v, cu = make_qkv([512, 300, 129], 3, 2, 128, seed=11, outliers=2)
    for name, x, blk in ([] if os.environ.get("TILEMIX_GOLDEN_ONLY") else [("q128", q, 128), ("k64", k, 64)]):
        x8, xs, cus = per_block_int8_single(x, cu, 512, BLK=blk, sm_scale=1.0)
        np.savez_compressed(HERE / f"interp_quant_{name}.npz", x8=x8.numpy(), scale=xs.numpy(),
                            cu_scale=cus.numpy(), checksum=checksum(x.numpy()))
        print("quant", name, flush=True)

    cases = [
        # (name, lens, hq, hk, d, block_m, pattern, mode, seed, outliers, int8_use_fp16_v, bias seed or None)
        ("cfg1_sptrans", [512], 4, 4, 64, 64, "sptrans", "mixed", 0, 0, True, None),
        ("cfg1_zero", [512], 4, 4, 64, 64, "zero", "mixed", 0, 0, True, None),
        ("cfg1_one", [512], 4, 4, 64, 64, "one", "mixed", 0, 0, True, None),
        ("gqa128_sptrans", [256], 3, 1, 128, 128, "sptrans", "mixed", 5, 4, True, None),
        ("gqa128_bigbird_varlen", [256, 160], 4, 2, 128, 128, "bigbird", "mixed", 7, 0, True, None),
        # the INT8-V PV path (the API's default int8_use_fp16_v=False)
        ("cfg1_sptrans_v8", [512], 4, 4, 64, 64, "sptrans", "mixed", 0, 0, False, None),
        ("gqa128_sptrans_v8", [256, 200], 3, 1, 128, 128, "sptrans", "mixed", 5, 4, False, None),
        # additive bias (indexed without a batch offset by the reference)
        ("gqa128_sptrans_bias", [256, 200], 4, 2, 128, 128, "sptrans", "mixed", 9, 2, True, 21),
        ("cfg1_one_bias_v8", [320, 192], 4, 2, 64, 64, "one", "mixed", 3, 0, False, 22),
    ]
    only = os.environ.get("TILEMIX_GOLDEN_ONLY")  # comma-separated case names (default: all)
    for name, lens, hq, hk, d, bm, pattern, mode, seed, outl, fp16_v, bias_seed in cases:
        if only and name not in only.split(","):
            continue
        q, k, v, cu = make_qkv(lens, hq, hk, d, seed=seed, outliers=outl)
        bias = None if bias_seed is None else make_bias(len(lens), hq, max(lens), bias_seed)
        T = max(lens)
        bn = 64
        bnm = pick_mask_block_n(T, bn)
        row = make_precision_bitmask(T, bm, bnm, None, percentage=0.5, pattern_type=pattern,
                                     pattern_params={"percentage": 0.5}, COMPUTE_BLOCK_N=bn)
        pm = row.repeat(hk)
        os.environ["TILEMIX_FORCE_CONFIG"] = f"{bm},{bn},4,1"
        o, m = tmx.tilemix_attention_with_quant(q, k, v, cu, cu, T, T, pm, block_m=bm, block_n=bn,
                                                block_n_mask=bnm, causal=True, sm_scale=d ** -0.5,
                                                routing_mode=mode, scalar_scales=(bm == 128 and bn == 64),
                                                int8_use_fp16_v=fp16_v, bias=bias)
        np.savez_compressed(HERE / f"interp_attn_{name}.npz", out=o.numpy(), bitmask=pm.numpy().view(np.int64),
                            lens=np.array(lens), hq=hq, hk=hk, d=d, block_m=bm, block_n=bn, block_n_mask=bnm,
                            seed=seed, outliers=outl, int8_use_fp16_v=fp16_v,
                            bias_seed=-1 if bias_seed is None else bias_seed,
                            checksum=checksum(q.numpy(), k.numpy(), v.numpy()))
        print("attn", name, m, flush=True)


def make_prefill(ref_root: str):
    """The reference's prefill rotary kernel (models/tilemix_llama.py:797-822) under the
    Triton interpreter; its SiLU kernel calls libdevice exp, which the interpreter cannot run."""
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    import models.tilemix_llama as ref_llama

    for name, b, hq, hk, t, d, cos_b, seed in [("d64", 2, 3, 1, 40, 64, 1, 31), ("d128_b2", 2, 4, 2, 33, 128, 2, 32)]:
        g = torch.Generator().manual_seed(seed)
        q = (torch.randn(b, hq, t, d, generator=g) * 3).half()
        k = (torch.randn(b, hk, t, d, generator=g) * 3).half()
        cos = torch.randn(cos_b, t, d, generator=g).half()
        sin = torch.randn(cos_b, t, d, generator=g).half()
        oq, ok = ref_llama.rotary_token_major(q, k, cos, sin)
        np.savez_compressed(HERE / f"interp_rotary_{name}.npz", q=q.numpy(), k=k.numpy(), cos=cos.numpy(),
                            sin=sin.numpy(), oq=oq.transpose(1, 2).contiguous().numpy(),
                            ok=ok.transpose(1, 2).contiguous().numpy())
        print("rotary", name, flush=True)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TILEMIX_REFERENCE_ROOT", "")
    if not root or not Path(root).exists():
        sys.exit("usage: make_golden.py <reference root>")
    what = sys.argv[2] if len(sys.argv) > 2 else "all"
    if what in ("all", "maps"):
        make_maps(root)
    if what in ("all", "interp"):
        make_interp(root)
    if what in ("all", "prefill"):
        make_prefill(root)
