"""CPU tests of the boundary: the C-ABI library loads and exports every entry
point its header declares, the ctypes structures match the header's layout,
and the host mirror raises the reference's errors before touching a GPU."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent


def _declared_functions():
    names = []
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(tm_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from tilemix_b200._lib import LIB_PATH, SIGNATURES, lib

    assert LIB_PATH.exists(), "build the library first: python -m tilemix_b200.build"
    handle = lib()
    declared = _declared_functions()
    assert len(declared) >= 5, declared
    for name in declared:
        assert hasattr(handle, name), name
    assert set(declared) == set(SIGNATURES), (declared, sorted(SIGNATURES))


def test_status_strings():
    from tilemix_b200._lib import lib

    for code in (0, -1, -2, -3, -4, -5, -6):
        assert lib().tm_status_string(code)


def test_argument_errors_need_no_gpu():
    """Host-side validation of the C ABI returns a status without launching anything."""
    from tilemix_b200._lib import TmAttnParams, TmMapParams, lib

    assert lib().tm_attn_fwd(None, None) == -1
    p = TmAttnParams()
    assert lib().tm_attn_fwd(ctypes.byref(p), None) < 0
    m = TmMapParams()
    assert lib().tm_build_precision_map(None, None, None, None) == -1
    m.seq_len, m.block_m, m.block_n_mask, m.compute_block_n, m.pattern = 8192, 128, 64, 64, 7
    out = ctypes.c_uint64(0)
    assert lib().tm_build_precision_map(ctypes.byref(m), ctypes.byref(out), None, None) == -2  # 128 mask groups
    m.seq_len, m.block_m = 131072 * 2, 64
    m.block_n_mask = 4096
    assert lib().tm_build_precision_map(ctypes.byref(m), ctypes.byref(out), None, None) == -4  # too many rows
    m.seq_len, m.block_m, m.block_n_mask, m.pattern, m.percentage = 4096, 128, 64, 2, 1.5
    assert lib().tm_build_precision_map(ctypes.byref(m), ctypes.byref(out), None, None) == -2  # percentage


def test_ctypes_layout_matches_header():
    """Offsets of the ctypes mirrors agree with a C compiler's layout of the header structs."""
    import subprocess
    import tempfile

    from tilemix_b200._lib import TmAttnParams, TmAttnTuning, TmMapParams

    fields = {"tm_attn_params": [f[0] for f in TmAttnParams._fields_],
              "tm_map_params": [f[0] for f in TmMapParams._fields_],
              "tm_attn_tuning": [f[0] for f in TmAttnTuning._fields_]}
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "tilemix_b200.h"', "int main(void) {"]
    for struct, names in fields.items():
        src.append(f'printf("{struct} %zu\\n", sizeof({struct}));')
        for n in names:
            src.append(f'printf("{struct}.{n} %zu\\n", offsetof({struct}, {n}));')
    src.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        c = Path(d) / "layout.c"
        c.write_text("\n".join(src))
        exe = Path(d) / "layout"
        subprocess.run(["gcc", "-I", str(REPO / "include"), str(c), "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    got = dict(line.rsplit(" ", 1) for line in out.splitlines())
    for struct, cls in (("tm_attn_params", TmAttnParams), ("tm_map_params", TmMapParams),
                        ("tm_attn_tuning", TmAttnTuning)):
        assert int(got[struct]) == ctypes.sizeof(cls), struct
        for n in fields[struct]:
            assert int(got[f"{struct}.{n}"]) == getattr(cls, n).offset, (struct, n)


@pytest.mark.parametrize("kwargs,exc", [
    (dict(seq_len=8192, BLOCK_M=128, BLOCK_N=64, pattern_type="sptrans", percentage=0.5,
          pattern_params={"percentage": 0.5}, COMPUTE_BLOCK_N=64), ValueError),       # 128 mask groups
    (dict(seq_len=4096, BLOCK_M=128, BLOCK_N=96, pattern_type="band", percentage=0.5,
          pattern_params={"percentage": 0.5}, COMPUTE_BLOCK_N=64), ValueError),       # 96 % 64
    (dict(seq_len=4096, BLOCK_M=128, BLOCK_N=64, pattern_type="band", percentage=0.5,
          pattern_params=None, COMPUTE_BLOCK_N=64), ValueError),                      # needs params
    (dict(seq_len=4096, BLOCK_M=128, BLOCK_N=64, pattern_type="band", percentage=1.5,
          pattern_params={"percentage": 1.5}, COMPUTE_BLOCK_N=64), ValueError),       # percentage range
    (dict(seq_len=3, BLOCK_M=64, BLOCK_N=64, pattern_type="sptrans", percentage=0.5,
          pattern_params={"percentage": 0.5}, COMPUTE_BLOCK_N=64), ZeroDivisionError),  # stride 0
])
def test_map_host_validation(kwargs, exc):
    from tilemix_b200.attention.precision_maps import make_precision_bitmask

    with pytest.raises(exc):
        make_precision_bitmask(token_mask=None, **kwargs)


def test_map_token_mask_path_not_built():
    from tilemix_b200.attention.precision_maps import make_precision_bitmask

    with pytest.raises(NotImplementedError):
        make_precision_bitmask(512, 64, 64, torch.ones(1, 1, 512, 512, dtype=torch.bool), None, "causal", None, 64)


def test_attention_requires_cuda_tensors():
    from tilemix_b200.attention.tilemix import tilemix_attention_with_quant

    q = torch.zeros(128, 2, 64, dtype=torch.float16)
    cu = torch.tensor([0, 128], dtype=torch.int32)
    pm = torch.zeros(2, dtype=torch.uint64)
    with pytest.raises(RuntimeError):
        tilemix_attention_with_quant(q, q, q, cu, cu, 128, 128, pm, block_m=128, block_n=64, causal=True,
                                     routing_mode="mixed")


class _FakeTensor:
    """Just the attributes the argument checks read (no device needed)."""

    def __init__(self, shape, dtype=torch.float16, device="cuda:0", is_cuda=True):
        self.shape, self.dtype, self.device, self.is_cuda = torch.Size(shape), dtype, torch.device(device), is_cuda
        self.ndim = len(shape)

    def numel(self):
        n = 1
        for s in self.shape:
            n *= s
        return n


@pytest.mark.parametrize("change,exc,text", [
    (dict(q=_FakeTensor((64, 4, 64), is_cuda=False)), RuntimeError, "CUDA-only"),
    (dict(q=_FakeTensor((64, 4, 64, 1))), ValueError, "flattened"),
    (dict(v=_FakeTensor((64, 1, 64))), ValueError, "K/V shapes"),
    (dict(q=_FakeTensor((64, 3, 64))), ValueError, "divisible"),
    (dict(v=_FakeTensor((64, 2, 64), device="cuda:1")), ValueError, "one CUDA device"),
    (dict(v=_FakeTensor((64, 2, 64), dtype=torch.bfloat16)), TypeError, "one dtype"),
    (dict(max_k=32), ValueError, "equal Q/K lengths"),
    (dict(block_n_mask=96), ValueError, "multiple of block_n"),
    (dict(max_q=64 * 65, max_k=64 * 65), ValueError, "64 mask blocks"),
    (dict(BLKQ=128), ValueError, "scalar_scales"),
    (dict(bitmask=_FakeTensor((2,), dtype=torch.int64)), TypeError, "torch.uint64"),
    (dict(bitmask=_FakeTensor((3,), dtype=torch.uint64)), ValueError, "rows, expected 2"),
])
def test_validate_order_and_messages(change, exc, text):
    """launch_prequantized's checks (tilemix.py:1167-1201): the first failing rule raises the
    reference's exception type and message; a valid call raises nothing."""
    from tilemix_b200.attention.tilemix import _validate

    args = dict(q=_FakeTensor((64, 4, 64)), k=_FakeTensor((64, 2, 64)), v=_FakeTensor((64, 2, 64)), max_q=64,
                max_k=64, bitmask=_FakeTensor((2,), dtype=torch.uint64), block_m=64, block_n=64, block_n_mask=64,
                BLKQ=64, BLKK=64, scalar_scales=True)
    _validate(**args)
    args.update(change)
    with pytest.raises(exc, match=text):
        _validate(**args)


def _int8_v_params(**over):
    """tm_attn_params of an INT8-routed INT8-V call with stand-in (aligned, never read) pointers."""
    from tilemix_b200._lib import TmAttnParams

    p = TmAttnParams()
    fake = 0x100000
    for name in ("q", "k", "v", "out", "cu_seqlens_q", "cu_seqlens_k", "k8", "k_scale", "cu_k_scale", "v8",
                 "v_scale", "cu_v_scale"):
        setattr(p, name, fake)
    p.q_stride_tok, p.q_stride_head = 8 * 128, 128
    p.k_stride_tok, p.k_stride_head = 8 * 128, 128
    p.v_stride_tok, p.v_stride_head = 8 * 128, 128
    p.o_stride_tok, p.o_stride_head = 8 * 128, 128
    p.k8_stride_tok, p.k8_stride_head = 8 * 128, 128
    p.v8_stride_tok, p.v8_stride_head = 8 * 128, 128
    p.q_tokens = p.k_tokens = 256
    p.batch, p.heads_q, p.heads_k, p.head_dim = 0, 8, 8, 128
    p.max_seqlen_q = p.max_seqlen_k = 256
    p.block_m, p.block_n, p.block_n_mask, p.blkq, p.blkk = 128, 64, 64, 128, 64
    p.routing_mode, p.int8_use_fp16_v, p.sm_scale = 2, 0, 0.088
    for k, v in over.items():
        setattr(p, k, v)
    return p


def test_int8_v_operand_rules_need_no_gpu():
    """INT8-V takes the int8 V codes (any kernel) or their fp16 copy (the paired kernel's shape:
    head_dim 128, block_m 128, Q quantised in the kernel, no bias, automatic kernel choice)."""
    from tilemix_b200._lib import TmAttnTuning, lib

    def rc(p, force_general=0):
        t = TmAttnTuning()
        t.force_general = force_general
        return lib().tm_attn_fwd_ex(ctypes.byref(p), ctypes.byref(t), None)

    fake = 0x200000
    assert rc(_int8_v_params()) == 0                                    # int8 codes, empty batch
    assert rc(_int8_v_params(v8=None)) == -1                            # neither operand
    assert rc(_int8_v_params(v8=None, v8_f16=fake, v8_f16_stride_tok=1024, v8_f16_stride_head=128)) == 0
    assert rc(_int8_v_params(v8=None, v8_f16=fake), force_general=1) == -1             # general kernel
    assert rc(_int8_v_params(v8=None, v8_f16=fake, head_dim=64, q_stride_head=64)) == -1  # not the paired shape
    assert rc(_int8_v_params(v8=None, v8_f16=fake, q8=fake, q_scale=fake, cu_q_scale=fake)) == -1  # prequantised Q
    assert rc(_int8_v_params(v_scale=None)) == -1                       # V scales
    # a misaligned fp16 copy is rejected before anything runs (non-empty batch)
    assert rc(_int8_v_params(batch=1, v8=None, v8_f16=fake + 8, v8_f16_stride_tok=1024,
                             v8_f16_stride_head=128)) == -3
