"""CPU checks of the C ABI: libsvla.so loads and exports every function include/svla.h declares, and the
ctypes mirror of each struct has the size the C compiler gives it.  No compute calls (no GPU here)."""

import re
import subprocess
from pathlib import Path

import pytest

from smolvla_mujoco_libero_b200 import _lib

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "svla.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\*\s]+?\b(svla_\w+)\s*\(", text, flags=re.M)))


def test_header_declarations_have_ctypes_signatures():
    names = declared_functions()
    assert len(names) >= 15
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (svla_\w+)", out))
    assert set(declared_functions()) <= exported


def test_version_and_error_string_without_gpu():
    lib = _lib.lib()
    assert b"sm_100a" in lib.svla_version()
    assert isinstance(lib.svla_last_error(), bytes)


def _c_sizeof(struct: str, tmp_path: Path) -> int:
    src = f'#include "{HEADER}"\n#include <stdio.h>\nint main(){{printf("%zu", sizeof({struct}));return 0;}}\n'
    probe = tmp_path / "sizeof_probe"
    probe.with_suffix(".c").write_text(src)
    subprocess.run(["gcc", "-o", str(probe), str(probe.with_suffix(".c"))], check=True)
    return int(subprocess.run([str(probe)], capture_output=True, text=True).stdout)


@pytest.mark.parametrize("cname,pyname", [("svla_gemm_desc", "GemmDesc"), ("svla_gemm_seg", "GemmSeg"),
                                          ("svla_norm_desc", "NormDesc"), ("svla_attn_desc", "AttnDesc"),
                                          ("svla_engine_info", "EngineInfo"), ("svla_flow_desc", "FlowDesc"),
                                          ("svla_flow_layer", "FlowLayer")])
def test_struct_layouts_match(cname, pyname, tmp_path):
    import ctypes
    assert ctypes.sizeof(getattr(_lib, pyname)) == _c_sizeof(cname, tmp_path)


def test_argument_errors_are_reported_without_a_gpu():
    import ctypes
    lib = _lib.lib()
    d = _lib.GemmDesc()
    d.kind = 7
    assert lib.svla_gemm(ctypes.byref(d), None) == 1
    assert b"kind" in lib.svla_last_error()
    assert lib.svla_quantize_smooth(None, 8, None, 1.0, None, 8, 1, 8, None) == 1
    assert lib.svla_sq_linear_w8a8(None, None, 1.0, None, None, None, 4, 16, 16, None, None, 0, None) == 1
    assert b"workspace" in lib.svla_last_error()


def test_flow_arguments_are_checked_before_any_launch():
    """svla_flow rejects what the persistent kernel cannot take (more than 64 action rows, widths that are not
    multiples of 16, too many layers, missing pointers) with status 1, without touching the GPU."""
    import ctypes
    lib = _lib.lib()
    assert lib.svla_flow(None, None) == 1

    def desc(**kw):
        d = _lib.FlowDesc()
        d.batch, d.chunk, d.prefix_len, d.hidden, d.action_dim = 1, 50, 177, 720, 32
        d.heads, d.kv_heads, d.mlp, d.n_layers, d.num_steps = 15, 5, 2048, 16, 10
        d.max_pos, d.eps = 227, 1e-5
        for k, v in kw.items():
            setattr(d, k, v)
        return d

    cases = [
        (dict(batch=2), "batch * chunk"),          # 100 rows
        (dict(hidden=712), "hidden"),              # not a multiple of 16
        (dict(mlp=2040), "multiples of 16"),
        (dict(kv_heads=4), "kv_heads"),            # 15 heads over 4 kv heads
        (dict(n_layers=33), "n_layers"),
        (dict(max_pos=0), "max_pos"),
        (dict(), "null pointer"),                  # no buffers at all
    ]
    for kw, word in cases:
        d = desc(**kw)
        assert lib.svla_flow(ctypes.byref(d), None) == 1, kw
        assert word.encode() in lib.svla_last_error(), (kw, lib.svla_last_error())


def test_flow_weight_packing_arguments_are_checked_before_any_launch():
    lib = _lib.lib()
    assert lib.svla_flow_packed_bytes(720, 960, 1) == 720 * 960
    assert lib.svla_flow_packed_bytes(720, 960, 2) == 2 * 720 * 960
    assert lib.svla_flow_packed_bytes(720, 968, 1) == 0   # k not a multiple of 16
    assert lib.svla_flow_packed_bytes(720, 960, 4) == 0   # int8 or bf16 only
    assert lib.svla_flow_pack_weight(0x100000, 1, 960, 720, 968, 0x200000, None) == 1
    assert lib.svla_flow_pack_weight(0x100000, 1, 900, 720, 960, 0x200000, None) == 1  # ld < k
    assert lib.svla_flow_pack_weight(0x100000, 1, 960, 720, 960, 0x200008, None) == 1  # out not 16-byte aligned
    assert b"aligned" in lib.svla_last_error()


def test_gemm_epilogue_pointers_are_checked_before_any_launch():
    """Outputs, residuals and int8 outputs that the epilogue would touch with 16-byte vectors must be 16-byte
    aligned with row strides that keep every row aligned; a bad one is status 1, not a GPU fault.  The fake
    device addresses are never dereferenced: every case fails on the host."""
    import ctypes
    lib = _lib.lib()

    def desc(epi=_lib.EPI_BF16, kind=_lib.KIND_I8, out=0x100000, ldo=64, **kw):
        d = _lib.GemmDesc()
        d.kind, d.epi, d.m, d.k, d.nseg = kind, epi, 128, 128, 1
        g = d.seg[0]
        g.a, g.lda, g.b, g.ldb, g.wscale = 0x200000, 128, 0x300000, 128, 0x400000
        g.out, g.ldo, g.n, g.act_scale = out, ldo, 64, 1.0
        for k, v in kw.items():
            setattr(d, k, v)
        return d

    cases = [
        (desc(out=0x100002), "16-byte"),                      # bf16 output 2 bytes off
        (desc(ldo=60), "row stride"),                         # below n
        (desc(ldo=68), "row stride"),                         # 136-byte rows
        (desc(epi=_lib.EPI_I32, ldo=66), "row stride"),       # int32 rows not 16-byte multiples
        (desc(epi=_lib.EPI_RESID, resid=0x500008, ldr=64), "RESID"),
        (desc(epi=_lib.EPI_RESID, resid=0x500000, ldr=60), "RESID"),
        (desc(epi=_lib.EPI_GELU_QUANT, out=None, qout=0x600004, ldq=64, q_smooth=0x700000, q_act=1.0), "qout"),
        (desc(epi=_lib.EPI_GELU_QUANT, out=None, qout=0x600000, ldq=72, q_smooth=0x700000, q_act=1.0), "qout"),
        (desc(epi=11), "epilogue"),
    ]
    for d, word in cases:
        assert lib.svla_gemm(ctypes.byref(d), None) == 1, word
        assert word.encode() in lib.svla_last_error(), (word, lib.svla_last_error())


def test_quantize_and_linear_alignment_is_checked_before_any_launch():
    lib = _lib.lib()
    # x 2 bytes off a 16-byte boundary, q 4 bytes off an 8-byte one
    assert lib.svla_quantize_smooth(0x100002, 64, None, 1.0, 0x200000, 64, 4, 64, None) == 1
    assert b"aligned" in lib.svla_last_error()
    assert lib.svla_quantize_smooth(0x100000, 64, None, 1.0, 0x200004, 64, 4, 64, None) == 1
    assert lib.svla_quantize_smooth(0x100000, 32, None, 1.0, 0x200000, 64, 4, 64, None) == 1  # ldx < k
    assert lib.svla_sq_linear_w8a8(0x100002, None, 1.0, 0x300000, 0x400000, None, 4, 64, 64, 0x500000, 0x600000,
                                   4096, None) == 1
    assert b"aligned" in lib.svla_last_error()


def test_channel_percentile_arguments_are_checked_before_any_launch():
    lib = _lib.lib()
    f = lib.svla_channel_percentile
    assert f(0x100000, 64, 1, 4097, 64, 0.5, 0x200000, 0x300000, None) == 1  # more than 4096 rows a call
    assert b"rows" in lib.svla_last_error()
    assert f(0x100000, 32, 1, 16, 64, 0.5, 0x200000, 0x300000, None) == 1    # ldx < k
    assert f(0x100000, 64, 1, 16, 64, -0.1, 0x200000, 0x300000, None) == 1   # q outside [0, 1]
    assert f(0x100000, 64, 0, 16, 64, 0.5, 0x200000, 0x300000, None) == 1    # no calls
    assert f(0x100001, 64, 1, 16, 64, 0.5, 0x200000, 0x300000, None) == 1    # odd bf16 address
    assert b"misaligned" in lib.svla_last_error()
    assert f(0x100000, 64, 1, 16, 64, 0.5, None, 0x300000, None) == 1
