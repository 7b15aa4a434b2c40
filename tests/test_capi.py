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
        d.ld_time_in, d.max_pos, d.eps = 1440, 227, 1e-5
        for k, v in kw.items():
            setattr(d, k, v)
        return d

    cases = [
        (dict(batch=2), "batch * chunk"),          # 100 rows
        (dict(hidden=712), "hidden"),              # not a multiple of 16
        (dict(mlp=2040), "multiples of 16"),
        (dict(kv_heads=4), "kv_heads"),            # 15 heads over 4 kv heads
        (dict(n_layers=33), "n_layers"),
        (dict(ld_time_in=700), "ld_time_in"),
        (dict(), "null pointer"),                  # no buffers at all
    ]
    for kw, word in cases:
        d = desc(**kw)
        assert lib.svla_flow(ctypes.byref(d), None) == 1, kw
        assert word.encode() in lib.svla_last_error(), (kw, lib.svla_last_error())
