"""The C ABI library: builds, loads and exports every symbol the header
declares; the ctypes struct layouts match the C compiler's."""

import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "heatvit_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"HV_API\s+(?:const\s+char\s*\*|int)\s*(hv_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "hv_infer_batch" in syms and "hv_model_create" in syms and len(syms) >= 19


def test_library_exports_every_declared_symbol():
    from heatvit_b200 import build
    lib = build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (hv_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_library_loads_without_gpu():
    import ctypes
    from heatvit_b200 import build
    lib = ctypes.CDLL(build.build())
    lib.hv_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.hv_version()


def test_struct_layout_matches_c(tmp_path):
    from heatvit_b200 import abi
    import ctypes
    prog = tmp_path / "sz.c"
    prog.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "heatvit_b200.h"\n'
                    'int main(){printf("%zu %zu %zu %zu %zu %zu %zu\\n", sizeof(hv_params), '
                    'sizeof(hv_block_params), sizeof(hv_selector_params), sizeof(hv_patch_params), '
                    'sizeof(hv_selector_summary), offsetof(hv_params, num_selectors), '
                    'offsetof(hv_params, head_w_scale_exp));return 0;}\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(prog), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals == [ctypes.sizeof(abi.HvParams), ctypes.sizeof(abi.HvBlockParams),
                    ctypes.sizeof(abi.HvSelectorParams), ctypes.sizeof(abi.HvPatchParams),
                    ctypes.sizeof(abi.HvSelectorSummary), abi.HvParams.num_selectors.offset,
                    abi.HvParams.head_w_scale_exp.offset]


def test_no_cuda_means_loud_failure(monkeypatch):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from heatvit_b200 import engine
    with pytest.raises(RuntimeError, match="CUDA"):
        engine._torch()
