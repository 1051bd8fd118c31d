"""CPU-side checks of the C ABI: the library loads, exports every symbol the
header declares, and its host-only logic behaves (no compute calls here)."""
import re
import os

import pytest

import rgpu_b200
from rgpu_b200 import gpu as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "rtgpu.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rt_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    L = G.lib()
    declared = _declared_symbols()
    assert len(declared) > 40
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, f"symbols declared in include/rtgpu.h but not exported: {missing}"


def test_python_mirror_binds_every_declared_symbol():
    assert sorted(set(G.exported_symbols())) == _declared_symbols()


def test_abi_version():
    assert G.lib().rt_abi_version() == 2


def test_python_structs_match_the_header_layout(tmp_path):
    # The ctypes mirrors of rt_gemm_args and rt_mlp_config must have the C
    # structs' size and field offsets (compiled from include/rtgpu.h by gcc).
    import ctypes as C
    import subprocess

    structs = {"rt_gemm_args": G.GemmArgs, "rt_mlp_config": G.MlpConfig}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "rtgpu.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l}
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[(cname, f)] == getattr(py, f).offset, (cname, f)


def test_no_device_is_reported_not_faked():
    # Without a GPU the context must fail loudly (no CPU fallback).
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises(rgpu_b200.RtError) as e:
        rgpu_b200.Gpu(0)
    assert e.value.code == G.RT_ERR_UNSUPPORTED


def test_fatias_sugeridas_rules():
    # tests/gpu.rs:432-441
    f = rgpu_b200.Gpu.fatias_sugeridas
    assert f(64, 64, 8192) > 1
    assert f(4096, 4096, 4096) == 1
    assert f(64, 64, 64) == 1
    # the measured optima quoted at gpu/mod.rs:1064-1070
    assert f(64, 64, 8192) == 64
    assert f(128, 128, 4096) == 16


def test_bf16_roundtrip_helpers():
    import numpy as np

    x = np.array([1.0, -2.5, 3.14159, 1e-3, 65504.0], np.float32)
    b = rgpu_b200.f32_to_bf16(x)
    y = rgpu_b200.bf16_to_f32(b)
    assert np.all(np.abs(y - x) <= np.abs(x) * 2.0 ** -8)
