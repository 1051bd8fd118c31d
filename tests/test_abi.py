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
    assert G.lib().rt_abi_version() == 1


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
