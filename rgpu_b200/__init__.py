"""rgpu_b200: B200 (sm_100a) CUDA backend for rtensor's training hot path.

The compute lives in ``librtgpu.so`` (C ABI, ``include/rtgpu.h``); this
package is the Python mirror of rtensor's GPU API used by the tests and the
benchmark.  See ``rgpu_b200.gpu``.
"""
from .gpu import (  # noqa: F401
    Comm,
    Gpu,
    GpuMlp,
    GpuTensor,
    RtError,
    bf16_to_f32,
    f32_to_bf16,
    lib,
    upload_labels,
)

__all__ = ["Comm", "Gpu", "GpuMlp", "GpuTensor", "RtError", "bf16_to_f32", "f32_to_bf16", "lib", "upload_labels"]


def build(verbose: bool = False) -> str:
    """Compile librtgpu.so for sm_100a with nvcc (in-tree)."""
    import os
    import subprocess

    here = os.path.dirname(os.path.abspath(__file__))
    subprocess.run(["make", "-s", "-j8", "-C", os.path.join(here, "csrc")], check=True,
                   stdout=None if verbose else subprocess.DEVNULL)
    return os.path.join(here, "librtgpu.so")
