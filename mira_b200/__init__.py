"""mira_b200: a B200 (sm_100a) `cuda` target for MIRA's W8A8 path.

`install()` registers the target with the host framework (the reference `mira` package) so that
`mira.compile_*(..., "cuda", quantize="w8a8")` and `mira run ... -t cuda --quantize w8a8` run the
quantized matmuls and convolutions on hand-written tcgen05 kernels (libmira_cuda.so).
"""
from __future__ import annotations

__all__ = ["install", "CudaTarget", "int8_depthwise"]


def install():
    from .plugin import install as _install
    return _install()


def __getattr__(name):
    if name == "CudaTarget":
        from .target import CudaTarget
        return CudaTarget
    if name == "int8_depthwise":
        from .depthwise import int8_depthwise
        return int8_depthwise
    raise AttributeError(name)
