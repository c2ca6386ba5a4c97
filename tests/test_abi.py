"""The C ABI library without a GPU: it loads, exports every entry point include/mira_cuda.h
declares with the signatures the Python binding uses, and reports "no device" as an error instead
of computing anything on the host."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from mira_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "mira_cuda.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(mira_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(str(_lib.LIB_PATH))
    names = declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_abi_version_and_defines_match_header():
    text = HEADER.read_text()
    defines = dict(re.findall(r"#define (MIRA_\w+) (-?\d+)", text))
    assert int(defines["MIRA_CUDA_ABI_VERSION"]) == _lib.ABI_VERSION == _lib.load().mira_cuda_abi_version()
    assert int(defines["MIRA_EPI_RELU"]) == _lib.EPI_RELU and int(defines["MIRA_EPI_ADD"]) == _lib.EPI_ADD
    assert int(defines["MIRA_OPND_FULL"]) == _lib.OPND_FULL and int(defines["MIRA_EPI_MAX_STEPS"]) == _lib.EPI_MAX_STEPS


def test_struct_layouts_match_the_c_declarations():
    # mira_epi_step: 3 int32 + float + pointer + int64 = 32 bytes; mira_epilogue embeds 8 of them
    assert C.sizeof(_lib.EpiStep) == 32
    assert _lib.Epilogue.steps.offset == 8
    assert C.sizeof(_lib.Dequant) == 5 * C.sizeof(C.c_void_p)


@pytest.mark.skipif(_lib.device_count() > 0, reason="this machine has a GPU")
def test_no_gpu_is_an_error_not_a_fallback():
    with pytest.raises(_lib.CudaError) as e:
        _lib.call("mira_cuda_set_device", 0)
    assert e.value.code == _lib.ENODEV
    p = C.c_void_p()
    with pytest.raises(_lib.CudaError):
        _lib.call("mira_cuda_malloc", C.byref(p), C.c_size_t(64))
    assert "device" in _lib.last_error()


def test_chunk_planar_layout_helpers_round_trip():
    """MIRA_LAYOUT_CP on the host: to_cp / from_cp invert each other, the padding ring and the
    guards are zero, and the byte count matches the header's formula."""
    from mira_b200 import kernels as K
    rng = np.random.default_rng(0)
    for n, h, w, cp in ((2, 5, 7, 32), (1, 56, 56, 64), (3, 1, 1, 16)):
        x = rng.integers(-127, 128, (n, h, w, cp)).astype(np.int8)
        b = K.to_cp(x)
        g = K.cp_guard(w)
        assert b.size == K.cp_bytes(n, h, w, cp) == (2 * g + 128 + cp // 16 * n * (h + 2) * (w + 2)) * 16
        assert np.array_equal(K.from_cp(b, n, h, w, cp), x)
        assert int(np.abs(b.astype(np.int64)).sum()) == int(np.abs(x.astype(np.int64)).sum())
        # slot (c16, img, y, x) = g + c16 * plane + (img * (h + 2) + y + 1) * (w + 2) + x + 1
        plane = n * (h + 2) * (w + 2)
        slot = g + (cp // 16 - 1) * plane + ((n - 1) * (h + 2) + h) * (w + 2) + w
        assert np.array_equal(b[slot * 16:slot * 16 + 16], x[n - 1, h - 1, w - 1, cp - 16:])
