"""ctypes binding of libmira_cuda.so (the C ABI in include/mira_cuda.h).

The library is loaded from this package directory.  There is no fallback: if the library is
missing or the machine has no sm_100 GPU, calls raise instead of computing anything on the CPU.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmira_cuda.so"

# mirrors of the #defines in include/mira_cuda.h
ABI_VERSION = 1
OK, EINVAL, ECUDA, ENODEV, EKERNEL = 0, 1, 2, 3, 4
EPI_RELU, EPI_GELU, EPI_SIGMOID, EPI_TANH = 1, 2, 3, 4
EPI_ADD, EPI_SUB, EPI_MUL, EPI_DIV, EPI_MAXIMUM, EPI_MINIMUM = 16, 17, 18, 19, 20, 21
OPND_NONE, OPND_SCALAR, OPND_CHANNEL, OPND_FULL, OPND_ROW = 0, 1, 2, 3, 4
OPND_VIEW = 5
LAYOUT_NHWC, LAYOUT_ROW4, LAYOUT_CP = 0, 1, 2
EPI_MAX_STEPS = 8
ROW_MAX = 8192

UNARY_CODES = {"relu": EPI_RELU, "gelu": EPI_GELU, "sigmoid": EPI_SIGMOID, "tanh": EPI_TANH}
BINARY_CODES = {"add": EPI_ADD, "sub": EPI_SUB, "mul": EPI_MUL, "div": EPI_DIV,
                "maximum": EPI_MAXIMUM, "minimum": EPI_MINIMUM}


class EpiStep(C.Structure):
    _fields_ = [("op", C.c_int32), ("operand", C.c_int32), ("swapped", C.c_int32), ("scalar", C.c_float),
                ("ptr", C.c_void_p), ("ld", C.c_int64)]


class Epilogue(C.Structure):
    _fields_ = [("n_steps", C.c_int32), ("steps", EpiStep * EPI_MAX_STEPS), ("out_f32", C.c_void_p),
                ("ld_f32", C.c_int64), ("out_i8", C.c_void_p), ("ld_i8", C.c_int64), ("out_scale", C.c_float),
                ("i8_layout", C.c_int32)]


class Dequant(C.Structure):
    _fields_ = [("scale64", C.c_void_p), ("scale_hi", C.c_void_p), ("scale_lo", C.c_void_p),
                ("row_scale", C.c_void_p), ("col_scale", C.c_void_p)]


class View4(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("stride", C.c_int64 * 4)]


class BmmStep(C.Structure):
    _fields_ = [("op", C.c_int32), ("operand", C.c_int32), ("swapped", C.c_int32), ("scalar", C.c_float),
                ("view", View4)]


class BmmEpilogue(C.Structure):
    _fields_ = [("n_steps", C.c_int32), ("steps", BmmStep * EPI_MAX_STEPS), ("out_f32", View4), ("out_i8", View4),
                ("out_scale", C.c_float)]


class Attention(C.Structure):
    _fields_ = [("batch0", C.c_int64), ("batch1", C.c_int64), ("tq", C.c_int64), ("tk", C.c_int64), ("dh", C.c_int64),
                ("q", View4), ("k", View4), ("v", View4), ("scale_op", C.c_int32), ("scale", C.c_float),
                ("mask", View4), ("tile_max", C.c_void_p), ("kmax", C.c_void_p), ("tile_zero", C.c_void_p),
                ("out_f32", View4),
                ("out_i8", View4), ("out_scale", C.c_float), ("workspace", C.c_void_p),
                ("workspace_bytes", C.c_int64)]


_i64, _f32, _vp, _i32 = C.c_int64, C.c_float, C.c_void_p, C.c_int

# name -> (restype, argtypes); every symbol include/mira_cuda.h declares
SIGNATURES: dict[str, tuple] = {
    "mira_cuda_abi_version": (_i32, []),
    "mira_cuda_last_error": (_i32, [C.c_char_p, C.c_size_t]),
    "mira_cuda_device_count": (_i32, []),
    "mira_cuda_set_device": (_i32, [_i32]),
    "mira_cuda_device_info": (_i32, [C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_i32)]),
    "mira_cuda_malloc": (_i32, [C.POINTER(_vp), C.c_size_t]),
    "mira_cuda_free": (_i32, [_vp]),
    "mira_cuda_host_alloc": (_i32, [C.POINTER(_vp), C.c_size_t]),
    "mira_cuda_host_free": (_i32, [_vp]),
    "mira_cuda_memset": (_i32, [_vp, _i32, C.c_size_t]),
    "mira_cuda_h2d_copy_stream": (_i32, [_vp, _vp, C.c_size_t]),
    "mira_cuda_copy_stream_record": (_i32, [_vp]),
    "mira_cuda_copy_stream_wait": (_i32, [_vp]),
    "mira_cuda_stream_wait": (_i32, [_vp]),
    "mira_cuda_event_sync": (_i32, [_vp]),
    "mira_cuda_h2d": (_i32, [_vp, _vp, C.c_size_t]),
    "mira_cuda_d2h": (_i32, [_vp, _vp, C.c_size_t]),
    "mira_cuda_d2d": (_i32, [_vp, _vp, C.c_size_t]),
    "mira_cuda_sync": (_i32, []),
    "mira_cuda_get_stream": (_i32, [C.POINTER(_vp)]),
    "mira_cuda_event_create": (_i32, [C.POINTER(_vp)]),
    "mira_cuda_event_record": (_i32, [_vp]),
    "mira_cuda_event_elapsed": (_i32, [_vp, _vp, C.POINTER(_f32)]),
    "mira_cuda_event_destroy": (_i32, [_vp]),
    "mira_cuda_graph_begin": (_i32, []),
    "mira_cuda_graph_end": (_i32, [C.POINTER(_vp)]),
    "mira_cuda_graph_launch": (_i32, [_vp]),
    "mira_cuda_graph_destroy": (_i32, [_vp]),
    "mira_cuda_launch_count": (_i64, []),
    "mira_cuda_selftest_wait_timeout": (_i32, [_i64]),
    "mira_cuda_quantize_rows": (_i32, [_vp, _i64, _i64, _i64, _f32, _vp, _i64]),
    "mira_cuda_quantize_nchw_to_nhwc": (_i32, [_vp, _i64, _i64, _i64, _i64, _f32, _vp, _i64]),
    "mira_cuda_qgemm": (_i32, [_i64, _i64, _i64, _vp, _i64, _vp, _i64, C.POINTER(Dequant), C.POINTER(Epilogue)]),
    "mira_cuda_qgemm_workspace": (_i64, [_i64, _i64, _i64]),
    "mira_cuda_qgemm_splitk": (_i32, [_i64, _i64, _i64, _vp, _i64, _vp, _i64, C.POINTER(Dequant), C.POINTER(Epilogue),
                                      _vp, _i64]),
    "mira_cuda_qgemm_splitk_static": (_i32, [_i64, _i64, _i64, _vp, _i64, _vp, _i64, C.POINTER(Dequant),
                                             C.POINTER(Epilogue)]),
    "mira_cuda_quantize_nchw_to_row4": (_i32, [_vp, _i64, _i64, _i64, _i64, _f32, _vp, _i64, _i64, _i64]),
    "mira_cuda_qconv2d": (_i32, [_i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64,
                                 _i64, _i64, _i64, _i64, C.POINTER(Dequant), C.POINTER(Epilogue)]),
    "mira_cuda_qconv2d_maxpool": (_i32, [_i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64,
                                         _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, C.POINTER(Dequant),
                                         C.POINTER(Epilogue)]),
    "mira_cuda_maxpool2d_nhwc": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _i64,
                                        _vp, _i64, _f32]),
    "mira_cuda_maxpool2d_nhwc_ex": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _vp,
                                           _i64, _vp, _i64, _f32, _i64]),
    "mira_cuda_cp_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "mira_cuda_mean_hw_nhwc": (_i32, [_vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _f32]),
    "mira_cuda_dwconv2d_nhwc": (_i32, [_vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                       _i64, C.POINTER(Epilogue)]),
    "mira_cuda_qdwconv2d_nhwc": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                        _i64, _i64, C.POINTER(Dequant), C.POINTER(Epilogue)]),
    "mira_cuda_nchw_to_nhwc_f32": (_i32, [_vp, _i64, _i64, _i64, _i64, _vp, _i64]),
    "mira_cuda_nhwc_to_nchw_f32": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mira_cuda_bmm_f32": (_i32, [_i64, _i64, _i64, _i64, _i64, C.POINTER(View4), C.POINTER(View4),
                                 C.POINTER(BmmEpilogue)]),
    "mira_cuda_dynamic_slice": (_i32, [C.POINTER(View4), C.POINTER(_i64), _vp, _i64, C.POINTER(_i64),
                                       C.POINTER(View4)]),
    "mira_cuda_dynamic_update_slice": (_i32, [C.POINTER(View4), C.POINTER(_i64), C.POINTER(View4),
                                              C.POINTER(_i64), _vp, _i64]),
    "mira_cuda_elementwise_f32": (_i32, [_i32, _i64, _i64, _i64, _i64, C.POINTER(View4), C.POINTER(View4), _f32, _i32,
                                         C.POINTER(View4)]),
    "mira_cuda_im2col_f32": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                    _vp, _i64]),
    "mira_cuda_bmm_f32_w8": (_i32, [_i64, _i64, _i64, _i64, _i64, C.POINTER(View4), C.POINTER(View4), _vp,
                                    C.POINTER(BmmEpilogue)]),
    "mira_cuda_layernorm_rows": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _f32, _vp, _i64, _vp, _i64, _f32]),
    "mira_cuda_softmax_rows": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64]),
    "mira_cuda_embed_rows": (_i32, [_vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64]),
    "mira_cuda_copy_view_f32": (_i32, [_i64, _i64, _i64, _i64, C.POINTER(View4), C.POINTER(View4)]),
    "mira_cuda_attention_f32": (_i32, [C.POINTER(Attention)]),
    "mira_cuda_attention_workspace": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "mira_cuda_absmax_f32": (_i32, [_i64, _i64, _i64, _i64, C.POINTER(View4), _vp]),
}


class CudaError(RuntimeError):
    """A libmira_cuda call failed; `code` is the MIRA_CUDA_E* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lib = None


def load() -> C.CDLL:
    """The loaded library; raises if it was not built (run `python -m mira_b200.build`)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run `python -m mira_b200.build` (needs nvcc)")
        lib = C.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL | getattr(os, "RTLD_NOW", 2))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.mira_cuda_abi_version() != ABI_VERSION:
            raise RuntimeError("libmira_cuda.so ABI version does not match this package")
        _lib = lib
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load().mira_cuda_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def call(name: str, *args):
    """Calls an int-returning entry point and raises CudaError on a non-zero status."""
    rc = getattr(load(), name)(*args)
    if rc != OK:
        raise CudaError(rc, f"{name}: {last_error()}")
    return rc


def device_count() -> int:
    return load().mira_cuda_device_count()


def launch_count() -> int:
    return int(load().mira_cuda_launch_count())
