"""Python-side launchers for the kernels of libmira_cuda.so.

Each function takes device pointers (DeviceBuffer, int addresses) and plain sizes and fills the
descriptor structs of include/mira_cuda.h.  Host-side preparation of constants (int8 weight
re-layout, per-channel scale splits) lives here too, because it defines what the kernels expect.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _lib
from .device import ptr

CHANNEL_PAD = 256    # per-channel arrays are padded to this many entries


def round_up(x: int, m: int) -> int:
    return (int(x) + m - 1) // m * m


# ----------------------------------------------------------------------------- host preparation

def scale_arrays(x_scale: float, w_scale: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(scale64, scale_hi, scale_lo) for per-channel dequant, padded to a multiple of CHANNEL_PAD.
    scale64 = float64(x_scale) * float64(w_scale), the reference's factor (ops.py:619, ops.py:633)."""
    n = len(w_scale)
    npad = round_up(max(n, 1), CHANNEL_PAD)
    s64 = np.zeros(npad, np.float64)
    s64[:n] = np.float64(x_scale) * np.asarray(w_scale).astype(np.float64)
    hi = s64.astype(np.float32)
    lo = (s64 - hi.astype(np.float64)).astype(np.float32)
    return s64, hi, lo


def pad_channels(v: np.ndarray) -> np.ndarray:
    """f32 per-channel operand padded to a multiple of CHANNEL_PAD."""
    v = np.asarray(v, np.float32).ravel()
    out = np.zeros(round_up(max(len(v), 1), CHANNEL_PAD), np.float32)
    out[:len(v)] = v
    return out


def matmul_weight(q_kn: np.ndarray) -> np.ndarray:
    """Reference qmatmul weight int8 [K, N] -> K-major [N, round_up(K, 16)] (zero padded)."""
    k, n = q_kn.shape
    out = np.zeros((n, round_up(k, 16)), np.int8)
    out[:, :k] = q_kn.T
    return out


def conv_channels(c: int) -> int:
    """Padded channel count of an NHWC int8 activation: 4 for c <= 4, else a multiple of 16."""
    return 4 if c <= 4 else round_up(c, 16)


def conv_weight(q_oihw: np.ndarray, cp: Optional[int] = None) -> tuple[np.ndarray, int]:
    """Reference qconv2d weight int8 [O, C, KH, KW] -> [O, round_up(KH*KW*Cp, 16)] with
    k = (i * KW + j) * Cp + c (zero padded channels; Cp defaults to conv_channels(C)).
    Returns (weights, Cp)."""
    o, c, kh, kw = q_oihw.shape
    cp = conv_channels(c) if cp is None else int(cp)
    assert cp >= c
    t = np.zeros((o, kh, kw, cp), np.int8)
    t[:, :, :, :c] = q_oihw.transpose(0, 2, 3, 1)
    k = kh * kw * cp
    out = np.zeros((o, round_up(k, 16)), np.int8)
    out[:, :k] = t.reshape(o, k)
    return out, cp


def row4_entries(ow: int, stride_w: int) -> int:
    """16-byte entries per image row of the row-expanded layout read by a conv with output width ow
    and horizontal stride stride_w (1, 2 or 4; entries are laid out at that stride)."""
    return int(ow) + 4 // int(stride_w)


def cp_guard(w: int) -> int:
    """Guard slots in front of the planes of the chunk-planar layout (MIRA_LAYOUT_CP) of width w."""
    return round_up(int(w) + 3, 8)


# bytes of one halo buffer of the chunk-planar conv kernels per input channel count (libmira_cuda's
# patch_cap): a 3x3 stride-1 conv reads the layout when (128 + 2 (w + 3)) * c fits
PATCH_CAP = {64: 16384, 128: 24576, 256: 41984, 512: 75776}


def patch_fits(c: int, w: int) -> bool:
    """A 3x3 stride-1 pad-1 conv over [., c, ., w] int8 inputs has a chunk-planar kernel."""
    cap = PATCH_CAP.get(int(c))
    return cap is not None and (128 + 2 * (int(w) + 3)) * int(c) <= cap


# The chunk-planar conv computes every slot of the zero-padded plane, (h + 2)(w + 2) per image
# instead of h w, and its epilogue (the conv's bound) runs on all of them: on narrow images that
# extra work outweighs the cheaper operand loads (measured on ResNet-18: faster at 56 x 56, slower
# at 28 x 28 and below), so the planner uses it from this width on.
PATCH_MIN_WIDTH = 40


def patch_preferred(c: int, w: int) -> bool:
    return int(w) >= PATCH_MIN_WIDTH and patch_fits(c, w)


def cp_bytes(n: int, h: int, w: int, cp: int) -> int:
    """Bytes of an int8 [n, h, w, cp] activation in the chunk-planar, zero-padded layout."""
    g = cp_guard(w)
    return (2 * g + 128 + (int(cp) // 16) * int(n) * (int(h) + 2) * (int(w) + 2)) * 16


def to_cp(x_nhwc: np.ndarray) -> np.ndarray:
    """int8 NHWC [n, h, w, cp] (cp % 16 == 0) -> its MIRA_LAYOUT_CP bytes (host-side, for tests)."""
    n, h, w, cp = x_nhwc.shape
    g = cp_guard(w)
    planes = np.zeros((cp // 16, n, h + 2, w + 2, 16), np.int8)
    planes[:, :, 1:h + 1, 1:w + 1, :] = x_nhwc.reshape(n, h, w, cp // 16, 16).transpose(3, 0, 1, 2, 4)
    out = np.zeros(cp_bytes(n, h, w, cp), np.int8)
    out[g * 16:g * 16 + planes.size] = planes.ravel()
    return out


def from_cp(buf: np.ndarray, n: int, h: int, w: int, cp: int) -> np.ndarray:
    """The inverse of to_cp: MIRA_LAYOUT_CP bytes -> int8 NHWC [n, h, w, cp]."""
    g = cp_guard(w)
    size = (cp // 16) * n * (h + 2) * (w + 2) * 16
    planes = np.asarray(buf, np.int8)[g * 16:g * 16 + size].reshape(cp // 16, n, h + 2, w + 2, 16)
    return np.ascontiguousarray(planes[:, :, 1:h + 1, 1:w + 1, :].transpose(1, 2, 3, 0, 4).reshape(n, h, w, cp))


def conv_weight_row4(q_oihw: np.ndarray) -> np.ndarray:
    """Reference qconv2d weight int8 [O, C<=4, KH, KW<=8] -> [O, KH*32] for MIRA_LAYOUT_ROW4 inputs:
    k = i * 32 + j * 4 + c (taps j >= KW and channels c >= C are 0)."""
    o, c, kh, kw = q_oihw.shape
    assert c <= 4 and kw <= 8
    t = np.zeros((o, kh, 8, 4), np.int8)
    t[:, :, :kw, :c] = q_oihw.transpose(0, 2, 3, 1)
    return t.reshape(o, kh * 32)


# ----------------------------------------------------------------------------- epilogue descriptors

@dataclass
class Step:
    """One fused epilogue step: `op` a reference UNARY/BINARY name, `operand` one of
    "none" / "scalar" / "channel" / "full" / "row"."""
    op: str
    operand: str = "none"
    swapped: bool = False
    scalar: float = 0.0
    ptr: object = None
    ld: int = 0


_OPND = {"none": _lib.OPND_NONE, "scalar": _lib.OPND_SCALAR, "channel": _lib.OPND_CHANNEL,
         "full": _lib.OPND_FULL, "row": _lib.OPND_ROW}


@dataclass
class Epi:
    steps: Sequence[Step] = field(default_factory=list)
    out_f32: object = None
    ld_f32: int = 0
    out_i8: object = None
    ld_i8: int = 0
    out_scale: float = 1.0
    i8_layout: int = 0       # _lib.LAYOUT_NHWC or _lib.LAYOUT_CP (convolutions)

    def struct(self) -> _lib.Epilogue:
        e = _lib.Epilogue()
        if len(self.steps) > _lib.EPI_MAX_STEPS:
            raise ValueError(f"at most {_lib.EPI_MAX_STEPS} fused epilogue steps")
        e.n_steps = len(self.steps)
        for i, s in enumerate(self.steps):
            code = _lib.UNARY_CODES.get(s.op) or _lib.BINARY_CODES.get(s.op)
            if code is None:
                raise ValueError(f"epilogue op {s.op!r} has no device implementation")
            e.steps[i].op = code
            e.steps[i].operand = _OPND[s.operand]
            e.steps[i].swapped = int(bool(s.swapped))
            e.steps[i].scalar = float(np.float32(s.scalar))
            e.steps[i].ptr = ptr(s.ptr).value or 0
            e.steps[i].ld = int(s.ld)
        e.out_f32 = ptr(self.out_f32).value or 0
        e.ld_f32 = int(self.ld_f32)
        e.out_i8 = ptr(self.out_i8).value or 0
        e.ld_i8 = int(self.ld_i8)
        e.out_scale = float(np.float32(self.out_scale))
        e.i8_layout = int(self.i8_layout)
        return e


def dequant_channel(scale64, scale_hi, scale_lo) -> _lib.Dequant:
    d = _lib.Dequant()
    d.scale64, d.scale_hi, d.scale_lo = ptr(scale64).value, ptr(scale_hi).value, ptr(scale_lo).value
    return d


def dequant_rowcol(row_scale, col_scale) -> _lib.Dequant:
    d = _lib.Dequant()
    d.row_scale, d.col_scale = ptr(row_scale).value, ptr(col_scale).value
    return d


# ----------------------------------------------------------------------------- launchers

def quantize_rows(x, rows: int, cols: int, ld_x: int, scale: float, xq, ld_q: int) -> None:
    _lib.call("mira_cuda_quantize_rows", ptr(x), rows, cols, ld_x, float(np.float32(scale)), ptr(xq), ld_q)


def quantize_nchw_to_nhwc(x, n: int, c: int, h: int, w: int, scale: float, xq, cp: int) -> None:
    _lib.call("mira_cuda_quantize_nchw_to_nhwc", ptr(x), n, c, h, w, float(np.float32(scale)), ptr(xq), cp)


def qgemm(M: int, N: int, K: int, A, lda: int, B, ldb: int, dq: _lib.Dequant, epi: Epi) -> None:
    e = epi.struct()
    _lib.call("mira_cuda_qgemm", M, N, K, ptr(A), lda, ptr(B), ldb, C.byref(dq), C.byref(e))


def qgemm_workspace(M: int, N: int, K: int) -> int:
    """Workspace bytes of qgemm_splitk for this shape on the current device (0: no split)."""
    return int(_lib.load().mira_cuda_qgemm_workspace(M, N, K))


def qgemm_splitk(M: int, N: int, K: int, A, lda: int, B, ldb: int, dq: _lib.Dequant, epi: Epi, workspace,
                 workspace_bytes: int) -> None:
    e = epi.struct()
    _lib.call("mira_cuda_qgemm_splitk", M, N, K, ptr(A), lda, ptr(B), ldb, C.byref(dq), C.byref(e), ptr(workspace),
              workspace_bytes)


def quantize_nchw_to_row4(x, n: int, c: int, h: int, w: int, scale: float, xq, row_entries: int, pad: int,
                          entry_stride: int = 1) -> None:
    _lib.call("mira_cuda_quantize_nchw_to_row4", ptr(x), n, c, h, w, float(np.float32(scale)), ptr(xq), row_entries,
              pad, entry_stride)


def qconv2d(n: int, h: int, w: int, cp: int, x, o: int, kh: int, kw: int, wq, ldw: int, stride, padding,
            dilation, dq: _lib.Dequant, epi: Epi, layout: int = 0, row_entries: int = 0) -> None:
    e = epi.struct()
    _lib.call("mira_cuda_qconv2d", n, h, w, cp, ptr(x), layout, row_entries, o, kh, kw, ptr(wq), ldw, stride[0],
              stride[1], padding[0], padding[1], dilation[0], dilation[1], C.byref(dq), C.byref(e))


def qconv2d_maxpool(n: int, h: int, w: int, cp: int, x, o: int, kh: int, kw: int, wq, ldw: int, stride, padding,
                    dilation, pool_size: int, pool_stride: int, pool_pad: int, pool_pad_value: float,
                    dq: _lib.Dequant, epi: Epi, layout: int = 0, row_entries: int = 0) -> None:
    e = epi.struct()
    _lib.call("mira_cuda_qconv2d_maxpool", n, h, w, cp, ptr(x), layout, row_entries, o, kh, kw, ptr(wq), ldw,
              stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1], pool_size, pool_stride,
              pool_pad, float(np.float32(pool_pad_value)), C.byref(dq), C.byref(e))


def maxpool2d(n, h, w, c, ldc_in, size, stride, pad, pad_value, x_f32=None, x_i8=None, out_f32=None,
              ldc_out_f32=0, out_i8=None, ldc_out_i8=0, out_scale=1.0, i8_layout: int = 0) -> None:
    _lib.call("mira_cuda_maxpool2d_nhwc_ex", ptr(x_f32), ptr(x_i8), n, h, w, c, ldc_in, size, stride, pad,
              float(np.float32(pad_value)), ptr(out_f32), ldc_out_f32, ptr(out_i8), ldc_out_i8,
              float(np.float32(out_scale)), int(i8_layout))


def mean_hw(x, n, hw, c, ldc, out_f32=None, out_i8=None, ld_i8=0, out_scale=1.0) -> None:
    _lib.call("mira_cuda_mean_hw_nhwc", ptr(x), n, hw, c, ldc, ptr(out_f32), ptr(out_i8), ld_i8,
              float(np.float32(out_scale)))


def dwconv2d(x, n, h, w, c, wt, kh, kw, stride, padding, dilation, epi: Epi) -> None:
    e = epi.struct()
    _lib.call("mira_cuda_dwconv2d_nhwc", ptr(x), n, h, w, c, ptr(wt), kh, kw, stride[0], stride[1],
              padding[0], padding[1], dilation[0], dilation[1], C.byref(e))


def qdwconv2d(x, ldx, n, h, w, c, wq, kh, kw, stride, padding, dilation, dq, epi: Epi) -> None:
    """Opt-in int8 depthwise conv: x int8 NHWC (pixels ldx bytes apart), wq int8 [kh * kw, c]."""
    e = epi.struct()
    _lib.call("mira_cuda_qdwconv2d_nhwc", ptr(x), n, h, w, c, ldx, ptr(wq), kh, kw, stride[0], stride[1],
              padding[0], padding[1], dilation[0], dilation[1], C.byref(dq), C.byref(e))


def elementwise_f32(op: str, shape4, a: View, out: View, b: Optional[View] = None, scalar: float = 0.0,
                    swapped: bool = False) -> None:
    """out = op(a) (unary) or op(a, b-or-scalar) (op(b, a) when swapped) over a 4-D shape."""
    code = _lib.UNARY_CODES.get(op) or _lib.BINARY_CODES.get(op)
    if code is None:
        raise ValueError(f"no element-wise kernel for {op}")
    av, ov = a.struct(), out.struct()
    bv = b.struct() if b is not None else None
    n = tuple(int(d) for d in shape4)
    _lib.call("mira_cuda_elementwise_f32", code, *n, C.byref(av), C.byref(bv) if bv is not None else None,
              float(np.float32(scalar)), int(bool(swapped)), C.byref(ov))


def im2col_f32(x, n: int, h: int, w: int, c: int, ldc: int, kh: int, kw: int, stride, padding, dilation, out,
               ld_out: int) -> None:
    """Patch matrix [n * oh * ow, kh * kw * c] of an NHWC f32 input (column (i * kw + j) * c + ch)."""
    _lib.call("mira_cuda_im2col_f32", ptr(x), n, h, w, c, ldc, kh, kw, stride[0], stride[1], padding[0], padding[1],
              dilation[0], dilation[1], ptr(out), ld_out)


def nchw_to_nhwc(x, n, c, h, w, y, ldc) -> None:
    _lib.call("mira_cuda_nchw_to_nhwc_f32", ptr(x), n, c, h, w, ptr(y), ldc)


def nhwc_to_nchw(x, n, h, w, c, ldc, y) -> None:
    _lib.call("mira_cuda_nhwc_to_nchw_f32", ptr(x), n, h, w, c, ldc, ptr(y))


# ----------------------------------------------------------------------------- sequence (transformer) ops

@dataclass
class View:
    """A view of at most 4 dimensions for the sequence kernels: buffer `buf` (a DeviceBuffer or
    DeviceSlice), element `offset` and element `strides` over (batch0, batch1, row, col); broadcast
    dimensions have stride 0."""
    buf: object
    strides: tuple
    offset: int = 0
    itemsize: int = 4

    def struct(self) -> _lib.View4:
        v = _lib.View4()
        if self.buf is not None:
            v.ptr = (ptr(self.buf).value or 0) + int(self.offset) * self.itemsize
        for i, s in enumerate(self.strides):
            v.stride[i] = int(s)
        return v


@dataclass
class BmmStep:
    """One epilogue step of the batched f32 matmul: operand "none", "scalar" or "view"."""
    op: str
    operand: str = "none"
    swapped: bool = False
    scalar: float = 0.0
    view: Optional[View] = None


_BMM_OPND = {"none": _lib.OPND_NONE, "scalar": _lib.OPND_SCALAR, "view": _lib.OPND_VIEW}


@dataclass
class BmmEpi:
    steps: Sequence[BmmStep] = field(default_factory=list)
    out: Optional[View] = None
    out_i8: Optional[View] = None
    out_scale: float = 1.0

    def struct(self) -> _lib.BmmEpilogue:
        e = _lib.BmmEpilogue()
        if len(self.steps) > _lib.EPI_MAX_STEPS:
            raise ValueError(f"at most {_lib.EPI_MAX_STEPS} fused epilogue steps")
        e.n_steps = len(self.steps)
        for i, s in enumerate(self.steps):
            code = _lib.UNARY_CODES.get(s.op) or _lib.BINARY_CODES.get(s.op)
            if code is None:
                raise ValueError(f"epilogue op {s.op!r} has no device implementation")
            e.steps[i].op = code
            e.steps[i].operand = _BMM_OPND[s.operand]
            e.steps[i].swapped = int(bool(s.swapped))
            e.steps[i].scalar = float(np.float32(s.scalar))
            if s.view is not None:
                e.steps[i].view = s.view.struct()
        if self.out is not None:
            e.out_f32 = self.out.struct()
        if self.out_i8 is not None:
            e.out_i8 = self.out_i8.struct()
        e.out_scale = float(np.float32(self.out_scale))
        return e


def bmm_f32(batch0: int, batch1: int, m: int, n: int, k: int, a: View, b: View, epi: BmmEpi) -> None:
    av, bv, e = a.struct(), b.struct(), epi.struct()
    _lib.call("mira_cuda_bmm_f32", batch0, batch1, m, n, k, C.byref(av), C.byref(bv), C.byref(e))


def dims4(shape) -> "C.Array":
    """A shape of at most 4 dimensions padded with leading 1s, as the int64[4] the C-ABI takes."""
    shape = tuple(int(d) for d in shape)
    if len(shape) > 4:
        raise ValueError("at most 4 dimensions")
    return (C.c_int64 * 4)(*((1,) * (4 - len(shape)) + shape))


def dynamic_slice(x: View, x_shape, start, rank: int, size, out: View) -> None:
    """out = x[start : start + size] with the start vector (int32, `rank` entries) in device memory."""
    xv, ov = x.struct(), out.struct()
    _lib.call("mira_cuda_dynamic_slice", C.byref(xv), dims4(x_shape), ptr(start), rank, dims4(size), C.byref(ov))


def dynamic_update_slice(x: View, x_shape, upd: View, upd_shape, start, rank: int) -> None:
    """x[start : start + upd_shape] = upd in place, start vector in device memory."""
    xv, uv = x.struct(), upd.struct()
    _lib.call("mira_cuda_dynamic_update_slice", C.byref(xv), dims4(x_shape), C.byref(uv), dims4(upd_shape),
              ptr(start), rank)


def bmm_f32_w8(batch0: int, batch1: int, m: int, n: int, k: int, a: View, b_i8: View, b_scale, epi: BmmEpi) -> None:
    """bmm_f32 with int8 weights: b_i8 views q (itemsize 1), b_scale holds one f32 scale per column."""
    av, bv, e = a.struct(), b_i8.struct(), epi.struct()
    _lib.call("mira_cuda_bmm_f32_w8", batch0, batch1, m, n, k, C.byref(av), C.byref(bv), ptr(b_scale), C.byref(e))


def layernorm_rows(x, rows: int, d: int, ld_x: int, gamma, beta, eps: float, out_f32=None, ld_f32: int = 0,
                   out_i8=None, ld_i8: int = 0, out_scale: float = 1.0) -> None:
    _lib.call("mira_cuda_layernorm_rows", ptr(x), rows, d, ld_x, ptr(gamma), ptr(beta), float(np.float32(eps)),
              ptr(out_f32), ld_f32, ptr(out_i8), ld_i8, float(np.float32(out_scale)))


def softmax_rows(x, rows: int, n: int, ld_x: int, out, ld_out: int) -> None:
    _lib.call("mira_cuda_softmax_rows", ptr(x), rows, n, ld_x, ptr(out), ld_out)


def embed_rows(table, vocab: int, d: int, idx, rows: int, out, ld_out: int, addend=None, addend_rows: int = 0) -> None:
    _lib.call("mira_cuda_embed_rows", ptr(table), vocab, d, ptr(idx), rows, ptr(addend), addend_rows, ptr(out), ld_out)


def copy_view(shape4, src: View, dst: View) -> None:
    s, d = src.struct(), dst.struct()
    n0, n1, n2, n3 = (int(x) for x in shape4)
    _lib.call("mira_cuda_copy_view_f32", n0, n1, n2, n3, C.byref(s), C.byref(d))


ATT_TILE = 64    # query and key rows per attention tile


@dataclass
class Attn:
    """Descriptor of one fused attention launch (mira_attention): q/k/v views with keys as rows,
    the scale step ("mul"/"div" or None), an optional mask view, tile maxima and a device scalar
    max|k| for exact tile skipping, and f32 / int8 outputs."""
    batch0: int
    batch1: int
    tq: int
    tk: int
    dh: int
    q: View
    k: View
    v: View
    scale_op: Optional[str] = None
    scale: float = 1.0
    mask: Optional[View] = None
    tile_max: object = None
    kmax: object = None
    tile_zero: object = None
    out: Optional[View] = None
    out_i8: Optional[View] = None
    out_scale: float = 1.0
    workspace: object = None      # scratch of attention_workspace() bytes: the tensor-core path
    workspace_bytes: int = 0

    def struct(self) -> _lib.Attention:
        a = _lib.Attention()
        a.batch0, a.batch1, a.tq, a.tk, a.dh = (int(x) for x in (self.batch0, self.batch1, self.tq, self.tk, self.dh))
        a.q, a.k, a.v = self.q.struct(), self.k.struct(), self.v.struct()
        a.scale_op = {None: 0, "mul": _lib.EPI_MUL, "div": _lib.EPI_DIV}[self.scale_op]
        a.scale = float(np.float32(self.scale))
        if self.mask is not None:
            a.mask = self.mask.struct()
        a.tile_max = ptr(self.tile_max).value or 0
        a.kmax = ptr(self.kmax).value or 0
        a.tile_zero = ptr(self.tile_zero).value or 0
        if self.out is not None:
            a.out_f32 = self.out.struct()
        if self.out_i8 is not None:
            a.out_i8 = self.out_i8.struct()
        a.out_scale = float(np.float32(self.out_scale))
        a.workspace = ptr(self.workspace).value or 0
        a.workspace_bytes = int(self.workspace_bytes)
        return a


def mask_tile_max(mask: np.ndarray, tq: int, tk: int) -> np.ndarray:
    """Maximum of each ATT_TILE x ATT_TILE tile of a [tq, tk] mask, [ceil(tq/64), ceil(tk/64)] f32."""
    nq, nk = -(-tq // ATT_TILE), -(-tk // ATT_TILE)
    padded = np.full((nq * ATT_TILE, nk * ATT_TILE), -np.inf, np.float32)
    padded[:tq, :tk] = np.broadcast_to(np.asarray(mask, np.float32), (tq, tk))
    return padded.reshape(nq, ATT_TILE, nk, ATT_TILE).max(axis=(1, 3)).astype(np.float32)


def mask_tile_zero(mask: np.ndarray, tq: int, tk: int) -> np.ndarray:
    """1 for each ATT_TILE x ATT_TILE tile of a [tq, tk] mask whose entries are all +0.0, as uint8."""
    nq, nk = -(-tq // ATT_TILE), -(-tk // ATT_TILE)
    m = np.broadcast_to(np.asarray(mask, np.float32), (tq, tk))
    plus_zero = (m == 0) & ~np.signbit(m)
    padded = np.ones((nq * ATT_TILE, nk * ATT_TILE), bool)
    padded[:tq, :tk] = plus_zero
    return padded.reshape(nq, ATT_TILE, nk, ATT_TILE).all(axis=(1, 3)).astype(np.uint8)


def attention_workspace(batch0: int, batch1: int, tq: int, tk: int, dh: int) -> int:
    """Bytes of scratch for the tensor-core attention path (0: the f32 kernel takes the shape)."""
    return int(_lib.load().mira_cuda_attention_workspace(batch0, batch1, tq, tk, dh))


def attention_f32(desc: Attn) -> None:
    a = desc.struct()
    _lib.call("mira_cuda_attention_f32", C.byref(a))


def collapse_view(shape, strides) -> tuple[tuple, tuple]:
    """An equivalent view of at most 4 dimensions with the fewest dimensions, for reductions whose
    result does not depend on element order (dimensions reordered by stride and merged where
    contiguous with each other), padded with leading size-1 dimensions."""
    dims = sorted(((int(n), int(st)) for n, st in zip(shape, strides) if int(n) != 1), key=lambda t: -abs(t[1]))
    out: list = []
    for n, st in dims:
        if out and out[-1][1] == st * n:
            out[-1] = (out[-1][0] * n, st)
        else:
            out.append((n, st))
    out = [(1, 0)] * (4 - len(out)) + out
    return tuple(n for n, _ in out), tuple(st for _, st in out)


def absmax_f32(shape4, x: View, out) -> None:
    xv = x.struct()
    n0, n1, n2, n3 = (int(v) for v in shape4)
    _lib.call("mira_cuda_absmax_f32", n0, n1, n2, n3, C.byref(xv), ptr(out))
