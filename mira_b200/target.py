"""The `cuda` target: MIRA's Target/Executable protocol (reference mira/backends/base.py:13-26) on
B200 kernels.

`CudaTarget.check(op)` decides placement (reference partition.py:73-80): every quantized op is
accepted, plus the f32 ops that sit between them on the W8A8 path (max pooling and its -inf pad,
the global mean, depthwise convolutions, reshapes).  `CudaTarget.compile(g)` plans a segment
graph once: it chooses a device representation for every value (int8 and/or f32, NHWC for 4-D
tensors, row-major otherwise), uploads the constants (K-major int8 weights, split dequant scales,
padded epilogue operands) and records one kernel launch per op.  `CudaExecutable.run(feeds)`
then does host->device copies, the launches (replayed from a CUDA graph after the first run) and
device->host copies, and returns NumPy arrays like the reference's CPUExecutable (cpu.py:28-36).

All device work goes through a `device` object (CudaDevice here), so the planning logic can also
be driven by a host-side stand-in.
"""
from __future__ import annotations

import ctypes as C
import os
import time
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import _lib
from . import kernels as K
from .device import DeviceBuffer, PinnedBuffer, ptr, set_device

QOPS = ("qmatmul", "qconv2d")


# ============================================================================ device access

@dataclass
class Launch:
    """One kernel launch of the plan: `kind` names a libmira_cuda entry point family."""
    kind: str
    args: dict


class CudaDevice:
    """Executes a plan on one GPU through libmira_cuda.so."""

    name = "cuda"

    def __init__(self, index: int = 0):
        self.index = int(index)
        set_device(self.index)
        self._lib = _lib.load()

    def activate(self) -> None:
        set_device(self.index)

    def alloc(self, nbytes: int, zero: bool = False) -> DeviceBuffer:
        return DeviceBuffer(nbytes, zero=zero)

    def upload(self, arr: np.ndarray) -> DeviceBuffer:
        return DeviceBuffer.from_array(np.ascontiguousarray(arr))

    def pinned(self, nbytes: int) -> PinnedBuffer:
        return PinnedBuffer(nbytes)

    def h2d(self, dst, src: PinnedBuffer, nbytes: int) -> None:
        _lib.call("mira_cuda_h2d", ptr(dst), ptr(src), C.c_size_t(nbytes))

    def d2h(self, dst: PinnedBuffer, src, nbytes: int) -> None:
        _lib.call("mira_cuda_d2h", ptr(dst), ptr(src), C.c_size_t(nbytes))

    def sync(self) -> None:
        _lib.call("mira_cuda_sync")

    def graph_begin(self) -> None:
        _lib.call("mira_cuda_graph_begin")

    def graph_end(self):
        g = C.c_void_p()
        _lib.call("mira_cuda_graph_end", C.byref(g))
        return g

    def graph_launch(self, g) -> None:
        _lib.call("mira_cuda_graph_launch", g)

    def graph_destroy(self, g) -> None:
        _lib.call("mira_cuda_graph_destroy", g)

    def thunk(self, launch: Launch):
        """Pre-builds the C arguments of a launch; returns a zero-argument callable."""
        a = launch.args
        L = self._lib
        keep = []
        k = launch.kind
        if k == "quantize_rows":
            fn = L.mira_cuda_quantize_rows
            args = (ptr(a["x"]), a["rows"], a["cols"], a["ld_x"], float(np.float32(a["scale"])), ptr(a["xq"]), a["ld_q"])
        elif k == "quantize_nchw":
            fn = L.mira_cuda_quantize_nchw_to_nhwc
            args = (ptr(a["x"]), a["n"], a["c"], a["h"], a["w"], float(np.float32(a["scale"])), ptr(a["xq"]), a["cp"])
        elif k == "quantize_row4":
            fn = L.mira_cuda_quantize_nchw_to_row4
            args = (ptr(a["x"]), a["n"], a["c"], a["h"], a["w"], float(np.float32(a["scale"])), ptr(a["xq"]),
                    a["row_entries"], a["pad"])
        elif k == "nchw_to_nhwc":
            fn = L.mira_cuda_nchw_to_nhwc_f32
            args = (ptr(a["x"]), a["n"], a["c"], a["h"], a["w"], ptr(a["y"]), a["ldc"])
        elif k == "nhwc_to_nchw":
            fn = L.mira_cuda_nhwc_to_nchw_f32
            args = (ptr(a["x"]), a["n"], a["h"], a["w"], a["c"], a["ldc"], ptr(a["y"]))
        elif k in ("qgemm", "qconv2d", "qconv2d_pool"):
            dq = K.dequant_channel(*a["dq"]) if len(a["dq"]) == 3 else K.dequant_rowcol(*a["dq"])
            e = a["epi"].struct()
            keep += [dq, e]
            if k == "qgemm":
                fn = L.mira_cuda_qgemm
                args = (a["M"], a["N"], a["K"], ptr(a["A"]), a["lda"], ptr(a["B"]), a["ldb"], C.byref(dq), C.byref(e))
            elif k == "qconv2d_pool":
                fn = L.mira_cuda_qconv2d_maxpool
                (sh, sw), (ph, pw), (dh, dw) = a["stride"], a["padding"], a["dilation"]
                args = (a["n"], a["h"], a["w"], a["cp"], ptr(a["x"]), a["layout"], a["row_entries"], a["o"], a["kh"],
                        a["kw"], ptr(a["wq"]), a["ldw"], sh, sw, ph, pw, dh, dw, a["pool_size"], a["pool_stride"],
                        a["pool_pad"],
                        float(np.float32(a["pool_pad_value"])), C.byref(dq), C.byref(e))
            else:
                fn = L.mira_cuda_qconv2d
                (sh, sw), (ph, pw), (dh, dw) = a["stride"], a["padding"], a["dilation"]
                args = (a["n"], a["h"], a["w"], a["cp"], ptr(a["x"]), a["layout"], a["row_entries"], a["o"], a["kh"],
                        a["kw"], ptr(a["wq"]), a["ldw"], sh, sw, ph, pw, dh, dw, C.byref(dq), C.byref(e))
        elif k == "maxpool":
            fn = L.mira_cuda_maxpool2d_nhwc
            args = (ptr(a.get("x_f32")), ptr(a.get("x_i8")), a["n"], a["h"], a["w"], a["c"], a["ldc"], a["size"],
                    a["stride"], a["pad"], float(np.float32(a["pad_value"])), ptr(a.get("out_f32")), a.get("ldo", 0),
                    ptr(a.get("out_i8")), a.get("ldo_i8", 0), float(np.float32(a.get("scale", 1.0))))
        elif k == "mean_hw":
            fn = L.mira_cuda_mean_hw_nhwc
            args = (ptr(a["x"]), a["n"], a["hw"], a["c"], a["ldc"], ptr(a.get("out_f32")), ptr(a.get("out_i8")),
                    a.get("ld_i8", 0), float(np.float32(a.get("scale", 1.0))))
        elif k == "dwconv":
            e = a["epi"].struct()
            keep.append(e)
            fn = L.mira_cuda_dwconv2d_nhwc
            (sh, sw), (ph, pw), (dh, dw) = a["stride"], a["padding"], a["dilation"]
            args = (ptr(a["x"]), a["n"], a["h"], a["w"], a["c"], ptr(a["wt"]), a["kh"], a["kw"], sh, sw, ph, pw, dh, dw,
                    C.byref(e))
        elif k == "copy":
            fn = L.mira_cuda_d2d
            args = (ptr(a["dst"]), ptr(a["src"]), C.c_size_t(a["nbytes"]))
        else:
            raise ValueError(f"unknown launch kind {k!r}")

        def run(fn=fn, args=args, keep=keep, name=k):
            rc = fn(*args)
            if rc != _lib.OK:
                raise _lib.CudaError(rc, f"{name}: {_lib.last_error()}")
        return run


# ============================================================================ planning

@dataclass
class DVal:
    """Device representation of one IR value.  `shape` is the reference shape (NCHW for 4-D).
    layout "nhwc": 4-D tensors stored channels-last; "rows": row-major [prod(shape[:-1]), shape[-1]]."""
    shape: tuple
    layout: str
    f32: object = None
    i8: object = None
    i8_scale: Optional[float] = None
    i8_ld: int = 0
    i8_layout: str = "nhwc"      # or "row4" (MIRA_LAYOUT_ROW4, graph inputs of at most 4 channels)
    row_entries: int = 0

    @property
    def rows(self) -> int:
        if self.layout == "nhwc":
            n, _, h, w = self.shape
            return n * h * w
        return int(np.prod(self.shape[:-1], dtype=np.int64)) if len(self.shape) > 1 else 1

    @property
    def cols(self) -> int:
        if self.layout == "nhwc":
            return self.shape[1]
        return self.shape[-1] if self.shape else 1

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64))


def _layout_for(shape) -> str:
    return "nhwc" if len(shape) == 4 else "rows"


def _f32(scale) -> float:
    return float(np.float32(scale))


class UnsupportedOnCuda(NotImplementedError):
    pass


def conv_attrs(a: dict):
    """(stride, padding, dilation, groups) with the reference's defaults (ops.py conv_params)."""
    return tuple(a["stride"]), tuple(a["padding"]), tuple(a.get("dilation", (1, 1))), a.get("groups", 1)


def _pad_hw(op) -> Optional[tuple[int, float]]:
    """(p, value) if `op` is a constant pad of H and W only, by the same p on every side."""
    pads = tuple(tuple(p) for p in op.attrs["pads"])
    if len(pads) != 4 or pads[0] != (0, 0) or pads[1] != (0, 0):
        return None
    (a, b), (c, d) = pads[2], pads[3]
    if not (a == b == c == d) or a < 0:
        return None
    return a, float(np.float32(np.asarray(op.attrs.get("value", 0)).astype(np.float32)))


class Plan:
    """Device buffers and launches for one segment graph.  fuse_pool: run a qconv2d whose only
    consumer is a max pool inside the pooling kernel (mira_cuda_qconv2d_maxpool)."""

    def __init__(self, g, device, fuse_pool: bool = False):
        self.g = g
        self.dev = device
        self.fuse_pool = fuse_pool
        self.vals: dict = {}
        self.launches: list[Launch] = []
        self.inputs: list = []       # (value, device buffer in reference layout, nbytes)
        self.outputs: list = []      # (value, device buffer in reference layout, nbytes)
        self.const_outputs: dict = {}
        self.keep: list = []         # constant uploads
        self.skipped: set = set()
        self.kernel_counts: dict = {}
        self._build()

    # ------------------------------------------------------------------ helpers

    def _alloc(self, nbytes: int, zero: bool = False):
        return self.dev.alloc(int(nbytes), zero=zero)

    def _upload(self, arr: np.ndarray):
        buf = self.dev.upload(arr)
        self.keep.append(buf)
        return buf

    def _launch(self, kind: str, **args) -> None:
        self.launches.append(Launch(kind, args))
        self.kernel_counts[kind] = self.kernel_counts.get(kind, 0) + 1

    def _const(self, v) -> Optional[np.ndarray]:
        p = v.producer
        if p is not None and p.kind == "const":
            return np.asarray(p.attrs["value"])
        if p is not None and p.kind == "dequantize":
            from .hostfw import import_mira
            import_mira()
            from mira import ops as O
            return np.asarray(O.evaluate("dequantize", [], p.attrs))
        return None

    # ------------------------------------------------------------------ requirements

    def _requirements(self):
        g = self.g
        users = g.users()
        self.users = users
        self.pad_into_pool = {}      # maxpool op -> (source value, pad, pad value)
        self.conv_into_pool = {}     # maxpool op -> qconv2d op computed inside the pooling kernel
        for op in g.ops:
            if op.kind != "maxpool2d":
                continue
            src = op.inputs[0]
            pad_op = src.producer
            if (pad_op is not None and pad_op.kind == "pad" and _pad_hw(pad_op) is not None
                    and users.get(src, []) == [op] and src not in g.outputs):
                p, val = _pad_hw(pad_op)
                self.pad_into_pool[op] = (pad_op.inputs[0], p, val)
                self.skipped.add(pad_op)
                src = pad_op.inputs[0]
            conv = src.producer
            pad_ok = op not in self.pad_into_pool or self.pad_into_pool[op][2] == float("-inf")
            if (self.fuse_pool and pad_ok and conv is not None and conv.kind == "qconv2d"
                    and len(users.get(src, [])) == 1 and src not in g.outputs and self._conv_pool_fusable(conv)):
                self.conv_into_pool[op] = conv
                self.skipped.add(conv)
        fused_convs = set(self.conv_into_pool.values())
        need_f32, i8_req = set(), {}
        for op in g.ops:
            if op.is_constant_like or (op in self.skipped and op not in fused_convs):
                continue
            if op.kind in QOPS:
                x = op.inputs[0]
                s = _f32(op.attrs["x_scale"])
                if x in i8_req and i8_req[x] != s:
                    need_f32.add(x)      # a second scale is quantized from f32 separately
                else:
                    i8_req.setdefault(x, s)
                for v in op.inputs[1:]:
                    need_f32.add(v)
            elif op.kind == "maxpool2d" and op in self.conv_into_pool:
                pass
            elif op.kind == "maxpool2d" and op in self.pad_into_pool:
                need_f32.add(self.pad_into_pool[op][0])
            else:
                for v in op.inputs:
                    need_f32.add(v)
        need_f32.update(g.outputs)
        self.need_f32 = {v for v in need_f32 if self._const(v) is None}
        self.i8_req = i8_req

    def _conv_pool_fusable(self, conv) -> bool:
        """A qconv2d whose only consumer is a max pool can run inside the pooling kernel when it has
        at most 64 output channels and its epilogue is monotone non-decreasing (relu, and add /
        non-swapped sub / maximum / minimum of constant scalars or per-channel values): the kernel
        pools the int32 accumulators and applies the epilogue to the pooled values."""
        _, _, _, groups = conv_attrs(conv.attrs)
        o = np.asarray(conv.attrs["q"]).shape[0]
        if groups != 1 or o > 64:
            return False
        probe = DVal(tuple(conv.result.type.shape), "nhwc")
        for fn, idx, swapped in conv.attrs.get("epilogue", ()):
            if idx is None:
                if fn != "relu":
                    return False
                continue
            if fn not in ("add", "maximum", "minimum", "sub") or (fn == "sub" and swapped):
                return False
            val = self._const(conv.inputs[idx])
            if val is None or not (val.size == 1 or self._is_channel(val.shape, probe)):
                return False
        return True

    # ------------------------------------------------------------------ build

    def _build(self):
        self._requirements()
        for v in self.g.inputs:
            self._input(v)
        for op in self.g.ops:
            if op.is_constant_like or op in self.skipped:
                continue
            fn = getattr(self, "_op_" + op.kind, None)
            if fn is None:
                raise UnsupportedOnCuda(f"{op.kind} has no cuda kernel")
            fn(op)
        for v in self.g.outputs:
            self._output(v)

    def _new_out(self, v, layout: Optional[str] = None) -> DVal:
        shape = tuple(v.type.shape)
        dv = DVal(shape, layout or _layout_for(shape))
        if v in self.need_f32:
            dv.f32 = self._alloc(dv.numel * 4)
        if v in self.i8_req:
            dv.i8_scale = self.i8_req[v]
            dv.i8_ld = K.round_up(dv.cols, 16)
            dv.i8 = self._alloc(dv.rows * dv.i8_ld, zero=True)
        self.vals[v] = dv
        return dv

    def _from_reference_order(self, v, buf) -> DVal:
        """A DVal for `v` from an f32 buffer in the reference's element order (NCHW / row-major)."""
        shape = tuple(v.type.shape)
        dv = DVal(shape, _layout_for(shape))
        if dv.layout == "nhwc":
            n, c, h, w = shape
            if v in self.need_f32:
                if h * w == 1:
                    dv.f32 = buf
                else:
                    dv.f32 = self._alloc(dv.numel * 4)
                    self._launch("nchw_to_nhwc", x=buf, n=n, c=c, h=h, w=w, y=dv.f32, ldc=c)
            if v in self.i8_req:
                row4 = self._row4_geometry(v)
                dv.i8_scale = self.i8_req[v]
                if row4 is not None:
                    entries, pad = row4
                    dv.i8, dv.i8_layout, dv.row_entries, dv.i8_ld = self._alloc(n * h * entries * 16), "row4", entries, 4
                    self._launch("quantize_row4", x=buf, n=n, c=c, h=h, w=w, scale=dv.i8_scale, xq=dv.i8,
                                 row_entries=entries, pad=pad)
                else:
                    cp = 4 if c <= 4 else K.round_up(c, 16)
                    dv.i8, dv.i8_ld = self._alloc(n * h * w * cp, zero=True), cp
                    self._launch("quantize_nchw", x=buf, n=n, c=c, h=h, w=w, scale=dv.i8_scale, xq=dv.i8, cp=cp)
        else:
            dv.f32 = buf
            if v in self.i8_req:
                dv.i8_scale, dv.i8_ld = self.i8_req[v], K.round_up(dv.cols, 16)
                dv.i8 = self._alloc(dv.rows * dv.i8_ld, zero=True)
                self._launch("quantize_rows", x=buf, rows=dv.rows, cols=dv.cols, ld_x=dv.cols, scale=dv.i8_scale,
                             xq=dv.i8, ld_q=dv.i8_ld)
        self.vals[v] = dv
        return dv

    def _row4_geometry(self, v):
        """(entries, pad) when every consumer of the int8 value of `v` is a convolution that can read
        the row-expanded layout (at most 4 channels, kernel width <= 8, no dilation) with one common
        horizontal geometry; None otherwise."""
        if v.type.shape[1] > 4:
            return None
        geo = None
        for op in self.users.get(v, []):
            if op.kind != "qconv2d":
                if op.kind in QOPS:
                    return None
                continue
            stride, padding, dilation, groups = conv_attrs(op.attrs)
            kw = np.asarray(op.attrs["q"]).shape[3]
            if groups != 1 or kw > 8 or tuple(dilation) != (1, 1) or op.inputs[0] is not v:
                return None
            ow = op.result.type.shape[3]
            g = (K.row4_entries(ow, stride[1]), padding[1])
            if geo is not None and g != geo:
                return None
            geo = g
        return geo

    def _conv_input(self, v, scale: float):
        """(int8 buffer, channels per pixel, layout code, entries per row) of a conv input."""
        dv = self.vals[v]
        if dv.i8 is not None and dv.i8_scale == scale and dv.i8_layout == "row4":
            return dv.i8, 4, _lib.LAYOUT_ROW4, dv.row_entries
        buf, cp = self._i8_of(v, scale)
        return buf, cp, _lib.LAYOUT_NHWC, 0

    def _conv_weight(self, q, cp: int, layout: int) -> np.ndarray:
        if layout == _lib.LAYOUT_ROW4:
            return K.conv_weight_row4(q)
        return K.conv_weight(q, cp)[0]

    def _i8_of(self, v, scale: float):
        """(int8 buffer, row stride) of `v` quantized with `scale`."""
        dv = self.vals[v]
        if dv.i8 is not None and dv.i8_scale == scale and dv.i8_layout == "nhwc":
            return dv.i8, dv.i8_ld
        if dv.f32 is None:
            raise UnsupportedOnCuda("int8 operand without an f32 source")
        ld = K.round_up(dv.cols, 16)
        buf = self._alloc(dv.rows * ld, zero=True)
        self._launch("quantize_rows", x=dv.f32, rows=dv.rows, cols=dv.cols, ld_x=dv.cols, scale=scale, xq=buf, ld_q=ld)
        if dv.i8 is None:
            dv.i8, dv.i8_scale, dv.i8_ld = buf, scale, ld
        return buf, ld

    def _input(self, v) -> None:
        if v.type.dtype != "f32":
            raise UnsupportedOnCuda(f"input {v!r} is {v.type.dtype}; the cuda target takes f32 inputs")
        nbytes = v.type.numel * 4
        raw = self._alloc(nbytes)
        self.inputs.append((v, raw, nbytes))
        self._from_reference_order(v, raw)

    def _output(self, v) -> None:
        c = self._const(v)
        if c is not None:
            self.const_outputs[v] = c.astype(v.type.np_dtype)
            return
        dv = self.vals[v]
        nbytes = dv.numel * 4
        if dv.layout == "nhwc" and dv.shape[2] * dv.shape[3] > 1:
            n, ch, h, w = dv.shape
            buf = self._alloc(nbytes)
            self._launch("nhwc_to_nchw", x=dv.f32, n=n, h=h, w=w, c=ch, ldc=ch, y=buf)
        else:
            buf = dv.f32
        self.outputs.append((v, buf, nbytes))

    # ------------------------------------------------------------------ epilogue operands

    def _epilogue(self, op, out: DVal, operand_base: int = 0) -> K.Epi:
        steps = []
        for fn, idx, swapped in op.attrs.get("epilogue", ()):
            if idx is None:
                steps.append(K.Step(fn))
            else:
                steps.append(self._operand_step(fn, bool(swapped), op.inputs[idx], out))
        return K.Epi(steps, out_f32=out.f32, ld_f32=out.cols, out_i8=out.i8, ld_i8=out.i8_ld,
                     out_scale=out.i8_scale if out.i8 is not None else 1.0)

    def _operand_step(self, fn: str, swapped: bool, v, out: DVal) -> K.Step:
        val = self._const(v)
        oshape = out.shape
        if val is not None:
            val = val.astype(np.float32)
            if val.size == 1:
                return K.Step(fn, "scalar", swapped, scalar=float(val.ravel()[0]))
            if self._is_channel(val.shape, out):
                return K.Step(fn, "channel", swapped, ptr=self._upload(K.pad_channels(val.ravel())))
            full = np.broadcast_to(val, oshape)
            if out.layout == "nhwc":
                full = full.transpose(0, 2, 3, 1)
            return K.Step(fn, "full", swapped, ptr=self._upload(np.ascontiguousarray(full, np.float32)), ld=out.cols)
        dv = self.vals[v]
        if dv.f32 is None:
            raise UnsupportedOnCuda("epilogue operand has no f32 representation")
        if tuple(dv.shape) == tuple(oshape) and dv.layout == out.layout:
            return K.Step(fn, "full", swapped, ptr=dv.f32, ld=dv.cols)
        if self._is_channel(dv.shape, out):
            padded = self._alloc(K.round_up(max(out.cols, 1), K.CHANNEL_PAD) * 4, zero=True)
            self._launch("copy", dst=padded, src=dv.f32, nbytes=out.cols * 4)
            return K.Step(fn, "channel", swapped, ptr=padded)
        raise UnsupportedOnCuda(f"runtime epilogue operand of shape {list(dv.shape)} against {list(oshape)}")

    @staticmethod
    def _is_channel(shape, out: DVal) -> bool:
        shape = tuple(shape)
        if out.layout == "nhwc":
            s4 = (1,) * (4 - len(shape)) + shape
            return len(shape) <= 4 and s4[0] == 1 and s4[2] == 1 and s4[3] == 1 and s4[1] == out.shape[1]
        nd = len(out.shape)
        s = (1,) * (nd - len(shape)) + shape
        return len(shape) <= nd and s[-1] == out.shape[-1] and all(d == 1 for d in s[:-1])

    # ------------------------------------------------------------------ ops

    def _scales(self, x_scale: float, w_scale: np.ndarray):
        s64, hi, lo = K.scale_arrays(x_scale, w_scale)
        return self._upload(s64), self._upload(hi), self._upload(lo)

    def _op_qmatmul(self, op) -> None:
        a = op.attrs
        x = self.vals[op.inputs[0]]
        if x.layout != "rows":
            raise UnsupportedOnCuda("qmatmul on a 4-D input")
        q = np.asarray(a["q"])
        kdim, n = q.shape
        A, lda = self._i8_of(op.inputs[0], _f32(a["x_scale"]))
        wq = self._upload(K.matmul_weight(q))
        out = self._new_out(op.result)
        self._launch("qgemm", M=x.rows, N=n, K=kdim, A=A, lda=lda, B=wq, ldb=K.round_up(kdim, 16),
                     dq=self._scales(a["x_scale"], a["w_scale"]), epi=self._epilogue(op, out))

    def _op_qconv2d(self, op) -> None:
        a = op.attrs
        stride, padding, dilation, groups = conv_attrs(a)
        if groups != 1:
            raise UnsupportedOnCuda("grouped qconv2d")
        x = self.vals[op.inputs[0]]
        n, c, h, w = x.shape
        q = np.asarray(a["q"])
        o, _, kh, kw = q.shape
        xi8, cp, layout, entries = self._conv_input(op.inputs[0], _f32(a["x_scale"]))
        wq = self._conv_weight(q, cp, layout)
        out = self._new_out(op.result, "nhwc")
        self._launch("qconv2d", n=n, h=h, w=w, cp=cp, x=xi8, layout=layout, row_entries=entries, o=o, kh=kh, kw=kw,
                     wq=self._upload(wq), ldw=wq.shape[1], stride=stride, padding=padding, dilation=dilation,
                     dq=self._scales(a["x_scale"], a["w_scale"]), epi=self._epilogue(op, out))

    def _op_conv2d(self, op) -> None:
        stride, padding, dilation, groups = conv_attrs(op.attrs)
        x = self.vals[op.inputs[0]]
        n, c, h, w = x.shape
        wt = self._const(op.inputs[1])
        if wt is None or groups != c or wt.shape[0] != c or wt.shape[1] != 1:
            raise UnsupportedOnCuda("only depthwise f32 conv2d with constant weights runs on cuda")
        kh, kw = wt.shape[2:]
        wtap = np.ascontiguousarray(wt[:, 0].reshape(c, kh * kw).T.astype(np.float32))
        out = self._new_out(op.result, "nhwc")
        self._launch("dwconv", x=x.f32, n=n, h=h, w=w, c=c, wt=self._upload(wtap), kh=kh, kw=kw, stride=stride,
                     padding=padding, dilation=dilation, epi=self._epilogue(op, out))

    def _op_maxpool2d(self, op) -> None:
        if op in self.pad_into_pool:
            src, pad, pad_value = self.pad_into_pool[op]
        else:
            src, pad, pad_value = op.inputs[0], 0, float("-inf")
        if op in self.conv_into_pool:
            self._conv_pool(op, self.conv_into_pool[op], pad, pad_value)
            return
        x = self.vals[src]
        n, c, h, w = x.shape
        out = self._new_out(op.result, "nhwc")
        self._launch("maxpool", x_f32=x.f32, n=n, h=h, w=w, c=c, ldc=c, size=op.attrs["size"],
                     stride=op.attrs["stride"], pad=pad, pad_value=pad_value, out_f32=out.f32, ldo=c,
                     out_i8=out.i8, ldo_i8=out.i8_ld, scale=out.i8_scale or 1.0)

    def _conv_pool(self, pool, conv, pad: int, pad_value: float) -> None:
        """qconv2d -> (pad) -> maxpool2d as one kernel: the conv epilogue runs on the conv outputs,
        the pooled values are written (reference ops.py:630-634, then 469-470 and 293-296)."""
        a = conv.attrs
        stride, padding, dilation, _ = conv_attrs(a)
        x = self.vals[conv.inputs[0]]
        n, c, h, w = x.shape
        q = np.asarray(a["q"])
        o, _, kh, kw = q.shape
        xi8, cp, layout, entries = self._conv_input(conv.inputs[0], _f32(a["x_scale"]))
        wq = self._conv_weight(q, cp, layout)
        out = self._new_out(pool.result, "nhwc")
        probe = DVal(tuple(conv.result.type.shape), "nhwc")
        epi = self._epilogue(conv, probe)
        epi.out_f32, epi.ld_f32 = out.f32, out.cols
        epi.out_i8, epi.ld_i8 = out.i8, out.i8_ld
        epi.out_scale = out.i8_scale if out.i8 is not None else 1.0
        self._launch("qconv2d_pool", n=n, h=h, w=w, cp=cp, x=xi8, layout=layout, row_entries=entries, o=o, kh=kh,
                     kw=kw, wq=self._upload(wq),
                     ldw=wq.shape[1], stride=stride, padding=padding, dilation=dilation,
                     pool_size=pool.attrs["size"], pool_stride=pool.attrs["stride"], pool_pad=pad,
                     pool_pad_value=pad_value, dq=self._scales(a["x_scale"], a["w_scale"]), epi=epi)

    def _op_pad(self, op) -> None:
        p, value = _pad_hw(op)
        x = self.vals[op.inputs[0]]
        n, c, h, w = x.shape
        out = self._new_out(op.result, "nhwc")
        self._launch("maxpool", x_f32=x.f32, n=n, h=h, w=w, c=c, ldc=c, size=1, stride=1, pad=p, pad_value=value,
                     out_f32=out.f32, ldo=c, out_i8=out.i8, ldo_i8=out.i8_ld, scale=out.i8_scale or 1.0)

    def _op_reduce_mean(self, op) -> None:
        x = self.vals[op.inputs[0]]
        n, c, h, w = x.shape
        out = self._new_out(op.result)
        self._launch("mean_hw", x=x.f32, n=n, hw=h * w, c=c, ldc=c, out_f32=out.f32, out_i8=out.i8, ld_i8=out.i8_ld,
                     scale=out.i8_scale or 1.0)

    def _op_reshape(self, op) -> None:
        x = self.vals[op.inputs[0]]
        if x.layout == "nhwc" and x.shape[2] * x.shape[3] > 1:
            n, c, h, w = x.shape
            buf = self._alloc(x.numel * 4)
            self._launch("nhwc_to_nchw", x=x.f32, n=n, h=h, w=w, c=c, ldc=c, y=buf)
        else:
            buf = x.f32
        self._from_reference_order(op.result, buf)


def supported_reason(op) -> Optional[str]:
    """None if the cuda target runs `op`, else why not (reference Target.check, base.py:22-23)."""
    k = op.kind
    if k in QOPS:
        return None
    if op.is_control:
        return "control flow runs on the host"
    rank4 = op.inputs and op.inputs[0].type.rank == 4
    if any(v.type.dtype != "f32" for v in op.inputs) or op.result.type.dtype != "f32":
        return f"{k}: the cuda target computes in f32 (got {op.result.type.dtype})"
    if k == "maxpool2d" and rank4:
        return None
    if k == "pad" and rank4 and _pad_hw(op) is not None:
        return None
    if k == "reduce_mean" and rank4 and sorted(a % 4 for a in op.attrs["axes"]) == [2, 3]:
        return None
    if k == "reshape":
        return None
    if k == "conv2d" and rank4:
        _, _, _, groups = conv_attrs(op.attrs)
        c = op.inputs[0].type.shape[1]
        w = op.inputs[1]
        if groups == c and w.type.shape[0] == c and w.producer is not None and w.producer.is_constant_like:
            return None
        return "conv2d: only depthwise convolutions with constant weights run on cuda in f32"
    return f"{k} has no cuda kernel"


# ============================================================================ target / executable

class CudaExecutable:
    """Runs one compiled segment (reference Executable protocol, base.py:13-16)."""

    def __init__(self, g, device, use_graph: bool = True, fuse_pool: bool = False):
        self.g = g
        self.device = device
        t0 = time.perf_counter()
        self.plan = Plan(g, device, fuse_pool=fuse_pool)
        self.thunks = [device.thunk(l) for l in self.plan.launches]
        self.pin_in = {v: device.pinned(nb) for v, _, nb in self.plan.inputs}
        self.pin_out = {v: device.pinned(nb) for v, _, nb in self.plan.outputs}
        self.use_graph = use_graph and hasattr(device, "graph_begin")
        self._graph = None
        self._runs = 0
        self.compile_seconds = time.perf_counter() - t0
        self.last_seconds = 0.0

    # the pinned staging arrays: feeding these exact arrays skips a host copy
    def input_array(self, v) -> np.ndarray:
        return self.pin_in[v].view(tuple(v.type.shape), np.float32)

    def _launch_all(self) -> None:
        if self.use_graph and self._runs >= 1:
            if self._graph is None:
                self.device.graph_begin()
                try:
                    for t in self.thunks:
                        t()
                finally:
                    self._graph = self.device.graph_end()
            self.device.graph_launch(self._graph)
        else:
            for t in self.thunks:
                t()

    def replay(self) -> None:
        """Launches the plan's kernels once on device-resident inputs (no copies, no sync)."""
        self.device.activate()
        if self._runs == 0:
            raise RuntimeError("run() the executable once before replay()")
        self._launch_all()

    @property
    def launches_per_run(self) -> int:
        return len(self.thunks)

    def run(self, feeds: dict) -> dict:
        t0 = time.perf_counter()
        self.device.activate()
        for v, raw, nbytes in self.plan.inputs:
            view = self.input_array(v)
            arr = feeds[v]
            if not (isinstance(arr, np.ndarray) and arr.ctypes.data == view.ctypes.data):
                np.copyto(view, np.asarray(arr, np.float32).reshape(view.shape))
            self.device.h2d(raw, self.pin_in[v], nbytes)
        self._launch_all()
        for v, buf, nbytes in self.plan.outputs:
            self.device.d2h(self.pin_out[v], buf, nbytes)
        self.device.sync()
        self._runs += 1
        out = {v: self.pin_out[v].view(tuple(v.type.shape), np.float32).copy() for v, _, _ in self.plan.outputs}
        out.update({v: c.copy() for v, c in self.plan.const_outputs.items()})
        self.last_seconds = time.perf_counter() - t0
        return out

    def device_of(self, v) -> Optional[str]:
        return f"cuda:{self.device.index}" if hasattr(self.device, "index") else "cuda"

    def report(self) -> str:
        counts = ", ".join(f"{n}x{k}" for k, n in sorted(self.plan.kernel_counts.items()))
        nq = sum(op.kind in QOPS for op in self.g.ops)
        mode = "CUDA graph" if self.use_graph else "eager launches"
        return (f"cuda:{getattr(self.device, 'index', 0)} (B200, sm_100a): {len(self.g.compute_ops())} ops, "
                f"{nq} in int8 on tcgen05; kernels: {counts}; {mode}")

    def close(self) -> None:
        if self._graph is not None:
            try:
                self.device.graph_destroy(self._graph)
            except Exception:
                pass
            self._graph = None

    def __del__(self):
        self.close()


class CudaTarget:
    """MIRA target plug-in for the B200 (reference Target protocol, base.py:19-26)."""

    name = "cuda"

    def __init__(self, device: Optional[int] = None, graphs: bool = True, executor=None, fuse_pool: bool = False,
                 **_ignored):
        """device: GPU index (default $MIRA_CUDA_DEVICE or 0).  graphs: replay launches from a CUDA
        graph after the first run.  fuse_pool: compute a qconv2d that only feeds a max pool inside
        the pooling kernel.  executor: an object with CudaDevice's interface to run the plan on
        instead (host-side testing of the planner); options of other targets are ignored."""
        if device is None:
            device = int(os.environ.get("MIRA_CUDA_DEVICE", "0"))
        self.device_index = int(device)
        self.graphs = graphs
        self.fuse_pool = fuse_pool
        self._device = executor

    def check(self, op) -> Optional[str]:
        return supported_reason(op)

    def compile(self, g, compile_sub=None) -> CudaExecutable:
        if self._device is None:
            self._device = CudaDevice(self.device_index)
        return CudaExecutable(g, self._device, use_graph=self.graphs, fuse_pool=self.fuse_pool)
