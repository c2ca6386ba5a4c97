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
from .device import DeviceBuffer, DeviceSlice, PinnedBuffer, ptr, set_device

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

    def offset(self, buf, nbytes: int) -> DeviceSlice:
        return DeviceSlice(buf, nbytes)

    def qgemm_workspace(self, m: int, n: int, k: int) -> int:
        return K.qgemm_workspace(m, n, k)

    def attention_workspace(self, b0: int, b1: int, tq: int, tk: int, dh: int) -> int:
        return K.attention_workspace(b0, b1, tq, tk, dh)

    def h2d(self, dst, src: PinnedBuffer, nbytes: int) -> None:
        _lib.call("mira_cuda_h2d", ptr(dst), ptr(src), C.c_size_t(nbytes))

    def d2h(self, dst: PinnedBuffer, src, nbytes: int) -> None:
        _lib.call("mira_cuda_d2h", ptr(dst), ptr(src), C.c_size_t(nbytes))

    def sync(self) -> None:
        _lib.call("mira_cuda_sync")

    def zero(self, buf, nbytes: int) -> None:
        _lib.call("mira_cuda_memset", ptr(buf), 0, C.c_size_t(nbytes))

    # ---- the copy stream and events (run_many's overlap of input copies with kernels)
    def event(self):
        ev = C.c_void_p()
        _lib.call("mira_cuda_event_create", C.byref(ev))
        return ev

    def event_destroy(self, ev) -> None:
        _lib.call("mira_cuda_event_destroy", ev)

    def event_record(self, ev) -> None:
        _lib.call("mira_cuda_event_record", ev)

    def event_sync(self, ev) -> None:
        _lib.call("mira_cuda_event_sync", ev)

    def wait(self, ev) -> None:
        _lib.call("mira_cuda_stream_wait", ev)

    def copy_record(self, ev) -> None:
        _lib.call("mira_cuda_copy_stream_record", ev)

    def copy_wait(self, ev) -> None:
        _lib.call("mira_cuda_copy_stream_wait", ev)

    def h2d_copy(self, dst, src: PinnedBuffer, nbytes: int) -> None:
        _lib.call("mira_cuda_h2d_copy_stream", ptr(dst), ptr(src), C.c_size_t(nbytes))

    def d2d(self, dst, src, nbytes: int) -> None:
        _lib.call("mira_cuda_d2d", ptr(dst), ptr(src), C.c_size_t(nbytes))

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
                    a["row_entries"], a["pad"], a["stride"])
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
            if k == "qgemm" and a.get("ws") is not None:
                fn = L.mira_cuda_qgemm_splitk
                args = (a["M"], a["N"], a["K"], ptr(a["A"]), a["lda"], ptr(a["B"]), a["ldb"], C.byref(dq), C.byref(e),
                        ptr(a["ws"]), a["ws_bytes"])
            elif k == "qgemm":
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
            fn = L.mira_cuda_maxpool2d_nhwc_ex
            args = (ptr(a.get("x_f32")), ptr(a.get("x_i8")), a["n"], a["h"], a["w"], a["c"], a["ldc"], a["size"],
                    a["stride"], a["pad"], float(np.float32(a["pad_value"])), ptr(a.get("out_f32")), a.get("ldo", 0),
                    ptr(a.get("out_i8")), a.get("ldo_i8", 0), float(np.float32(a.get("scale", 1.0))),
                    int(a.get("i8_layout", 0)))
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
        elif k == "qdwconv":
            e = a["epi"].struct()
            dq = K.dequant_channel(*a["dq"])
            keep += [e, dq]
            fn = L.mira_cuda_qdwconv2d_nhwc
            (sh, sw), (ph, pw), (dh, dw) = a["stride"], a["padding"], a["dilation"]
            args = (ptr(a["x"]), a["n"], a["h"], a["w"], a["c"], a["ldx"], ptr(a["wq"]), a["kh"], a["kw"], sh, sw,
                    ph, pw, dh, dw, C.byref(dq), C.byref(e))
        elif k == "copy":
            fn = L.mira_cuda_d2d
            args = (ptr(a["dst"]), ptr(a["src"]), C.c_size_t(a["nbytes"]))
        elif k == "bmm":
            av, bv, e = a["a"].struct(), a["b"].struct(), a["epi"].struct()
            keep += [av, bv, e]
            if a.get("b_scale") is not None:
                fn = L.mira_cuda_bmm_f32_w8
                args = (a["batch0"], a["batch1"], a["m"], a["n"], a["k"], C.byref(av), C.byref(bv),
                        ptr(a["b_scale"]), C.byref(e))
            else:
                fn = L.mira_cuda_bmm_f32
                args = (a["batch0"], a["batch1"], a["m"], a["n"], a["k"], C.byref(av), C.byref(bv), C.byref(e))
        elif k == "elementwise":
            av, ov = a["a"].struct(), a["out"].struct()
            bv = a["b"].struct() if a.get("b") is not None else None
            n4 = tuple(int(d) for d in a["shape"])
            keep += [av, ov, bv]
            fn = L.mira_cuda_elementwise_f32
            args = (a["code"], *n4, C.byref(av), C.byref(bv) if bv is not None else None, _f32(a.get("scalar", 0.0)),
                    int(bool(a.get("swapped"))), C.byref(ov))
        elif k == "im2col":
            fn = L.mira_cuda_im2col_f32
            (sh, sw), (ph, pw), (dh, dw) = a["stride"], a["padding"], a["dilation"]
            args = (ptr(a["x"]), a["n"], a["h"], a["w"], a["c"], a["ldc"], a["kh"], a["kw"], sh, sw, ph, pw, dh, dw,
                    ptr(a["out"]), a["ld_out"])
        elif k == "dyn_slice":
            xv, ov, xd, sz = a["x"].struct(), a["out"].struct(), K.dims4(a["x_shape"]), K.dims4(a["size"])
            keep += [xv, ov, xd, sz]
            fn = L.mira_cuda_dynamic_slice
            args = (C.byref(xv), xd, ptr(a["start"]), a["rank"], sz, C.byref(ov))
        elif k == "dyn_update":
            xv, uv, xd, ud = a["x"].struct(), a["upd"].struct(), K.dims4(a["x_shape"]), K.dims4(a["upd_shape"])
            keep += [xv, uv, xd, ud]
            fn = L.mira_cuda_dynamic_update_slice
            args = (C.byref(xv), xd, C.byref(uv), ud, ptr(a["start"]), a["rank"])
        elif k == "layernorm":
            fn = L.mira_cuda_layernorm_rows
            args = (ptr(a["x"]), a["rows"], a["d"], a["ld_x"], ptr(a["gamma"]), ptr(a["beta"]), _f32(a["eps"]),
                    ptr(a.get("out_f32")), a.get("ld_f32", 0), ptr(a.get("out_i8")), a.get("ld_i8", 0),
                    _f32(a.get("scale", 1.0)))
        elif k == "softmax":
            fn = L.mira_cuda_softmax_rows
            args = (ptr(a["x"]), a["rows"], a["n"], a["ld_x"], ptr(a["out"]), a["ld_out"])
        elif k == "embed":
            fn = L.mira_cuda_embed_rows
            args = (ptr(a["table"]), a["vocab"], a["d"], ptr(a["idx"]), a["rows"], ptr(a.get("addend")),
                    a.get("addend_rows", 0), ptr(a["out"]), a["ld_out"])
        elif k == "attention":
            st = a["desc"].struct()
            keep.append(st)
            fn = L.mira_cuda_attention_f32
            args = (C.byref(st),)
        elif k == "absmax":
            xv = a["x"].struct()
            keep.append(xv)
            fn = L.mira_cuda_absmax_f32
            args = tuple(int(x) for x in a["shape"]) + (C.byref(xv), ptr(a["out"]))
        elif k == "copy_view":
            sv, dv = a["src"].struct(), a["dst"].struct()
            keep += [sv, dv]
            fn = L.mira_cuda_copy_view_f32
            args = tuple(int(x) for x in a["shape"]) + (C.byref(sv), C.byref(dv))
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
    i8_layout: str = "nhwc"      # or "row4" (MIRA_LAYOUT_ROW4, graph inputs of at most 4 channels), or "cp"
                                 # (MIRA_LAYOUT_CP, read by 3x3 stride-1 convolutions)
    row_entries: int = 0
    i32: object = None           # int32 graph inputs (token ids)
    strides: Optional[tuple] = None   # "rows" layout: element strides of the f32 view (None: row-major)
    offset: int = 0                   # "rows" layout: element offset of the f32 view
    contig: object = None             # row-major copy of a strided view, made on first need

    @property
    def f32_strides(self) -> tuple:
        return self.strides if self.strides is not None else contiguous_strides(self.shape)

    @property
    def is_contiguous(self) -> bool:
        if self.offset != 0:
            return False
        if self.strides is None:
            return True
        return all(d == 1 or s == c for d, s, c in zip(self.shape, self.strides, contiguous_strides(self.shape)))

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


def contiguous_strides(shape) -> tuple:
    st, acc = [], 1
    for d in reversed(tuple(shape)):
        st.append(acc)
        acc *= int(d)
    return tuple(reversed(st))


def view_strides(old_shape, old_strides, new_shape) -> Optional[tuple]:
    """Strides that present the elements of a strided view in `new_shape` (row-major element order
    kept), or None when the reshape needs a copy.  Dimensions are matched chunk by chunk: each run
    of old dimensions that are contiguous with one another must be covered exactly by a run of new
    dimensions."""
    old_shape, old_strides, new_shape = tuple(old_shape), tuple(old_strides), tuple(new_shape)
    if int(np.prod(new_shape, dtype=np.int64)) == 0 or not old_shape:
        return contiguous_strides(new_shape)
    new = [0] * len(new_shape)
    view_d = len(new_shape) - 1
    base = old_strides[-1]
    tensor_numel = view_numel = 1
    for d in range(len(old_shape) - 1, -1, -1):
        tensor_numel *= old_shape[d]
        if d == 0 or (old_shape[d - 1] != 1 and old_strides[d - 1] != tensor_numel * base):
            while view_d >= 0 and (view_numel < tensor_numel or new_shape[view_d] == 1):
                new[view_d] = view_numel * base
                view_numel *= new_shape[view_d]
                view_d -= 1
            if view_numel != tensor_numel:
                return None
            if d > 0:
                base = old_strides[d - 1]
                tensor_numel = view_numel = 1
    if view_d != -1:
        return None
    return tuple(new)


IMAGE_OPS = ("qconv2d", "conv2d", "maxpool2d", "pad", "reduce_mean")


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
        self._kmax = None            # device scalar max|k| shared by the attention launches
        self._attn_ws, self._attn_ws_bytes = None, 0   # tensor-core attention scratch
        self.w8_cache: dict = {}     # weight-only int8 matmul weights: value -> (int8 DVal, scales)
        self.aliases: dict = {}      # dynamic_update_slice result -> the graph input it updated in place
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
            if (pad_ok and conv is not None and conv.kind == "qconv2d" and len(users.get(src, [])) == 1
                    and src not in g.outputs and self._conv_pool_fusable(conv)
                    and (self.fuse_pool or self._stem_pool(conv, op))):
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
        self.need_f32 = {v for v in need_f32 if self._const(v) is None and v.type.dtype == "f32"}
        self.i8_req = i8_req
        self.image_values = set()
        for op in g.ops:
            if op.kind in IMAGE_OPS:
                for v in list(op.inputs) + list(op.results):
                    if v.type.rank == 4 and self._const(v) is None:
                        self.image_values.add(v)
        self._group_qmatmuls()
        self._find_attention()
        self.cp_values = {v for v in i8_req if self._cp_layout_ok(v)}

    def _cp_layout_ok(self, v) -> bool:
        """Whether the int8 form of `v` is kept in the chunk-planar layout (MIRA_LAYOUT_CP): every
        quantized op reading it is a 3x3, stride-1, pad-1 convolution of 64k channels whose halo
        fits the kernel's buffers, all at one scale, and `v` comes from a convolution epilogue or
        the f32 max pool (the producers that write the layout)."""
        if v.type.rank != 4 or v not in self.image_values:
            return False
        p = v.producer
        if p is None or p.kind not in ("qconv2d", "maxpool2d") or p in self.skipped:
            return False
        if p in self.conv_into_pool and not self._stem_pool(self.conv_into_pool[p], p):
            return False
        n, c, h, w = v.type.shape
        if c % 64 or not K.patch_preferred(c, w):
            return False
        readers = 0
        for op in self.users.get(v, []):
            if op.kind not in QOPS or op.inputs[0] is not v:
                continue
            stride, padding, dilation, groups = conv_attrs(op.attrs)
            kh, kw = np.asarray(op.attrs["q"]).shape[2:]
            if (op.kind != "qconv2d" or op in self.skipped or _f32(op.attrs["x_scale"]) != self.i8_req[v] or groups != 1
                    or (kh, kw) != (3, 3) or tuple(stride) != (1, 1) or tuple(padding) != (1, 1)
                    or tuple(dilation) != (1, 1)):
                return False
            readers += 1
        return readers > 0

    def _find_attention(self):
        """matmul(q, k^T) {scale, mask} -> softmax(axis=-1) -> matmul(., v) chains run as one fused
        attention launch (the scores are never stored).  When the output only reaches quantized
        matmuls through transpose(0, 2, 1, 3) + reshape (the heads merged back), the launch also
        writes their int8 input rows directly."""
        g, users = self.g, self.users
        self.attention: dict = {}
        for op in g.ops:
            if op.kind != "matmul" or op in self.skipped or op.result in g.outputs:
                continue
            uses = users.get(op.result, [])
            if len(uses) != 1 or uses[0].kind != "softmax" or uses[0].result in g.outputs:
                continue
            sm = uses[0]
            rank = sm.result.type.rank
            if rank < 2 or rank > 4 or sm.attrs.get("axis", -1) % rank != rank - 1:
                continue
            su = users.get(sm.result, [])
            if len(su) != 1 or su[0].kind != "matmul" or su[0].inputs[0] is not sm.result or su[0].attrs.get("epilogue"):
                continue
            mm2 = su[0]
            steps = list(op.attrs.get("epilogue", ()))
            scale_op, scale, mask = None, 1.0, None
            if steps and steps[0][0] in ("mul", "div") and steps[0][1] is not None:
                fn, idx, swapped = steps[0]
                val = self._const(op.inputs[idx])
                if val is not None and val.size == 1 and not (fn == "div" and swapped):
                    scale_op, scale = fn, float(np.float32(val.ravel()[0]))
                    steps.pop(0)
            if steps and steps[0][0] == "add" and steps[0][1] is not None:
                mask = op.inputs[steps[0][1]]
                steps.pop(0)
            if steps:
                continue
            q, kt, v = op.inputs[0], op.inputs[1], mm2.inputs[1]
            bshape = tuple(op.result.type.shape[:-2])
            if any(tuple(x.type.shape[:-2]) != bshape for x in (q, kt, v)) or self._const(q) is not None:
                continue
            dh, dv = q.type.shape[-1], v.type.shape[-1]
            if dh != dv or dh > 128 or kt.type.shape[-2] != dh:
                continue
            self.attention[op] = dict(softmax=sm, pv=mm2, scale_op=scale_op, scale=scale, mask=mask,
                                      i8_chain=self._attention_i8_chain(mm2))
            self.skipped.update((sm, mm2))
            chain = self.attention[op]["i8_chain"]
            if chain is not None:
                self.skipped.update(chain[:2])

    def _attention_i8_chain(self, mm2):
        """(transpose op, reshape op) when the attention output [B, H, T, dv] only reaches
        quantized matmuls as reshape(transpose(o, (0, 2, 1, 3)), [..., H * dv])."""
        g, users = self.g, self.users
        shape = tuple(mm2.result.type.shape)
        if len(shape) != 4 or mm2.result in g.outputs:
            return None
        u = users.get(mm2.result, [])
        if len(u) != 1 or u[0].kind != "transpose" or tuple(int(p) % 4 for p in u[0].attrs["perm"]) != (0, 2, 1, 3):
            return None
        tr = u[0]
        u2 = users.get(tr.result, [])
        if len(u2) != 1 or u2[0].kind != "reshape" or tr.result in g.outputs:
            return None
        rs = u2[0]
        b, h, t, dv = shape
        rshape = tuple(rs.result.type.shape)
        if not rshape or rshape[-1] != h * dv or int(np.prod(rshape[:-1], dtype=np.int64)) != b * t:
            return None
        if rs.result in g.outputs or rs.result in self.need_f32 or rs.result not in self.i8_req:
            return None
        if any(c.kind != "qmatmul" or c.inputs[0] is not rs.result for c in users.get(rs.result, [])):
            return None
        return tr, rs

    def _group_qmatmuls(self):
        """Quantized matmuls that read the same int8 activation (same value, same x_scale) and
        whose epilogues differ only in per-channel constants run as one GEMM over the concatenated
        weights (the q/k/v projections of attention); their results are column slices of one
        [M, sum(N)] buffer."""
        self.qgroup: dict = {}       # first op of a group -> all ops of the group
        self.qgrouped: set = set()   # later ops of a group (produced by the first)
        by_key: dict = {}
        for op in self.g.ops:
            if op.kind != "qmatmul" or op in self.skipped or op.result in self.g.outputs:
                continue
            if op.result in self.i8_req or op.result not in self.need_f32:
                continue
            sig = self._epilogue_signature(op)
            if sig is None:
                continue
            key = (op.inputs[0], _f32(op.attrs["x_scale"]), sig)
            by_key.setdefault(key, []).append(op)
        for ops in by_key.values():
            if len(ops) > 1:
                self.qgroup[ops[0]] = ops
                self.qgrouped.update(ops[1:])

    def _epilogue_signature(self, op):
        """Hashable form of an epilogue whose operands are constant scalars or per-column
        vectors (None for other epilogues)."""
        n = np.asarray(op.attrs["q"]).shape[1]
        sig = []
        for fn, idx, swapped in op.attrs.get("epilogue", ()):
            if idx is None:
                sig.append((fn, None, False))
                continue
            val = self._const(op.inputs[idx])
            if val is None:
                return None
            if val.size == 1:
                sig.append((fn, ("scalar", float(np.float32(val.ravel()[0]))), bool(swapped)))
            elif val.shape[-1] == n and val.size == n:
                sig.append((fn, "channel", bool(swapped)))
            else:
                return None
        return tuple(sig)

    def _stem_pool(self, conv, pool) -> bool:
        """The conv + pool pair has the form of the stem kernel (libmira_cuda stem_pool_kernel, always
        fused): a stride-2 conv reading the row-expanded layout of a graph input of at most 4
        channels, at most 8 x 8 taps, 64 or fewer output channels (a multiple of 4), an output row of
        at most 128 pixels, then a 3x3/2 max pool over one pixel of -inf padding."""
        stride, padding, dilation, groups = conv_attrs(conv.attrs)
        o, _, kh, kw = np.asarray(conv.attrs["q"]).shape
        x = conv.inputs[0]
        if (groups != 1 or tuple(stride) != (2, 2) or tuple(dilation) != (1, 1) or kh > 8 or kw > 8 or o > 64 or o % 4
                or conv.result.type.shape[3] > 128 or x.type.rank != 4 or x.type.shape[1] > 4
                or x.producer is not None or self._row4_geometry(x) is None):
            return False
        if pool.attrs["size"] != 3 or pool.attrs["stride"] != 2:
            return False
        return pool in self.pad_into_pool and self.pad_into_pool[pool][1] == 1

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

    def _layout_of(self, v) -> str:
        return "nhwc" if v.type.rank == 4 and v in self.image_values else "rows"

    def _new_out(self, v, layout: Optional[str] = None, strides: Optional[tuple] = None) -> DVal:
        shape = tuple(v.type.shape)
        dv = DVal(shape, layout or self._layout_of(v))
        if v in self.need_f32:
            dv.f32 = self._alloc(dv.numel * 4)
            dv.strides = strides
        if v in self.i8_req:
            dv.i8_scale = self.i8_req[v]
            dv.i8_ld = K.round_up(dv.cols, 16)
            if v in self.cp_values:
                n, c, h, w = shape
                dv.i8_layout = "cp"
                dv.i8 = self._alloc(K.cp_bytes(n, h, w, dv.i8_ld), zero=True)
            else:
                dv.i8 = self._alloc(dv.rows * dv.i8_ld, zero=True)
        self.vals[v] = dv
        return dv

    # ------------------------------------------------------------------ views

    def _at(self, buf, elem_offset: int, itemsize: int = 4):
        return buf if not elem_offset else self.dev.offset(buf, int(elem_offset) * itemsize)

    def _contiguous(self, dv: DVal):
        """A row-major f32 buffer holding the elements of `dv` (a copy for strided views)."""
        if dv.is_contiguous:
            return dv.f32
        if dv.contig is None:
            shape4, view = self._view4(dv)
            dv.contig = self._alloc(dv.numel * 4)
            self._launch("copy_view", shape=shape4, src=view,
                         dst=K.View(dv.contig, (0,) * (4 - len(dv.shape)) + contiguous_strides(dv.shape)))
        return dv.contig

    def _view4(self, dv: DVal):
        shape, st = tuple(dv.shape), dv.f32_strides
        if len(shape) > 4:
            raise UnsupportedOnCuda("views of more than 4 dimensions")
        pad = 4 - len(shape)
        return (1,) * pad + shape, K.View(dv.f32, (0,) * pad + tuple(st), dv.offset)

    def _rows_of(self, v):
        """(f32 buffer, row stride) of `v` read as rows [prod(shape[:-1]), shape[-1]]; strided views
        whose rows are not evenly spaced are copied first."""
        dv = self.vals[v]
        if dv.f32 is None:
            raise UnsupportedOnCuda("value has no f32 representation")
        if dv.layout != "rows":
            return dv.f32, dv.cols
        shape, st = tuple(dv.shape), dv.f32_strides
        cols = shape[-1] if shape else 1
        lead = [(d, x) for d, x in zip(shape[:-1], st[:-1]) if d != 1]
        ok = not shape or cols == 1 or st[-1] == 1
        ld = lead[-1][1] if lead else cols
        expect = ld
        for d, x in reversed(lead):
            ok = ok and x == expect
            expect = x * d
        if ok and ld >= cols:
            return self._at(dv.f32, dv.offset), ld
        return self._contiguous(dv), cols

    def _from_reference_order(self, v, buf) -> DVal:
        """A DVal for `v` from an f32 buffer in the reference's element order (NCHW / row-major)."""
        shape = tuple(v.type.shape)
        dv = DVal(shape, self._layout_of(v))
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
                    entries, pad, stride = row4
                    dv.i8, dv.i8_layout, dv.row_entries, dv.i8_ld = self._alloc(n * h * entries * 16), "row4", entries, 4
                    self._launch("quantize_row4", x=buf, n=n, c=c, h=h, w=w, scale=dv.i8_scale, xq=dv.i8,
                                 row_entries=entries, pad=pad, stride=stride)
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
        """(entries, pad, stride) when every consumer of the int8 value of `v` is a convolution that can
        read the row-expanded layout (at most 4 channels, kernel width <= 8, no dilation, horizontal
        stride 1, 2 or 4) with one common horizontal geometry; None otherwise."""
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
            if groups != 1 or kw > 8 or tuple(dilation) != (1, 1) or op.inputs[0] is not v or stride[1] not in (1, 2, 4):
                return None
            ow = op.result.type.shape[3]
            g = (K.row4_entries(ow, stride[1]), padding[1], stride[1])
            if geo is not None and g != geo:
                return None
            geo = g
        return geo

    def _conv_input(self, v, scale: float):
        """(int8 buffer, channels per pixel, layout code, entries per row) of a conv input."""
        dv = self.vals[v]
        if dv.i8 is not None and dv.i8_scale == scale and dv.i8_layout == "row4":
            return dv.i8, 4, _lib.LAYOUT_ROW4, dv.row_entries
        if dv.i8 is not None and dv.i8_scale == scale and dv.i8_layout == "cp":
            return dv.i8, dv.i8_ld, _lib.LAYOUT_CP, 0
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
        src, ld_x = self._rows_of(v)
        self._launch("quantize_rows", x=src, rows=dv.rows, cols=dv.cols, ld_x=ld_x, scale=scale, xq=buf, ld_q=ld)
        if dv.i8 is None:
            dv.i8, dv.i8_scale, dv.i8_ld = buf, scale, ld
        return buf, ld

    def _input(self, v) -> None:
        if v.type.dtype not in ("f32", "i32"):
            raise UnsupportedOnCuda(f"input {v!r} is {v.type.dtype}; the cuda target takes f32 and i32 inputs")
        nbytes = v.type.numel * 4
        raw = self._alloc(nbytes)
        self.inputs.append((v, raw, nbytes))
        if v.type.dtype == "i32":
            self.vals[v] = DVal(tuple(v.type.shape), "rows", i32=raw)
            return
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
        elif dv.layout == "rows":
            buf = self._contiguous(dv)
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
                     out_scale=out.i8_scale if out.i8 is not None else 1.0,
                     i8_layout=_lib.LAYOUT_CP if out.i8_layout == "cp" else _lib.LAYOUT_NHWC)

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
            src, ld = self._rows_of(v)
            return K.Step(fn, "full", swapped, ptr=src, ld=ld)
        if self._is_channel(dv.shape, out):
            padded = self._alloc(K.round_up(max(out.cols, 1), K.CHANNEL_PAD) * 4, zero=True)
            self._launch("copy", dst=padded, src=self._contiguous(dv), nbytes=out.cols * 4)
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
        if op in self.qgrouped:
            return
        a = op.attrs
        x = self.vals[op.inputs[0]]
        if x.layout != "rows":
            raise UnsupportedOnCuda("qmatmul on a 4-D input")
        if op in self.qgroup:
            self._qmatmul_group(self.qgroup[op])
            return
        q = np.asarray(a["q"])
        kdim, n = q.shape
        A, lda = self._i8_of(op.inputs[0], _f32(a["x_scale"]))
        wq = self._upload(K.matmul_weight(q))
        out = self._new_out(op.result)
        self._launch("qgemm", M=x.rows, N=n, K=kdim, A=A, lda=lda, B=wq, ldb=K.round_up(kdim, 16),
                     dq=self._scales(a["x_scale"], a["w_scale"]), epi=self._epilogue(op, out),
                     **self._splitk_workspace(x.rows, n, kdim))

    def _splitk_workspace(self, m: int, n: int, k: int) -> dict:
        """Workspace arguments for a GEMM with too few output tiles to fill the GPU (split-K)."""
        fn = getattr(self.dev, "qgemm_workspace", None)
        nbytes = int(fn(m, n, k)) if fn is not None else 0
        if nbytes <= 0:
            return {}
        return {"ws": self._alloc(nbytes), "ws_bytes": nbytes}

    def _qmatmul_group(self, ops) -> None:
        """One GEMM for quantized matmuls sharing their int8 input: weights, scales and per-column
        epilogue constants concatenated along N; every result is a column slice of the output."""
        first = ops[0]
        x = self.vals[first.inputs[0]]
        qs = [np.asarray(op.attrs["q"]) for op in ops]
        kdim = qs[0].shape[0]
        widths = [q.shape[1] for q in qs]
        total = int(sum(widths))
        A, lda = self._i8_of(first.inputs[0], _f32(first.attrs["x_scale"]))
        wq = self._upload(K.matmul_weight(np.concatenate(qs, axis=1)))
        w_scale = np.concatenate([np.asarray(op.attrs["w_scale"], np.float32) for op in ops])
        buf = self._alloc(x.rows * total * 4)
        steps = []
        for i, (fn, idx, swapped) in enumerate(first.attrs.get("epilogue", ())):
            if idx is None:
                steps.append(K.Step(fn))
                continue
            val = self._const(first.inputs[idx]).astype(np.float32)
            if val.size == 1:
                steps.append(K.Step(fn, "scalar", bool(swapped), scalar=float(val.ravel()[0])))
                continue
            cols = [self._const(op.inputs[op.attrs["epilogue"][i][1]]).astype(np.float32).ravel() for op in ops]
            steps.append(K.Step(fn, "channel", bool(swapped), ptr=self._upload(K.pad_channels(np.concatenate(cols)))))
        epi = K.Epi(steps, out_f32=buf, ld_f32=total)
        self._launch("qgemm", M=x.rows, N=total, K=kdim, A=A, lda=lda, B=wq, ldb=K.round_up(kdim, 16),
                     dq=self._scales(first.attrs["x_scale"], w_scale), epi=epi,
                     **self._splitk_workspace(x.rows, total, kdim))
        col = 0
        for op, w in zip(ops, widths):
            shape = tuple(op.result.type.shape)
            st = tuple(c * total for c in contiguous_strides(shape[:-1])) + (1,)
            self.vals[op.result] = DVal(shape, "rows", f32=buf, strides=st, offset=col)
            col += w

    def _op_qconv2d(self, op) -> None:
        a = op.attrs
        stride, padding, dilation, groups = conv_attrs(a)
        x = self.vals[op.inputs[0]]
        n, c, h, w = x.shape
        q = np.asarray(a["q"])
        o, _, kh, kw = q.shape
        if groups != 1:
            if not (groups == c == o and q.shape[1] == 1 and c % 4 == 0):
                raise UnsupportedOnCuda("grouped qconv2d other than depthwise")
            # opt-in int8 depthwise: int8 NHWC input, tap-major int8 weights, exact integer sums
            xi8, ldx = self._i8_of(op.inputs[0], _f32(a["x_scale"]))
            wtap = np.ascontiguousarray(q[:, 0].reshape(c, kh * kw).T.astype(np.int8))
            out = self._new_out(op.result, "nhwc")
            self._launch("qdwconv", x=xi8, ldx=ldx, n=n, h=h, w=w, c=c, wq=self._upload(wtap), kh=kh, kw=kw,
                         stride=stride, padding=padding, dilation=dilation,
                         dq=self._scales(a["x_scale"], a["w_scale"]), epi=self._epilogue(op, out))
            return
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
        if groups == 1:
            self._conv2d_general(op, x, stride, padding, dilation)
            return
        wt = self._const(op.inputs[1])
        if wt is None or groups != c or wt.shape[0] != c or wt.shape[1] != 1:
            raise UnsupportedOnCuda("only depthwise or ungrouped f32 conv2d with constant weights runs on cuda")
        kh, kw = wt.shape[2:]
        wtap = np.ascontiguousarray(wt[:, 0].reshape(c, kh * kw).T.astype(np.float32))
        out = self._new_out(op.result, "nhwc")
        self._launch("dwconv", x=x.f32, n=n, h=h, w=w, c=c, wt=self._upload(wtap), kh=kh, kw=kw, stride=stride,
                     padding=padding, dilation=dilation, epi=self._epilogue(op, out))

    def _conv2d_general(self, op, x: DVal, stride, padding, dilation) -> None:
        """An ungrouped f32 convolution (reference _conv2d_ref, ops.py:265-276) as the f32 matmul of its
        patch matrix (im2col over the NHWC input) with the weights reshaped to [kh * kw * c, o], the
        epilogue fused into the matmul.  A weight-only int8 weight (a `dequantize` constant with one
        scale per output channel, quantize.py:38-41) stays int8 and is rebuilt as RN(f32(q) * scale)
        while the matmul stages it.  Like the reference's per-tap f32 sums, the result is exact to
        f32 rounding, not bit for bit."""
        n, c, h, w = x.shape
        wv = op.inputs[1]
        p = wv.producer
        o, cin, kh, kw = wv.type.shape
        oh, ow = op.result.type.shape[2:]
        rows, kdim = n * oh * ow, kh * kw * cin
        if x.f32 is None or x.layout != "nhwc":
            raise UnsupportedOnCuda("conv2d input without an NHWC f32 form")
        patches = self._alloc(max(rows * kdim, 1) * 4)
        self._launch("im2col", x=x.f32, n=n, h=h, w=w, c=c, ldc=x.cols, kh=kh, kw=kw, stride=stride,
                     padding=padding, dilation=dilation, out=patches, ld_out=kdim)
        b_scale = None
        if p is not None and p.kind == "dequantize" and p.attrs["axis"] % 4 == 0 and wv.type.dtype == "f32":
            q = np.asarray(p.attrs["q"])
            bmat = self._upload(np.ascontiguousarray(q.transpose(2, 3, 1, 0).reshape(kdim, o)))
            b_scale = self._upload(np.ascontiguousarray(np.asarray(p.attrs["scale"], np.float32).reshape(-1)))
        else:
            wt = self._const(wv)
            if wt is None:
                raise UnsupportedOnCuda("conv2d with runtime weights")
            bmat = self._upload(np.ascontiguousarray(wt.astype(np.float32).transpose(2, 3, 1, 0).reshape(kdim, o)))
        out = self._new_out(op.result, "nhwc")
        if out.f32 is None and out.i8 is None:
            out.f32 = self._alloc(out.numel * 4)
        bview = K.View(bmat, (0, 0, o, 1), itemsize=1 if b_scale is not None else 4)
        self._launch("bmm", batch0=1, batch1=1, m=rows, n=o, k=kdim, a=K.View(patches, (0, 0, kdim, 1)), b=bview,
                     b_scale=b_scale, epi=self._as_bmm_epi(self._epilogue(op, out)))

    @staticmethod
    def _as_bmm_epi(epi: K.Epi) -> K.BmmEpi:
        """A conv-style epilogue over [rows, cols] outputs as the f32 matmul's view-based one: per-channel
        operands are rows of stride 0, full operands rows of stride ld, per-row operands columns of
        stride 0."""
        steps = []
        for st in epi.steps:
            if st.operand == "none":
                steps.append(K.BmmStep(st.op, swapped=st.swapped))
            elif st.operand == "scalar":
                steps.append(K.BmmStep(st.op, "scalar", st.swapped, scalar=st.scalar))
            else:
                strides = {"channel": (0, 0, 0, 1), "full": (0, 0, st.ld, 1), "row": (0, 0, 1, 0)}[st.operand]
                steps.append(K.BmmStep(st.op, "view", st.swapped, view=K.View(st.ptr, strides)))
        out = K.View(epi.out_f32, (0, 0, epi.ld_f32, 1)) if epi.out_f32 is not None else None
        out_i8 = K.View(epi.out_i8, (0, 0, epi.ld_i8, 1), itemsize=1) if epi.out_i8 is not None else None
        return K.BmmEpi(steps, out=out, out_i8=out_i8, out_scale=epi.out_scale)

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
                     out_i8=out.i8, ldo_i8=out.i8_ld, scale=out.i8_scale or 1.0,
                     i8_layout=_lib.LAYOUT_CP if out.i8_layout == "cp" else _lib.LAYOUT_NHWC)

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
        epi.i8_layout = _lib.LAYOUT_CP if out.i8_layout == "cp" else _lib.LAYOUT_NHWC
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

    def _reference_order(self, dv: DVal):
        """An f32 buffer with the elements of `dv` in the reference's row-major order."""
        if dv.layout == "nhwc" and dv.shape[2] * dv.shape[3] > 1:
            n, c, h, w = dv.shape
            buf = self._alloc(dv.numel * 4)
            self._launch("nhwc_to_nchw", x=dv.f32, n=n, h=h, w=w, c=c, ldc=c, y=buf)
            return buf
        if dv.layout == "nhwc":
            return dv.f32
        return self._contiguous(dv)

    def _op_reshape(self, op) -> None:
        x = self.vals[op.inputs[0]]
        shape = tuple(op.result.type.shape)
        if x.layout == "rows" and self._layout_of(op.result) == "rows" and x.f32 is not None:
            st = view_strides(x.shape, x.f32_strides, shape)
            if st is not None:
                dv = DVal(shape, "rows", f32=x.f32, strides=st, offset=x.offset)
                self.vals[op.result] = dv
                if op.result in self.i8_req:
                    self._i8_of(op.result, self.i8_req[op.result])
                return
        self._from_reference_order(op.result, self._reference_order(x))

    def _op_transpose(self, op) -> None:
        """A strided view: the reference's np.transpose (ops.py:375) moves no data here; a consumer
        that needs row-major data copies it (copy_view)."""
        x = self.vals[op.inputs[0]]
        perm = tuple(int(p) % max(len(x.shape), 1) for p in op.attrs["perm"])
        if x.layout != "rows":
            base = DVal(tuple(x.shape), "rows", f32=self._reference_order(x))
        else:
            base = x
        st = base.f32_strides
        dv = DVal(tuple(base.shape[p] for p in perm), "rows", f32=base.f32, strides=tuple(st[p] for p in perm),
                  offset=base.offset)
        self.vals[op.result] = dv
        if op.result in self.i8_req:
            self._i8_of(op.result, self.i8_req[op.result])

    # ------------------------------------------------------------------ sequence (transformer) ops

    def _f32_dval(self, v) -> DVal:
        c = self._const(v)
        if c is not None:
            c = np.ascontiguousarray(c.astype(np.float32))
            return DVal(tuple(c.shape), "rows", f32=self._upload(c))
        return self.vals[v]

    @staticmethod
    def _broadcast_view(dv: DVal, out_shape) -> K.View:
        """`dv` broadcast against `out_shape` (rank <= 4) as a 4-D view; size-1 dims get stride 0."""
        r = len(out_shape)
        shape = (1,) * (r - len(dv.shape)) + tuple(dv.shape)
        st = (0,) * (r - len(dv.shape)) + tuple(dv.f32_strides)
        st = tuple(0 if d == 1 else x for d, x in zip(shape, st))
        return K.View(dv.f32, (0,) * (4 - r) + st, dv.offset)

    def _attention(self, op, info) -> None:
        """One fused attention launch for matmul -> softmax -> matmul (see _find_attention)."""
        mm2 = info["pv"]
        qd, ktd, vd = (self._f32_dval(v) for v in (op.inputs[0], op.inputs[1], mm2.inputs[1]))
        sshape = tuple(op.result.type.shape)
        oshape = tuple(mm2.result.type.shape)
        tq, tk, dh = sshape[-2], sshape[-1], qd.shape[-1]
        batch = (1,) * (4 - len(oshape)) + oshape[:-2]
        qv = self._broadcast_view(qd, oshape[:-2] + (tq, dh))
        ktv = self._broadcast_view(ktd, oshape[:-2] + (dh, tk))
        kv = K.View(ktv.buf, ktv.strides[:2] + (ktv.strides[3], ktv.strides[2]), ktv.offset)
        vv = self._broadcast_view(vd, oshape[:-2] + (tk, dh))
        mask_view, tile_max, kmax, tile_zero = None, None, None, None
        if info["mask"] is not None:
            mask_view = self._broadcast_view(self._f32_dval(info["mask"]), sshape)
            mval = self._const(info["mask"])
            if mval is not None:
                m2 = np.broadcast_to(np.asarray(mval, np.float32), sshape)
                m2 = m2.reshape(-1, tq, tk)
                if all(np.array_equal(m2[0], m2[i]) for i in range(1, m2.shape[0])):
                    tile_max = self._upload(K.mask_tile_max(m2[0], tq, tk))
                    tile_zero = self._upload(K.mask_tile_zero(m2[0], tq, tk))
        if tile_max is not None:
            if self._kmax is None:
                self._kmax = self._alloc(16, zero=True)
            kmax = self._kmax
            cshape, cst = K.collapse_view(batch + (tk, dh), kv.strides)
            self._launch("absmax", shape=cshape, x=K.View(kv.buf, cst, kv.offset), out=kmax)
        desc = K.Attn(batch[0], batch[1], tq, tk, dh, qv, kv, vv, info["scale_op"], info["scale"], mask_view,
                      tile_max, kmax, tile_zero)
        # scratch of the tensor-core path (k and v split into bf16 pieces): one buffer, sized for the
        # largest attention of the plan, reused by every launch (they run in order on one stream)
        fn = getattr(self.dev, "attention_workspace", None)
        ws = int(fn(batch[0], batch[1], tq, tk, dh)) if fn is not None else 0
        if ws > 0:
            if self._attn_ws is None or self._attn_ws_bytes < ws:
                self._attn_ws, self._attn_ws_bytes = self._alloc(ws), ws
            desc.workspace, desc.workspace_bytes = self._attn_ws, self._attn_ws_bytes
        chain = info["i8_chain"]
        if chain is not None:
            rs = chain[1]
            scale = self.i8_req[rs.result]
            rshape = tuple(rs.result.type.shape)
            dv_ = DVal(rshape, "rows", i8_scale=scale)
            dv_.i8_ld = K.round_up(dv_.cols, 16)
            dv_.i8 = self._alloc(dv_.rows * dv_.i8_ld, zero=True)
            self.vals[rs.result] = dv_
            b, h, t, d = oshape
            desc.out_i8 = K.View(dv_.i8, (t * dv_.i8_ld, d, dv_.i8_ld, 1), itemsize=1)
            desc.out_scale = scale
        else:
            strides = self._transposed_strides(mm2)
            out = self._new_out(mm2.result, strides=strides)
            if out.f32 is None:
                out.f32 = self._alloc(out.numel * 4)
                out.strides = strides
            desc.out = self._broadcast_view(out, oshape)
            if out.i8 is not None:
                ist = tuple(c * out.i8_ld for c in contiguous_strides(oshape[:-1])) + (1,)
                desc.out_i8 = K.View(out.i8, (0,) * (4 - len(oshape)) + ist, itemsize=1)
                desc.out_scale = out.i8_scale
        self._launch("attention", desc=desc)

    def _transposed_strides(self, op) -> Optional[tuple]:
        """Strides that make the transpose consuming `op`'s result row-major, if it has exactly
        one consumer and that is a transpose."""
        users = self.users.get(op.result, [])
        if len(users) != 1 or users[0].kind != "transpose" or op.result in self.g.outputs:
            return None
        oshape = tuple(op.result.type.shape)
        perm = tuple(int(p) % len(oshape) for p in users[0].attrs["perm"])
        tst = contiguous_strides(tuple(oshape[p] for p in perm))
        inv = [0] * len(oshape)
        for i, p in enumerate(perm):
            inv[p] = tst[i]
        return tuple(inv)

    def _op_matmul(self, op) -> None:
        """f32 matmul with its fused epilogue (reference ops.py:217-219) on strided views: the
        attention products q @ k^T and p @ v read the q/k/v projections where they lie."""
        if op in self.attention:
            self._attention(op, self.attention[op])
            return
        xa = self._f32_dval(op.inputs[0])
        w8 = self._w8_weight(op.inputs[1])
        wb = w8[0] if w8 is not None else self._f32_dval(op.inputs[1])
        oshape = tuple(op.result.type.shape)
        if len(oshape) > 4 or len(xa.shape) > 4 or len(wb.shape) > 4:
            raise UnsupportedOnCuda("matmul of more than 4 dimensions")
        m, kdim = xa.shape[-2:]
        n = wb.shape[-1]
        out = self._new_out(op.result, strides=self._transposed_strides(op))
        batch = (1,) * (4 - len(oshape)) + oshape[:-2]
        steps = []
        for fn, idx, swapped in op.attrs.get("epilogue", ()):
            if idx is None:
                steps.append(K.BmmStep(fn))
                continue
            val = self._const(op.inputs[idx])
            if val is not None and val.size == 1:
                steps.append(K.BmmStep(fn, "scalar", bool(swapped), scalar=float(np.float32(val.ravel()[0]))))
                continue
            ov = self._f32_dval(op.inputs[idx])
            steps.append(K.BmmStep(fn, "view", bool(swapped), view=self._broadcast_view(ov, oshape)))
        out_view = None
        if out.f32 is not None:
            out_view = self._broadcast_view(out, oshape)
        out_i8 = None
        if out.i8 is not None:
            ist = tuple(c * out.i8_ld for c in contiguous_strides(oshape[:-1])) + (1,)
            out_i8 = K.View(out.i8, (0,) * (4 - len(oshape)) + ist, itemsize=1)
        bview = self._broadcast_view(wb, oshape[:-2] + (kdim, n))
        if w8 is not None:
            bview.itemsize = 1
        self._launch("bmm", batch0=batch[0], batch1=batch[1], m=m, n=n, k=kdim,
                     a=self._broadcast_view(xa, oshape[:-2] + (m, kdim)), b=bview,
                     b_scale=w8[1] if w8 is not None else None,
                     epi=K.BmmEpi(steps, out=out_view, out_i8=out_i8,
                                  out_scale=out.i8_scale if out.i8 is not None else 1.0))

    def _w8_weight(self, v):
        """(int8 DVal, per-column f32 scales) for a matmul weight that the reference stores as a
        `dequantize` constant with one scale per output column (quantize.py:45-68 with axis = last,
        ops.py:583-587): the int8 values and the scales are uploaded once and the matmul rebuilds
        each weight as RN(f32(q) * scale) while staging it.  None for anything else."""
        p = v.producer
        if p is None or p.kind != "dequantize" or v.type.dtype != "f32":
            return None
        q = np.asarray(p.attrs["q"])
        if q.dtype != np.int8 or q.ndim < 2 or p.attrs["axis"] % q.ndim != q.ndim - 1:
            return None
        hit = self.w8_cache.get(v)
        if hit is None:
            scale = np.ascontiguousarray(np.asarray(p.attrs["scale"], np.float32).reshape(-1))
            hit = (DVal(tuple(q.shape), "rows", f32=self._upload(np.ascontiguousarray(q))), self._upload(scale))
            self.w8_cache[v] = hit
        return hit

    # ------------------------------------------------------------------ runtime-position slices

    def _start_buf(self, v):
        """Device int32 start vector of a dynamic slice: a graph input, or an uploaded constant."""
        c = self._const(v)
        if c is not None:
            return self._upload(np.ascontiguousarray(np.asarray(c, np.int32).reshape(-1)))
        dv = self.vals[v]
        if dv.i32 is None:
            raise UnsupportedOnCuda("dynamic slice start vectors must be graph inputs or constants on cuda")
        return dv.i32

    def _data_view(self, v) -> K.View:
        """4-D view of the 4-byte elements of `v` (an uploaded constant or a value on the device)."""
        c = self._const(v)
        r = v.type.rank
        if c is not None:
            c = np.ascontiguousarray(np.asarray(c, v.type.np_dtype))
            return K.View(self._upload(c), (0,) * (4 - r) + contiguous_strides(tuple(c.shape)))
        dv = self.vals[v]
        if dv.i32 is not None:
            return K.View(dv.i32, (0,) * (4 - r) + contiguous_strides(tuple(dv.shape)))
        if dv.f32 is None or dv.layout != "rows":
            raise UnsupportedOnCuda("dynamic slice of a value without a row-major f32 form")
        return self._view4(dv)[1]

    def _op_dynamic_slice(self, op) -> None:
        """Reference ops.py:550-553: the window at the clamped runtime start, copied on the device."""
        x, start = op.inputs
        size = tuple(int(n) for n in op.attrs["size"])
        rank = x.type.rank
        dv = DVal(size, "rows", f32=self._alloc(max(int(np.prod(size, dtype=np.int64)), 1) * 4))
        self.vals[op.result] = dv
        self._launch("dyn_slice", x=self._data_view(x), x_shape=tuple(x.type.shape), start=self._start_buf(start),
                     rank=rank, size=size, out=K.View(dv.f32, (0,) * (4 - rank) + contiguous_strides(size)))
        if op.result in self.i8_req:
            dv.i8_scale = self.i8_req[op.result]
            dv.i8_ld = K.round_up(dv.cols, 16)
            dv.i8 = self._alloc(dv.rows * dv.i8_ld, zero=True)
            self._fill_i8(op.result)

    def _op_dynamic_update_slice(self, op) -> None:
        """Reference ops.py:565-570.  When x is a graph input used by nothing else (a key/value
        cache fed back each step) the update is written into x's own device buffer, so the result
        aliases the input; otherwise x is copied first."""
        x, upd, start = op.inputs
        shape = tuple(x.type.shape)
        rank = len(shape)
        xdv = self.vals.get(x)
        in_place = (x in self.g.inputs and self.users.get(x, []) == [op] and x not in self.g.outputs
                    and xdv is not None and xdv.f32 is not None and xdv.layout == "rows" and xdv.is_contiguous
                    and not xdv.offset)
        if in_place:
            buf = xdv.f32
        else:
            buf = self._alloc(max(int(np.prod(shape, dtype=np.int64)), 1) * 4)
            self._launch("copy_view", shape=(1,) * (4 - rank) + shape, src=self._data_view(x),
                         dst=K.View(buf, (0,) * (4 - rank) + contiguous_strides(shape)))
        self.vals[op.result] = DVal(shape, "rows", f32=buf)
        self.aliases[op.result] = x if in_place else None
        self._launch("dyn_update", x=K.View(buf, (0,) * (4 - rank) + contiguous_strides(shape)), x_shape=shape,
                     upd=self._data_view(upd), upd_shape=tuple(upd.type.shape), start=self._start_buf(start),
                     rank=rank)

    def _logical_view(self, dv: DVal, out_shape) -> K.View:
        """4-D view of `dv` in the reference's element order (NCHW for image values, whose buffer is
        NHWC), broadcast against `out_shape`."""
        if dv.layout != "nhwc":
            return self._broadcast_view(dv, out_shape)
        n, c, h, w = dv.shape
        st = (h * w * c, 1, w * c, c)
        return K.View(dv.f32, tuple(0 if d == 1 else x for d, x in zip(dv.shape, st)), dv.offset)

    def _op_elementwise(self, op) -> None:
        """A unary or binary f32 op the reference's epilogue fusion left standalone (ops.py:99-139):
        one strided element-wise launch; scalar constants are passed as scalars."""
        oshape = tuple(op.result.type.shape)
        if len(oshape) > 4:
            raise UnsupportedOnCuda("element-wise ops of more than 4 dimensions")
        shape4 = (1,) * (4 - len(oshape)) + oshape
        unary = op.kind in _lib.UNARY_CODES
        code = _lib.UNARY_CODES.get(op.kind) or _lib.BINARY_CODES[op.kind]

        def operand(v):
            c = self._const(v)
            if c is not None and c.size == 1:
                return None, float(np.float32(np.asarray(c).ravel()[0]))
            if c is not None:
                c = np.ascontiguousarray(np.asarray(c, np.float32))
                return self._broadcast_view(DVal(tuple(c.shape), "rows", f32=self._upload(c)), oshape), None
            dv = self.vals[v]
            if dv.f32 is None:
                raise UnsupportedOnCuda("element-wise operand without an f32 form")
            return self._logical_view(dv, oshape), None

        a, a_s = operand(op.inputs[0])
        b, b_s, swapped = None, 0.0, False
        if not unary:
            b, b_s = operand(op.inputs[1])
            if a is None:                 # scalar op tensor: f(scalar, tensor)
                if b is None:
                    raise UnsupportedOnCuda("element-wise op of two scalars")
                a, b, b_s, swapped = b, None, a_s, True
        elif a is None:
            raise UnsupportedOnCuda("element-wise op of a scalar")
        out = self._new_out(op.result)
        if out.f32 is None:
            out.f32 = self._alloc(max(out.numel, 1) * 4)
        self._launch("elementwise", code=code, shape=shape4, a=a, b=b, scalar=b_s, swapped=swapped,
                     out=self._logical_view(out, oshape))
        self._fill_i8(op.result)

    _op_relu = _op_gelu = _op_sigmoid = _op_tanh = _op_elementwise
    _op_add = _op_sub = _op_mul = _op_div = _op_maximum = _op_minimum = _op_elementwise

    def _op_softmax(self, op) -> None:
        x = self.vals[op.inputs[0]]
        src, ld = self._rows_of(op.inputs[0])
        out = self._new_out(op.result)
        if out.f32 is None:
            out.f32 = self._alloc(out.numel * 4)
        self._launch("softmax", x=src, rows=x.rows, n=x.cols, ld_x=ld, out=out.f32, ld_out=out.cols)
        self._fill_i8(op.result)

    def _op_layernorm(self, op) -> None:
        x = self.vals[op.inputs[0]]
        src, ld = self._rows_of(op.inputs[0])
        g, b = (self._const(v) for v in op.inputs[1:3])
        if g is None or b is None:
            raise UnsupportedOnCuda("layernorm with runtime gamma/beta")
        out = self._new_out(op.result)
        self._launch("layernorm", x=src, rows=x.rows, d=x.cols, ld_x=ld, gamma=self._upload(g.astype(np.float32)),
                     beta=self._upload(b.astype(np.float32)), eps=op.attrs.get("eps", 1e-5), out_f32=out.f32,
                     ld_f32=out.cols, out_i8=out.i8, ld_i8=out.i8_ld, scale=out.i8_scale or 1.0)

    def _op_gather(self, op) -> None:
        """Embedding lookup (reference ops.py:482-487) of int32 token ids, with a following add of
        a constant table that repeats along the rows (learned positions) done in the same pass."""
        table = self._const(op.inputs[0]).astype(np.float32)
        idx = self.vals[op.inputs[1]]
        vocab, d = table.shape
        rows = int(np.prod(op.inputs[1].type.shape, dtype=np.int64))
        add = self._embed_addend(op)
        target = op.result
        addend, period = None, 0
        if add is not None:
            add_op, val = add
            self.skipped.add(add_op)
            target = add_op.result
            if isinstance(val, DVal):         # a row sliced at a runtime position, already on the device
                period, addend = val.numel // d, val.f32
            else:
                period = val.size // d
                addend = self._upload(np.ascontiguousarray(val.reshape(period, d), np.float32))
        out = self._new_out(target)
        if out.f32 is None:
            out.f32 = self._alloc(out.numel * 4)
        self._launch("embed", table=self._upload(table), vocab=vocab, d=d, idx=idx.i32, rows=rows, out=out.f32,
                     ld_out=d, addend=addend, addend_rows=period)
        self._fill_i8(target)

    def _embed_addend(self, op):
        """(add op, constant) when the gather's only consumer adds a constant whose shape is a
        suffix of the gathered shape (so it repeats with a period of whole rows)."""
        uses = self.users.get(op.result, [])
        if len(uses) != 1 or uses[0].kind != "add" or op.result in self.g.outputs:
            return None
        add = uses[0]
        other = add.inputs[1] if add.inputs[0] is op.result else add.inputs[0]
        val = self._const(other)
        rshape = tuple(op.result.type.shape)
        if val is None and _const_row_slice(other) and other in self.vals:
            dv = self.vals[other]
            if dv.f32 is not None and dv.is_contiguous and not dv.offset:
                val = dv
        if val is None or other is op.result or tuple(add.result.type.shape) != rshape:
            return None
        if isinstance(val, DVal):
            vshape = tuple(val.shape)
            while vshape and vshape[0] == 1:
                vshape = vshape[1:]
            ok = vshape and vshape[-1] == rshape[-1] and rshape[len(rshape) - len(vshape):] == vshape
            return (add, val) if ok else None
        vshape = tuple(val.shape)
        while vshape and vshape[0] == 1:
            vshape = vshape[1:]
        if not vshape or vshape[-1] != rshape[-1] or rshape[len(rshape) - len(vshape):] != vshape:
            return None
        return add, val.astype(np.float32)

    def _fill_i8(self, v) -> None:
        dv = self.vals[v]
        if dv.i8 is not None:
            src, ld = self._rows_of(v)
            self._launch("quantize_rows", x=src, rows=dv.rows, cols=dv.cols, ld_x=ld, scale=dv.i8_scale, xq=dv.i8,
                         ld_q=dv.i8_ld)


def _const_row_slice(v) -> bool:
    """v is a dynamic_slice of a constant table (a position-embedding row read at runtime)."""
    p = v.producer
    return (p is not None and p.kind == "dynamic_slice" and p.inputs[0].producer is not None
            and p.inputs[0].producer.is_constant_like)


def supported_reason(op) -> Optional[str]:
    """None if the cuda target runs `op`, else why not (reference Target.check, base.py:22-23)."""
    k = op.kind
    if k == "qconv2d" and conv_attrs(op.attrs)[3] != 1:
        # grouped int8 convs exist only in the opt-in int8 depthwise mode (mira_b200.int8_depthwise)
        groups = conv_attrs(op.attrs)[3]
        q = np.asarray(op.attrs["q"])
        c = op.inputs[0].type.shape[1] if op.inputs[0].type.rank == 4 else -1
        if not (groups == c == q.shape[0] and q.shape[1] == 1 and c % 4 == 0):
            return "qconv2d: grouped int8 convolutions run on cuda only as depthwise with 4k channels"
        return None
    if k in QOPS:
        return None
    if op.is_control:
        return "control flow runs on the host"
    if k == "gather":
        table, idx = op.inputs[:2]
        tp = table.producer
        if (tp is None or not tp.is_constant_like or table.type.rank != 2 or table.type.dtype != "f32"
                or idx.type.dtype != "i32" or op.attrs.get("axis", 0) not in (0, -2)):
            return "gather: the cuda target looks up rows of a constant f32 table by int32 ids"
        return None
    if k in ("dynamic_slice", "dynamic_update_slice"):
        x, start = op.inputs[0], op.inputs[-1]
        if x.type.rank > 4 or x.type.dtype not in ("f32", "i32") or start.type.dtype != "i32":
            return f"{k}: 4-byte elements, at most 4 dimensions, int32 starts on cuda"
        if start.producer is not None and not start.producer.is_constant_like:
            return f"{k}: the start vector must be a graph input or a constant on cuda"
        return None
    rank4 = op.inputs and op.inputs[0].type.rank == 4
    if any(v.type.dtype != "f32" for v in op.inputs) or op.result.type.dtype != "f32":
        return f"{k}: the cuda target computes in f32 (got {op.result.type.dtype})"
    if k == "maxpool2d" and rank4:
        return None
    if k == "pad" and rank4 and _pad_hw(op) is not None:
        return None
    if k == "reduce_mean" and rank4 and sorted(a % 4 for a in op.attrs["axes"]) == [2, 3]:
        return None
    if k in ("reshape", "transpose"):
        return None if op.result.type.rank <= 4 or k == "reshape" else f"{k}: at most 4 dimensions"
    if k in ("layernorm", "softmax"):
        x = op.inputs[0].type
        if k == "softmax" and x.rank and op.attrs.get("axis", -1) % x.rank != x.rank - 1:
            return "softmax: only over the last axis on cuda"
        if k == "layernorm" and any(v.producer is None or not v.producer.is_constant_like for v in op.inputs[1:3]):
            return "layernorm: gamma and beta must be constants on cuda"
        if not x.rank or x.shape[-1] > _lib.ROW_MAX:
            return f"{k}: rows of at most {_lib.ROW_MAX} elements on cuda"
        return None
    if k == "matmul":
        if max(v.type.rank for v in op.inputs) > 4 or op.result.type.rank > 4:
            return "matmul: at most 4 dimensions on cuda"
        return None
    if k in _lib.UNARY_CODES or k in _lib.BINARY_CODES:
        if op.result.type.rank > 4:
            return f"{k}: at most 4 dimensions on cuda"
        return None
    if k == "reshape":
        return None
    if k == "conv2d" and rank4:
        _, _, _, groups = conv_attrs(op.attrs)
        c = op.inputs[0].type.shape[1]
        w = op.inputs[1]
        if w.producer is None or not w.producer.is_constant_like:
            return "conv2d: the cuda target takes constant weights"
        if groups == 1 or (groups == c and w.type.shape[0] == c):
            return None
        return "conv2d: grouped convolutions other than depthwise run on the host"
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
        self.resident_in: set = set()
        self.resident_out: set = set()
        self._many = None            # run_many's second input buffers, pinned rings and events
        self._graph = None
        self._runs = 0
        self.compile_seconds = time.perf_counter() - t0
        self.last_seconds = 0.0

    # the pinned staging arrays: feeding these exact arrays skips a host copy
    def input_array(self, v) -> np.ndarray:
        return self.pin_in[v].view(tuple(v.type.shape), v.type.np_dtype)

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

    # ---- device-resident state (an extension beyond the reference's Executable protocol)

    def state_pairs(self) -> list:
        """(graph input, graph output) pairs whose output is the input updated in place on the
        device (dynamic_update_slice of a cache fed back every step)."""
        return [(x, y) for y, x in self.plan.aliases.items() if x is not None and y in self.g.outputs]

    def keep_resident(self, pairs=None) -> None:
        """From now on run() leaves these inputs on the device unless a feed names them, and does
        not copy these outputs back (read them with state_read)."""
        pairs = self.state_pairs() if pairs is None else list(pairs)
        known = set(self.state_pairs())
        for p in pairs:
            if tuple(p) not in known:
                raise ValueError(f"{p} is not an input/output pair updated in place")
        self.resident_in = {x for x, _ in pairs}
        self.resident_out = {y for _, y in pairs}

    def _raw(self, v):
        for u, raw, nbytes in self.plan.inputs:
            if u is v:
                return raw, nbytes
        raise KeyError(v)

    def state_write(self, v, arr: np.ndarray) -> None:
        """Copies a host array into resident input `v`."""
        raw, nbytes = self._raw(v)
        self.device.activate()
        view = self.input_array(v)
        np.copyto(view, np.asarray(arr, view.dtype).reshape(view.shape))
        self.device.h2d(raw, self.pin_in[v], nbytes)
        self.device.sync()

    def state_zero(self, v) -> None:
        raw, nbytes = self._raw(v)
        self.device.activate()
        self.device.zero(raw, nbytes)

    def state_read(self, v) -> np.ndarray:
        raw, nbytes = self._raw(v)
        self.device.activate()
        self.device.d2h(self.pin_in[v], raw, nbytes)
        self.device.sync()
        return self.input_array(v).copy()

    def run(self, feeds: dict) -> dict:
        t0 = time.perf_counter()
        self.device.activate()
        for v, raw, nbytes in self.plan.inputs:
            if v in self.resident_in and v not in feeds:
                continue
            view = self.input_array(v)
            arr = feeds[v]
            if not (isinstance(arr, np.ndarray) and arr.ctypes.data == view.ctypes.data):
                np.copyto(view, np.asarray(arr, view.dtype).reshape(view.shape))
            self.device.h2d(raw, self.pin_in[v], nbytes)
        self._launch_all()
        outs = [(v, buf, nbytes) for v, buf, nbytes in self.plan.outputs if v not in self.resident_out]
        for v, buf, nbytes in outs:
            self.device.d2h(self.pin_out[v], buf, nbytes)
        self.device.sync()
        self._runs += 1
        out = {v: self.pin_out[v].view(tuple(v.type.shape), np.float32).copy() for v, _, _ in outs}
        out.update({v: c.copy() for v, c in self.plan.const_outputs.items()})
        self.last_seconds = time.perf_counter() - t0
        return out

    def run_many(self, feeds_list, gather=None) -> list:
        """Runs one step per feeds dict, like run() each (same results), but queues step i+1's
        host-to-device input copies on the copy stream while step i's kernels run: the copies go
        to a second device buffer per input, which a device-to-device copy moves into the plan's
        input buffer at the start of the next step.  Outputs are read back through a two-slot
        pinned ring.  Inputs fed as the executable's own pinned arrays (input_array) are copied
        without a host copy; other arrays are staged through pinned buffers.

        gather: for batch-sharded runs (mira_b200.shard.DeviceGather): called after each step's
        kernels are queued, it queues the collective on the device; the step then reads back
        `gather.outputs` ((value, device buffer, bytes, shape): the gathered global batch on the
        rank that receives it, nothing on the others) instead of the plan's outputs."""
        dev = self.device
        dev.activate()
        feeds_list = list(feeds_list)
        if not feeds_list:
            return []
        ins = [(v, raw, nb) for v, raw, nb in self.plan.inputs if v not in self.resident_in]
        outs = [(v, buf, nb) for v, buf, nb in self.plan.outputs if v not in self.resident_out]
        shapes = {v: tuple(v.type.shape) for v, _, _ in outs}
        if self._many is None:
            self._many = {
                "in2": {v: dev.alloc(nb) for v, _, nb in ins},
                "stage": {v: [dev.pinned(nb), dev.pinned(nb)] for v, _, nb in ins},
                "out": {v: [self.pin_out[v], dev.pinned(nb)] for v, _, nb in outs},
                "ev": {k: [dev.event(), dev.event()] for k in ("h2d", "d2d", "done")},
                "gout": {},
            }
        m = self._many
        ev = m["ev"]
        ring = m["out"]
        if gather is not None:
            outs = [(v, buf, nb) for v, buf, nb, _ in gather.outputs]
            shapes = {v: tuple(shape) for v, _, _, shape in gather.outputs}
            for v, _, nb in outs:
                if (v, nb) not in m["gout"]:
                    m["gout"][(v, nb)] = [dev.pinned(nb), dev.pinned(nb)]
            ring = {v: m["gout"][(v, nb)] for v, _, nb in outs}
        results: list = [None] * len(feeds_list)

        def enqueue(i: int) -> None:
            slot = i % 2
            feeds = feeds_list[i]
            srcs = {}
            for v, _, nb in ins:
                arr = feeds[v]
                own = self.input_array(v)
                if isinstance(arr, np.ndarray) and arr.ctypes.data == own.ctypes.data:
                    srcs[v] = self.pin_in[v]
                    continue
                if i >= 2:
                    dev.event_sync(ev["h2d"][slot])     # the slot's previous copy has been read
                st = m["stage"][v][slot]
                view = st.view(tuple(v.type.shape), v.type.np_dtype)
                np.copyto(view, np.asarray(arr, view.dtype).reshape(view.shape))
                srcs[v] = st
            if i >= 1:
                dev.copy_wait(ev["d2d"][(i - 1) % 2])   # the previous step took its input out
            for v, _, nb in ins:
                dev.h2d_copy(m["in2"][v], srcs[v], nb)
            dev.copy_record(ev["h2d"][slot])
            dev.wait(ev["h2d"][slot])
            for v, raw, nb in ins:
                dev.d2d(raw, m["in2"][v], nb)
            dev.event_record(ev["d2d"][slot])
            self._launch_all()
            self._runs += 1
            if gather is not None:
                gather()
            for v, buf, nb in outs:
                dev.d2h(ring[v][slot], buf, nb)
            dev.event_record(ev["done"][slot])

        def collect(i: int) -> None:
            slot = i % 2
            dev.event_sync(ev["done"][slot])
            r = {v: ring[v][slot].view(shapes[v], np.float32).copy() for v, _, _ in outs}
            r.update({v: c.copy() for v, c in self.plan.const_outputs.items()})
            results[i] = r

        t0 = time.perf_counter()
        for i in range(len(feeds_list)):
            enqueue(i)
            if i >= 1:
                collect(i - 1)
        collect(len(feeds_list) - 1)
        dev.sync()
        self.last_seconds = time.perf_counter() - t0
        return results

    def device_of(self, v) -> Optional[str]:
        return f"cuda:{self.device.index}" if hasattr(self.device, "index") else "cuda"

    def report(self) -> str:
        counts = ", ".join(f"{n}x{k}" for k, n in sorted(self.plan.kernel_counts.items()))
        nq = sum(op.kind in QOPS for op in self.g.ops)
        mode = "CUDA graph" if self.use_graph else "eager launches"
        return (f"cuda:{getattr(self.device, 'index', 0)} (B200, sm_100a): {len(self.g.compute_ops())} ops, "
                f"{nq} in int8 on tcgen05; kernels: {counts}; {mode}")

    def close(self) -> None:
        if self._many is not None:
            for pair in self._many["ev"].values():
                for e in pair:
                    try:
                        self.device.event_destroy(e)
                    except Exception:
                        pass
            self._many = None
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
