"""A host-side stand-in for CudaDevice (test infrastructure).

It executes the launch records of a Plan with the CPU oracle on NumPy buffers laid out exactly as
the device buffers are (NHWC int8 with padded channels, K-major weights, padded per-channel
arrays).  Driving MIRA programs through it checks the planner - representations, layouts, strides,
epilogue operand classification - against the reference cpu target without a GPU.
"""
from __future__ import annotations

import numpy as np

from oracle import w8a8 as ref


class FakeBuf:
    def __init__(self, nbytes: int):
        self.data = np.zeros(max(int(nbytes), 16), np.uint8)
        self.nbytes = int(nbytes)

    def view(self, dtype, shape):
        n = int(np.prod(shape, dtype=np.int64))
        return self.data[: n * np.dtype(dtype).itemsize].view(dtype).reshape(shape)


class FakeSlice(FakeBuf):
    """The bytes of a FakeBuf from an offset on (shares the parent's memory)."""

    def __init__(self, parent, offset: int):
        self.data = parent.data[int(offset):]
        self.nbytes = parent.nbytes - int(offset)


def _strided(view, shape4, dtype=np.float32):
    """NumPy array over a kernels.View (element offset and strides) of a FakeBuf."""
    item = np.dtype(dtype).itemsize
    base = view.buf.data[int(view.offset) * item:].view(dtype)
    return np.lib.stride_tricks.as_strided(base, tuple(int(d) for d in shape4),
                                           tuple(int(s) * item for s in view.strides))


def _pad4(shape) -> tuple:
    shape = tuple(int(d) for d in shape)
    return (1,) * (4 - len(shape)) + shape


class FakePinned(FakeBuf):
    def view(self, shape, dtype):  # PinnedBuffer's argument order
        return super().view(dtype, shape)


class FakeDevice:
    name = "fake"
    index = 0

    def __init__(self):
        self.launched: list[str] = []

    def activate(self):
        pass

    def alloc(self, nbytes, zero=False):
        return FakeBuf(nbytes)

    def upload(self, arr):
        arr = np.ascontiguousarray(arr)
        b = FakeBuf(arr.nbytes)
        b.data[: arr.nbytes] = arr.reshape(-1).view(np.uint8)
        return b

    def pinned(self, nbytes):
        return FakePinned(nbytes)

    def offset(self, buf, nbytes):
        return FakeSlice(buf, nbytes)

    def h2d(self, dst, src, nbytes):
        dst.data[:nbytes] = src.data[:nbytes]

    def d2h(self, dst, src, nbytes):
        dst.data[:nbytes] = src.data[:nbytes]

    def sync(self):
        pass

    def zero(self, buf, nbytes):
        buf.data[:nbytes] = 0

    # the copy stream and events: everything here completes at once, in program order
    def event(self):
        return object()

    def event_destroy(self, ev):
        pass

    def event_record(self, ev):
        pass

    def event_sync(self, ev):
        pass

    def wait(self, ev):
        pass

    def copy_record(self, ev):
        pass

    def copy_wait(self, ev):
        pass

    def h2d_copy(self, dst, src, nbytes):
        dst.data[:nbytes] = src.data[:nbytes]

    def d2d(self, dst, src, nbytes):
        dst.data[:nbytes] = src.data[:nbytes]

    def thunk(self, launch):
        fn = getattr(self, "_" + launch.kind)
        return lambda: (self.launched.append(launch.kind), fn(**launch.args))

    # ------------------------------------------------------------------ kernels

    def _quantize_rows(self, x, rows, cols, ld_x, scale, xq, ld_q):
        xv = x.view(np.float32, (rows, ld_x))[:, :cols]
        q = xq.view(np.int8, (rows, ld_q))
        q[:, :cols] = ref.quantize_activation(xv, scale)
        q[:, cols:] = 0

    def _quantize_nchw(self, x, n, c, h, w, scale, xq, cp):
        q = xq.view(np.int8, (n, h, w, cp))
        q[..., :c] = ref.quantize_activation(x.view(np.float32, (n, c, h, w)), scale).transpose(0, 2, 3, 1)
        q[..., c:] = 0

    def _quantize_row4(self, x, n, c, h, w, scale, xq, row_entries, pad, stride=1):
        """Entry e of a row holds pixels stride*e - pad .. stride*e - pad + 3 (4 channels each)."""
        q = np.zeros((n, h, stride * row_entries + 4 + 2 * pad, 4), np.int8)
        q[:, :, pad:pad + w, :c] = ref.quantize_activation(x.view(np.float32, (n, c, h, w)), scale).transpose(0, 2, 3, 1)
        out = xq.view(np.int8, (n, h, row_entries, 16))
        first = stride * np.arange(row_entries)            # index of pixel stride*e - pad in q
        for k in range(4):
            out[..., 4 * k:4 * k + 4] = q[:, :, first + k, :]

    @staticmethod
    def _conv_operands(x, n, h, w, cp, layout, row_entries, wq, o, kh, kw, ldw, pad_w, stride_w=1):
        """NCHW int8 input and OIHW weights, whatever the device layout."""
        if layout == 1:
            rows = x.view(np.int8, (n, h, row_entries, 16))
            full = np.zeros((n, h, stride_w * row_entries + 4, 4), np.int8)
            for k in range(4):             # pixel stride*e - pad + k is byte group k of entry e
                full[:, :, stride_w * np.arange(row_entries) + k, :] = rows[..., 4 * k:4 * k + 4]
            xn = full[:, :, pad_w:pad_w + w, :].transpose(0, 3, 1, 2)
            wt = wq.view(np.int8, (o, ldw))[:, : kh * 32].reshape(o, kh, 8, 4)[:, :, :kw, :].transpose(0, 3, 1, 2)
            return xn, wt
        if layout == 2:                    # chunk-planar, zero-padded
            from mira_b200 import kernels as K
            xn = K.from_cp(x.data[:K.cp_bytes(n, h, w, cp)].view(np.int8), n, h, w, cp).transpose(0, 3, 1, 2)
        else:
            xn = x.view(np.int8, (n, h, w, cp)).transpose(0, 3, 1, 2)
        wt = wq.view(np.int8, (o, ldw))[:, : kh * kw * cp].reshape(o, kh, kw, cp).transpose(0, 3, 1, 2)
        return xn, wt

    def _nchw_to_nhwc(self, x, n, c, h, w, y, ldc):
        y.view(np.float32, (n, h, w, ldc))[..., :c] = x.view(np.float32, (n, c, h, w)).transpose(0, 2, 3, 1)

    def _nhwc_to_nchw(self, x, n, h, w, c, ldc, y):
        y.view(np.float32, (n, c, h, w))[...] = x.view(np.float32, (n, h, w, ldc))[..., :c].transpose(0, 3, 1, 2)

    def _copy(self, dst, src, nbytes):
        dst.data[:nbytes] = src.data[:nbytes]

    @staticmethod
    def _put_i8(buf, q, ld, layout, geom):
        """int8 rows [M, N] into `buf`: rows of ld bytes, or (layout 2) the chunk-planar layout of
        the [n, oh, ow, ld] activation geom = (n, oh, ow) (its padding stays zero)."""
        m, nc = q.shape
        if layout == 2:
            from mira_b200 import kernels as K
            n, oh, ow = geom
            full = np.zeros((n, oh, ow, ld), np.int8)
            full.reshape(m, ld)[:, :nc] = q
            enc = K.to_cp(full)
            buf.data[:enc.size] = enc.view(np.uint8)
            return
        rows = buf.view(np.int8, (m, ld))
        rows[:, :nc] = q
        rows[:, nc:] = 0

    def _epi(self, y, epi, M, N, geom=None):
        """y: f32 [M, N] dequantized; applies steps and writes the outputs."""
        for s in epi.steps:
            if s.operand == "none":
                y = ref.UNARY[s.op](y).astype(np.float32)
                continue
            if s.operand == "scalar":
                o = np.float32(s.scalar)
            elif s.operand == "channel":
                o = s.ptr.view(np.float32, (N,))
            elif s.operand == "full":
                o = s.ptr.view(np.float32, (M, s.ld))[:, :N]
            else:
                o = s.ptr.view(np.float32, (M, 1))
            y = (ref.BINARY[s.op](o, y) if s.swapped else ref.BINARY[s.op](y, o)).astype(np.float32)
        if epi.out_f32 is not None:
            epi.out_f32.view(np.float32, (M, epi.ld_f32))[:, :N] = y
        if epi.out_i8 is not None:
            self._put_i8(epi.out_i8, ref.quantize_activation(y, epi.out_scale), epi.ld_i8, epi.i8_layout, geom)

    def _dequant(self, acc, dq, N):
        s64 = dq[0].view(np.float64, (N,))
        return (acc.astype(np.float64) * s64).astype(np.float32)

    def qgemm_workspace(self, M, N, K, sm_count=148):
        """The library's split-K rule (mira_cuda.cu splitk_plan) for a 148-SM device."""
        one_row = M <= 128
        num_kb = -(-K // 128)
        bn = 64 if N <= 64 else (128 if N <= 128 else 256)
        if one_row:                    # the widest tile whose split plan fills 3/4 of the SMs
            best, best_bn, w = -1, 64, bn
            while w >= 64:
                t = -(-N // w)
                sp = 1 if t * 2 > sm_count else min(sm_count // t, num_kb, 16)
                if t * max(sp, 1) * 4 >= sm_count * 3:
                    best_bn = w
                    break
                if t * max(sp, 1) > best:
                    best, best_bn = t * max(sp, 1), w
                w //= 2
            bn = best_bn
        tiles = -(-M // 128) * -(-N // bn)
        if tiles * 2 > sm_count or (not one_row and num_kb < 8):
            return 0
        s = min(sm_count // tiles, num_kb if one_row else num_kb // 4, 16)
        if s < 2:
            return 0
        per = -(-num_kb // s)
        s = -(-num_kb // per)
        return s * M * N * 4 if s > 1 else 0

    def _qgemm(self, M, N, K, A, lda, B, ldb, dq, epi, ws=None, ws_bytes=0):
        if ws is not None:
            assert ws_bytes == self.qgemm_workspace(M, N, K) and ws.nbytes >= ws_bytes
        a = A.view(np.int8, (M, lda))[:, :K]
        b = B.view(np.int8, (N, ldb))[:, :K]
        acc = ref.int_matmul(a, b.T)
        self._epi(self._dequant(acc, dq, N), epi, M, N)

    def _qconv2d(self, n, h, w, cp, x, o, kh, kw, wq, ldw, stride, padding, dilation, dq, epi, layout=0, row_entries=0):
        xn, wt = self._conv_operands(x, n, h, w, cp, layout, row_entries, wq, o, kh, kw, ldw, padding[1], stride[1])
        acc = ref.int_conv2d(xn, wt, stride, padding, dilation)       # [n, o, oh, ow]
        oh, ow = acc.shape[2:]
        rows = acc.transpose(0, 2, 3, 1).reshape(n * oh * ow, o)
        self._epi(self._dequant(rows, dq, o), epi, n * oh * ow, o, geom=(n, oh, ow))

    def _qconv2d_pool(self, n, h, w, cp, x, o, kh, kw, wq, ldw, stride, padding, dilation, pool_size, pool_stride,
                      pool_pad, pool_pad_value, dq, epi, layout=0, row_entries=0):
        xn, wt = self._conv_operands(x, n, h, w, cp, layout, row_entries, wq, o, kh, kw, ldw, padding[1], stride[1])
        acc = ref.int_conv2d(xn, wt, stride, padding, dilation)
        oh, ow = acc.shape[2:]
        rows = self._dequant(acc.transpose(0, 2, 3, 1).reshape(-1, o), dq, o)
        conv_out = FakeBuf(rows.size * 4)
        import copy
        inner = copy.copy(epi)
        inner.out_f32, inner.ld_f32, inner.out_i8 = conv_out, o, None
        self._epi(rows, inner, n * oh * ow, o)
        y = conv_out.view(np.float32, (n, oh, ow, o)).transpose(0, 3, 1, 2)
        pooled = ref.maxpool2d(y, pool_size, pool_stride, pool_pad, pool_pad_value)
        ph, pw = pooled.shape[2:]
        flat = pooled.transpose(0, 2, 3, 1).reshape(-1, o)
        if epi.out_f32 is not None:
            epi.out_f32.view(np.float32, (n * ph * pw, epi.ld_f32))[:, :o] = flat
        if epi.out_i8 is not None:
            self._put_i8(epi.out_i8, ref.quantize_activation(flat, epi.out_scale), epi.ld_i8, epi.i8_layout,
                         (n, ph, pw))

    def _maxpool(self, n, h, w, c, ldc, size, stride, pad, pad_value, x_f32=None, x_i8=None, out_f32=None, ldo=0,
                 out_i8=None, ldo_i8=0, scale=1.0, i8_layout=0):
        xv = x_f32.view(np.float32, (n, h, w, ldc))[..., :c].transpose(0, 3, 1, 2)
        y = ref.maxpool2d(xv, size, stride, pad, pad_value)
        oh, ow = y.shape[2:]
        rows = y.transpose(0, 2, 3, 1).reshape(-1, c)
        if out_f32 is not None:
            out_f32.view(np.float32, (n * oh * ow, ldo))[:, :c] = rows
        if out_i8 is not None:
            self._put_i8(out_i8, ref.quantize_activation(rows, scale), ldo_i8, i8_layout, (n, oh, ow))

    def _mean_hw(self, x, n, hw, c, ldc, out_f32=None, out_i8=None, ld_i8=0, scale=1.0):
        xv = x.view(np.float32, (n, hw, ldc))[..., :c].transpose(0, 2, 1)
        m = ref.mean_hw(np.ascontiguousarray(xv).reshape(n, c, hw, 1))
        if out_f32 is not None:
            out_f32.view(np.float32, (n, c))[...] = m
        if out_i8 is not None:
            out_i8.view(np.int8, (n, ld_i8))[:, :c] = ref.quantize_activation(m, scale)

    def _elementwise(self, code, shape, a, out, b=None, scalar=0.0, swapped=False):
        from mira_b200 import _lib
        names = {v: k for k, v in {**_lib.UNARY_CODES, **_lib.BINARY_CODES}.items()}
        op = names[code]
        x = _strided(a, shape).astype(np.float32)
        if op in ref.UNARY:
            y = ref.UNARY[op](x)
        else:
            o = _strided(b, shape) if b is not None else np.float32(scalar)
            y = ref.BINARY[op](o, x) if swapped else ref.BINARY[op](x, o)
        _strided(out, shape)[...] = np.asarray(y, np.float32)

    def _im2col(self, x, n, h, w, c, ldc, kh, kw, stride, padding, dilation, out, ld_out):
        (sh, sw), (ph, pw), (dh, dw) = stride, padding, dilation
        xp = np.zeros((n, h + 2 * ph, w + 2 * pw, c), np.float32)
        xp[:, ph:ph + h, pw:pw + w, :] = x.view(np.float32, (n, h, w, ldc))[..., :c]
        oh = (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1
        ow = (w + 2 * pw - dw * (kw - 1) - 1) // sw + 1
        cols = []
        for i in range(kh):
            for j in range(kw):
                cols.append(xp[:, i * dh:i * dh + sh * (oh - 1) + 1:sh, j * dw:j * dw + sw * (ow - 1) + 1:sw, :])
        out.view(np.float32, (n * oh * ow, ld_out))[:, :kh * kw * c] = np.concatenate(cols, axis=-1).reshape(-1, kh * kw * c)

    def _qdwconv(self, x, ldx, n, h, w, c, wq, kh, kw, stride, padding, dilation, dq, epi):
        xn = x.view(np.int8, (n, h, w, ldx))[..., :c].transpose(0, 3, 1, 2)
        q = wq.view(np.int8, (kh * kw, c)).T.reshape(c, 1, kh, kw)
        acc = ref.int_dwconv2d(xn, q, stride, padding, dilation)
        oh, ow = acc.shape[2:]
        rows = acc.transpose(0, 2, 3, 1).reshape(n * oh * ow, c)
        self._epi(self._dequant(rows, dq, c), epi, n * oh * ow, c, geom=(n, oh, ow))

    def _dwconv(self, x, n, h, w, c, wt, kh, kw, stride, padding, dilation, epi):
        xn = x.view(np.float32, (n, h, w, c)).transpose(0, 3, 1, 2)
        wk = wt.view(np.float32, (kh * kw, c)).T.reshape(c, 1, kh, kw)
        y = ref.dwconv2d(xn, wk, stride, padding, dilation)
        oh, ow = y.shape[2:]
        self._epi(y.transpose(0, 2, 3, 1).reshape(-1, c), epi, n * oh * ow, c)

    # ------------------------------------------------------------------ sequence ops

    def _bmm(self, batch0, batch1, m, n, k, a, b, epi, b_scale=None):
        av = _strided(a, (batch0, batch1, m, k))
        if b_scale is None:
            bv = _strided(b, (batch0, batch1, k, n))
        else:                        # int8 weights, one scale per column (the reference's dequantize)
            bv = _strided(b, (batch0, batch1, k, n), np.int8).astype(np.float32) * b_scale.view(np.float32, (n,))
        y = np.matmul(av.astype(np.float32), bv.astype(np.float32))
        for st in epi.steps:
            if st.operand == "none":
                y = ref.UNARY[st.op](y).astype(np.float32)
                continue
            o = np.float32(st.scalar) if st.operand == "scalar" else _strided(st.view, (batch0, batch1, m, n))
            y = (ref.BINARY[st.op](o, y) if st.swapped else ref.BINARY[st.op](y, o)).astype(np.float32)
        if epi.out is not None:
            _strided(epi.out, (batch0, batch1, m, n))[...] = y
        if epi.out_i8 is not None:
            _strided(epi.out_i8, (batch0, batch1, m, n), np.int8)[...] = ref.quantize_activation(y, epi.out_scale)

    def _layernorm(self, x, rows, d, ld_x, gamma, beta, eps, out_f32=None, ld_f32=0, out_i8=None, ld_i8=0, scale=1.0):
        xv = x.view(np.float32, (rows, ld_x))[:, :d]
        y = ref.layernorm(xv, gamma.view(np.float32, (d,)), beta.view(np.float32, (d,)), eps)
        if out_f32 is not None:
            out_f32.view(np.float32, (rows, ld_f32))[:, :d] = y
        if out_i8 is not None:
            out_i8.view(np.int8, (rows, ld_i8))[:, :d] = ref.quantize_activation(y, scale)

    def _softmax(self, x, rows, n, ld_x, out, ld_out):
        out.view(np.float32, (rows, ld_out))[:, :n] = ref.softmax(x.view(np.float32, (rows, ld_x))[:, :n])

    def _embed(self, table, vocab, d, idx, rows, out, ld_out, addend=None, addend_rows=0):
        ids = idx.view(np.int32, (rows,))
        add = None
        if addend is not None:
            add = np.tile(addend.view(np.float32, (addend_rows, d)), (rows // addend_rows, 1))
        out.view(np.float32, (rows, ld_out))[:, :d] = ref.embed(table.view(np.float32, (vocab, d)), ids, add)

    @staticmethod
    def _window(start, rank, dims, n):
        """Clamped starts over 4 dimensions (reference _clamped_starts, ops.py:536-537)."""
        st = [0] * 4
        vals = start.view(np.int32, (rank,)) if rank else []
        for j in range(rank):
            d = 4 - rank + j
            st[d] = int(min(max(int(vals[j]), 0), dims[d] - n[d]))
        return tuple(slice(s, s + k) for s, k in zip(st, n))

    def _dyn_slice(self, x, x_shape, start, rank, size, out):
        dims, n = _pad4(x_shape), _pad4(size)
        _strided(out, n)[...] = _strided(x, dims)[self._window(start, rank, dims, n)]

    def _dyn_update(self, x, x_shape, upd, upd_shape, start, rank):
        dims, n = _pad4(x_shape), _pad4(upd_shape)
        _strided(x, dims)[self._window(start, rank, dims, n)] = _strided(upd, n)

    def _copy_view(self, shape, src, dst):
        _strided(dst, shape)[...] = _strided(src, shape)

    def _absmax(self, shape, x, out):
        out.view(np.float32, (1,))[0] = np.abs(_strided(x, shape)).max() if np.prod(shape) else 0.0

    def _attention(self, desc):
        d = desc
        q = _strided(d.q, (d.batch0, d.batch1, d.tq, d.dh))
        k = _strided(d.k, (d.batch0, d.batch1, d.tk, d.dh))
        v = _strided(d.v, (d.batch0, d.batch1, d.tk, d.dh))
        steps, operands = [], []
        if d.scale_op is not None:
            steps.append((d.scale_op, len(operands), False))
            operands.append(np.float32(d.scale))
        if d.mask is not None:
            steps.append(("add", len(operands), False))
            operands.append(_strided(d.mask, (d.batch0, d.batch1, d.tq, d.tk)))
        s = ref.matmul_f32(q, np.swapaxes(k, -1, -2), steps, operands)
        o = ref.matmul_f32(ref.softmax(s), v)
        if d.out is not None:
            _strided(d.out, o.shape)[...] = o
        if d.out_i8 is not None:
            _strided(d.out_i8, o.shape, np.int8)[...] = ref.quantize_activation(o, d.out_scale)
