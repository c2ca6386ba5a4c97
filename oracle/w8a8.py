"""CPU oracle for the W8A8 hot path — TEST INFRASTRUCTURE ONLY.

A NumPy restatement of the reference's arithmetic for the path `mira run ... --quantize w8a8`
(myramay/MIRA, mira/ops.py).  Only the tests, `__graft_entry__.smoke()` and bench.py's CPU-baseline
leg use it, as the checker; the product (mira_b200) never imports it.

Pinning: tests/golden/*.npz hold input/output vectors produced by running the reference itself
(tests/golden/make_golden.py imports the reference's `mira.ops` / `mira.compile_ir`), and
tests/test_oracle.py checks every function here against them bit for bit.

Every function cites the reference line it restates.  Integer results are exact by construction
(int64 / exact float64 sums); f32 results follow the reference's rounding steps one by one.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------------------------
# quantization


def quantize_activation(x: np.ndarray, scale: float) -> np.ndarray:
    """int8 of clip(round(f32(x) / f32(scale)), -127, 127).  Reference ops.py:602-603 (which returns
    the integer values as floats; round is half-to-even)."""
    q = np.clip(np.round(np.asarray(x, np.float32) / np.float32(scale)), -127, 127)
    return q.astype(np.int8)


def quantize_array(w: np.ndarray, axis: int) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-channel int8 weights.  Reference quantize.py:24-31."""
    red = tuple(i for i in range(w.ndim) if i != axis)
    amax = np.abs(w.astype(np.float32)).max(axis=red)
    scale = np.where(amax > 0, amax / 127.0, 1.0).astype(np.float32)
    shape = [1] * w.ndim
    shape[axis] = -1
    q = np.clip(np.round(w.astype(np.float32) / scale.reshape(shape)), -127, 127).astype(np.int8)
    return q, scale


def dequantize(q: np.ndarray, scale: np.ndarray, axis: int) -> np.ndarray:
    """The weight-only int8 constant: f32(q) * scale broadcast along `axis`, one f32 rounding per
    weight.  Reference ops.py:583-587 (with dtype f32)."""
    shape = [1] * q.ndim
    shape[axis] = -1
    return q.astype(np.float32) * np.asarray(scale, np.float32).reshape(shape)


def combined_scale(x_scale: float, w_scale: np.ndarray) -> np.ndarray:
    """float64 x_scale * w_scale[c], the dequant factor of ops.py:619 / ops.py:633."""
    return np.float64(x_scale) * np.asarray(w_scale).astype(np.float64)


# ---------------------------------------------------------------------------------------------
# epilogue (reference ops.py:192-199 with the UNARY/BINARY tables of ops.py:94-139)


def _gelu(x):
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


UNARY = {
    "relu": lambda x: np.maximum(x, 0),
    "gelu": _gelu,
    "sigmoid": lambda x: 1.0 / (1.0 + np.exp(-x)),
    "tanh": np.tanh,
}
BINARY = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide,
          "maximum": np.maximum, "minimum": np.minimum}


def epilogue(acc: np.ndarray, operands: list, steps) -> np.ndarray:
    """Apply (fn, idx, swapped) steps to an f32 array; `operands[idx]` broadcasts against acc.
    Reference ops.py:192-199."""
    for fn, idx, swapped in steps:
        if idx is None:
            acc = UNARY[fn](acc)
        else:
            other = np.asarray(operands[idx]).astype(np.float32, copy=False)
            acc = BINARY[fn](other, acc) if swapped else BINARY[fn](acc, other)
    return acc


# ---------------------------------------------------------------------------------------------
# integer products


def int_matmul(a_q: np.ndarray, b_q: np.ndarray) -> np.ndarray:
    """Exact int64 a_q[M, K] @ b_q[K, N] (float64 BLAS is exact while |sums| < 2^53, which holds
    for int8 operands with K < 5e11; the reference uses int64 np.matmul, ops.py:617)."""
    return np.matmul(a_q.astype(np.float64), b_q.astype(np.float64)).astype(np.int64)


def dequant(acc: np.ndarray, scale64: np.ndarray) -> np.ndarray:
    """f32(f64(acc) * scale64), scale64 broadcasting along the last axis.  Reference ops.py:618."""
    return (acc.astype(np.float64) * scale64).astype(np.float32)


def qmatmul(x: np.ndarray, q: np.ndarray, w_scale: np.ndarray, x_scale: float, steps=(), operands=()):
    """Reference ops.py:616-620 (_qmatmul_ref).  x f32 [..., K]; q int8 [K, N] (reference layout).
    Returns (xq int8, acc int64, y f32) so tests can check every intermediate."""
    xq = quantize_activation(x, x_scale)
    acc = int_matmul(xq.reshape(-1, xq.shape[-1]), q).reshape(x.shape[:-1] + (q.shape[1],))
    y = dequant(acc, combined_scale(x_scale, w_scale))
    y = epilogue(y, [x, *operands], steps).astype(np.float32)
    return xq, acc, y


def qgemm_rowcol(a: np.ndarray, b_kn: np.ndarray, row_scale: np.ndarray, col_scale: np.ndarray,
                 bias: np.ndarray | None = None):
    """The standalone GEMM sweep (no reference counterpart; a restatement of ops.py:618 with a
    per-row activation scale): acc = A @ B exact, y = f32(f64(acc) * (f64(r[m]) * f64(c[n]))) + bias.
    With a constant row scale this is _qmatmul_ref on x = A (x_scale = row scale)."""
    acc = int_matmul(a, b_kn)
    s = row_scale.astype(np.float64)[:, None] * col_scale.astype(np.float64)[None, :]
    y = (acc.astype(np.float64) * s).astype(np.float32)
    if bias is not None:
        y = np.add(y, bias.astype(np.float32))
    return acc, y


# ---------------------------------------------------------------------------------------------
# convolutions


def _conv_out(size, k, stride, pad, dil):
    return (size + 2 * pad - dil * (k - 1) - 1) // stride + 1


def int_conv2d(xq: np.ndarray, q: np.ndarray, stride, padding, dilation=(1, 1)) -> np.ndarray:
    """Exact integer conv of NCHW int8 xq with OIHW int8 q (groups = 1), int64 NCHW result.
    Reference _conv2d_ref ops.py:265-276 sums one f32 einsum per tap; for int8 operands every
    partial sum is an integer and is exact while below 2^24, so the two agree (checked by
    `conv_sums_exact_in_f32`)."""
    n, c, h, w = xq.shape
    o, ci, kh, kw = q.shape
    assert ci == c, "groups != 1 is not a W8A8 conv"
    (sh, sw), (ph, pw), (dh, dw) = stride, padding, dilation
    oh, ow = _conv_out(h, kh, sh, ph, dh), _conv_out(w, kw, sw, pw, dw)
    xp = np.pad(xq.astype(np.float64), ((0, 0), (0, 0), (ph, ph), (pw, pw)))
    acc = np.zeros((n, o, oh, ow), np.float64)
    qf = q.astype(np.float64)
    for i in range(kh):
        for j in range(kw):
            xt = xp[:, :, i * dh:i * dh + sh * (oh - 1) + 1:sh, j * dw:j * dw + sw * (ow - 1) + 1:sw]
            acc += np.einsum("nchw,oc->nohw", xt, qf[:, :, i, j], optimize=True)
    return acc.astype(np.int64)


def conv_sums_exact_in_f32(xq: np.ndarray, q: np.ndarray) -> bool:
    """True when every per-tap partial sum of the reference's f32 accumulation is below 2^24 in
    magnitude (a sufficient bound: 127 * sum|q| per output channel)."""
    bound = 127.0 * np.abs(q.astype(np.float64)).reshape(q.shape[0], -1).sum(axis=1).max()
    return bool(bound < 2 ** 24)


def qconv2d(x: np.ndarray, q: np.ndarray, w_scale: np.ndarray, x_scale: float, stride, padding,
            dilation=(1, 1), steps=(), operands=()):
    """Reference ops.py:630-634 (_qconv2d_ref).  x f32 NCHW; q int8 OIHW.  Returns (xq, acc, y)."""
    xq = quantize_activation(x, x_scale)
    acc = int_conv2d(xq, q, stride, padding, dilation)
    s = combined_scale(x_scale, w_scale).reshape(1, -1, 1, 1)
    y = (acc.astype(np.float64) * s).astype(np.float32)
    y = epilogue(y, [x, *operands], steps).astype(np.float32)
    return xq, acc, y


def int_dwconv2d(xq: np.ndarray, q: np.ndarray, stride, padding, dilation=(1, 1)) -> np.ndarray:
    """Exact integer depthwise conv (groups == channels) of NCHW int8 xq with int8 q [c, 1, kh, kw],
    int64 NCHW result: the grouped branch of reference _conv2d_ref (ops.py:265-276; one einsum term
    per tap and group, `acc +=`) on int8 operands, whose f32 partial sums are integers below 2^24."""
    n, c, h, w = xq.shape
    o, cg, kh, kw = q.shape
    assert cg == 1 and o == c, "a depthwise conv has one weight per channel and tap"
    (sh, sw), (ph, pw), (dh, dw) = stride, padding, dilation
    oh, ow = _conv_out(h, kh, sh, ph, dh), _conv_out(w, kw, sw, pw, dw)
    xp = np.pad(xq.astype(np.int64), ((0, 0), (0, 0), (ph, ph), (pw, pw)))
    acc = np.zeros((n, c, oh, ow), np.int64)
    for i in range(kh):
        for j in range(kw):
            xt = xp[:, :, i * dh:i * dh + sh * (oh - 1) + 1:sh, j * dw:j * dw + sw * (ow - 1) + 1:sw]
            acc += xt * q[:, 0, i, j].astype(np.int64).reshape(1, c, 1, 1)
    return acc


def qdwconv2d(x: np.ndarray, q: np.ndarray, w_scale: np.ndarray, x_scale: float, stride, padding,
              dilation=(1, 1), steps=(), operands=()):
    """Reference _qconv2d_ref (ops.py:630-634) of a depthwise qconv2d (the opt-in int8 depthwise
    mode): quantize x, exact integer sums over the taps, dequant f32(f64(acc) * S[c]), epilogue.
    Returns (xq, acc, y)."""
    xq = quantize_activation(x, x_scale)
    acc = int_dwconv2d(xq, q, stride, padding, dilation)
    s = combined_scale(x_scale, w_scale).reshape(1, -1, 1, 1)
    y = (acc.astype(np.float64) * s).astype(np.float32)
    y = epilogue(y, [x, *operands], steps).astype(np.float32)
    return xq, acc, y


def dwconv2d(x: np.ndarray, w: np.ndarray, stride, padding, dilation=(1, 1), steps=(), operands=()):
    """f32 depthwise conv (groups == channels), reference _conv2d_ref ops.py:265-276: per tap (i, j)
    in order, acc += x_tap * w[c, 0, i, j] in float32 starting from 0."""
    n, c, h, wd = x.shape
    o, cg, kh, kw = w.shape
    assert cg == 1 and o == c
    (sh, sw), (ph, pw), (dh, dw) = stride, padding, dilation
    oh, ow = _conv_out(h, kh, sh, ph, dh), _conv_out(wd, kw, sw, pw, dw)
    xp = np.pad(x.astype(np.float32), ((0, 0), (0, 0), (ph, ph), (pw, pw)))
    acc = np.zeros((n, c, oh, ow), np.float32)
    for i in range(kh):
        for j in range(kw):
            xt = xp[:, :, i * dh:i * dh + sh * (oh - 1) + 1:sh, j * dw:j * dw + sw * (ow - 1) + 1:sw]
            acc += xt * w[:, 0, i, j].astype(np.float32).reshape(1, c, 1, 1)
    return epilogue(acc, [x, w, *operands], steps).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# f32 ops between the quantized ones


def maxpool2d(x: np.ndarray, size: int, stride: int, pad: int = 0, pad_value: float = -np.inf):
    """Reference pad (ops.py:469-470) with `pad_value` then maxpool2d (ops.py:293-296), NCHW."""
    if pad:
        x = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)), constant_values=np.float32(pad_value))
    win = np.lib.stride_tricks.sliding_window_view(x, (size, size), axis=(2, 3))[:, :, ::stride, ::stride]
    return win.max(axis=(-2, -1)).astype(x.dtype)


def _pairwise_block(v: np.ndarray) -> np.float32:
    n = len(v)
    if n < 8:
        r = np.float32(0)
        for t in v:
            r = np.float32(r + t)
        return r
    acc = [np.float32(v[j]) for j in range(8)]
    i = 8
    while i < n - (n % 8):
        for j in range(8):
            acc[j] = np.float32(acc[j] + v[i + j])
        i += 8
    r = np.float32(np.float32(np.float32(acc[0] + acc[1]) + np.float32(acc[2] + acc[3]))
                   + np.float32(np.float32(acc[4] + acc[5]) + np.float32(acc[6] + acc[7])))
    while i < n:
        r = np.float32(r + v[i])
        i += 1
    return r


def pairwise_sum_f32(v: np.ndarray) -> np.float32:
    """NumPy's float32 pairwise summation order (what np.sum / np.mean use on a contiguous axis)."""
    v = np.asarray(v, np.float32)
    if len(v) <= 128:
        return _pairwise_block(v)
    n2 = len(v) // 2
    n2 -= n2 % 8
    return np.float32(pairwise_sum_f32(v[:n2]) + pairwise_sum_f32(v[n2:]))


def mean_hw(x: np.ndarray) -> np.ndarray:
    """x.mean(axis=(2, 3)) of NCHW f32 written out in NumPy's summation order (reference
    reduce_mean, ops.py:318-343).  Equal to np.mean bit for bit; tests check that."""
    n, c = x.shape[:2]
    flat = x.reshape(n, c, -1)
    out = np.empty((n, c), np.float32)
    cnt = np.float32(flat.shape[2])
    for i in range(n):
        for j in range(c):
            out[i, j] = np.float32(pairwise_sum_f32(flat[i, j]) / cnt)
    return out


# ---------------------------------------------------------------------------------------------
# f32 sequence ops of the transformer (reference ops.py:217-219, 310-313, 356-360, 482-487).
# These restate the reference's NumPy expressions operation by operation; np.exp / np.tanh and
# the BLAS matmul are NumPy's own, so the device kernels agree with these to f32 rounding while
# layernorm (pairwise sums, IEEE divide and sqrt) agrees bit for bit.


def layernorm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """Reference _layernorm_ref, ops.py:356-360."""
    x, g, b = (np.asarray(v, np.float32) for v in (x, gamma, beta))
    mu = x.mean(axis=-1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=-1, keepdims=True)
    return ((x - mu) / np.sqrt(var + eps) * g + b).astype(np.float32)


def layernorm_rows_explicit(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """layernorm written with pairwise_sum_f32 row by row (the device kernel's order); tests
    check it equals `layernorm` bit for bit."""
    x = np.asarray(x, np.float32)
    rows = x.reshape(-1, x.shape[-1])
    out = np.empty_like(rows)
    d = np.float32(rows.shape[1])
    e = np.float32(eps)
    for r in range(rows.shape[0]):
        mu = np.float32(pairwise_sum_f32(rows[r]) / d)
        t = (rows[r] - mu).astype(np.float32)
        var = np.float32(pairwise_sum_f32((t * t).astype(np.float32)) / d)
        sd = np.sqrt(np.float32(var + e))
        out[r] = (t / sd * np.asarray(gamma, np.float32) + np.asarray(beta, np.float32)).astype(np.float32)
    return out.reshape(x.shape)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Reference _softmax_ref, ops.py:310-313."""
    x = np.asarray(x, np.float32)
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)


def matmul_f32(x: np.ndarray, w: np.ndarray, steps=(), operands=()) -> np.ndarray:
    """Reference _matmul_ref, ops.py:217-219: np.matmul of f32 operands, then the epilogue."""
    acc = np.matmul(np.asarray(x, np.float32), np.asarray(w, np.float32))
    return epilogue(acc, list(operands), steps).astype(np.float32)


def matmul_error_bound(x: np.ndarray, w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(exact float64 product, K * 2^-23 * |x| @ |w|): any f32 accumulation order of the K
    products lies within the bound of the exact value (standard dot-product error analysis)."""
    x64, w64 = np.asarray(x, np.float64), np.asarray(w, np.float64)
    k = x64.shape[-1]
    return np.matmul(x64, w64), (k + 2) * 2.0 ** -23 * np.matmul(np.abs(x64), np.abs(w64))


def embed(table: np.ndarray, idx: np.ndarray, addend=None) -> np.ndarray:
    """Reference _gather_ref, ops.py:482-487 (np.take on axis 0), then an optional f32 add."""
    out = np.take(np.asarray(table, np.float32), np.asarray(idx), axis=0)
    if addend is not None:
        out = (out + np.asarray(addend, np.float32)).astype(np.float32)
    return out
