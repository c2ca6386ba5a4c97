"""Per-kernel parity on the GPU: every kernel against the CPU oracle on identical seeded inputs.

int8 activations and int32 accumulators must be bit-exact; f32 results must be bit-identical to
the reference's NumPy arithmetic (tolerance 0) for the exact epilogue ops, and within 1e-5
relative for the transcendental ones (gelu/sigmoid/tanh use CUDA's tanhf/expf).
"""
import numpy as np
import pytest

from oracle import w8a8 as ref

pytestmark = pytest.mark.gpu


def _k():
    from mira_b200 import kernels as K
    from mira_b200.device import DeviceBuffer
    return K, DeviceBuffer


def _same_f32(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    bad = ~((got == want) | (np.isnan(got) & np.isnan(want)))
    assert not bad.any(), f"{bad.sum()} of {bad.size} f32 values differ; first at {np.argwhere(bad)[:3].tolist()}"


# ------------------------------------------------------------------------------ quantize

@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 17), (64, 784), (257, 1000), (1000, 16)])
def test_quantize_rows_matches_reference(cuda_device, rows, cols):
    K, DB = _k()
    rng = np.random.default_rng(rows * 7 + cols)
    scale = float(rng.uniform(0.01, 0.1))
    x = (rng.standard_normal((rows, cols)) * 60 * scale).astype(np.float32)
    # exact ties k + 0.5 in the quotient and values beyond the clip range
    x.ravel()[::7] = ((rng.integers(-140, 140, x.size)[::7] + 0.5) * np.float32(scale)).astype(np.float32)
    x.ravel()[::11] = np.float32(1e30)
    ldq = K.round_up(cols, 16)
    xb = DB.from_array(x)
    qb = DB(rows * ldq)
    K.quantize_rows(xb, rows, cols, cols, scale, qb, ldq)
    got = qb.download((rows, ldq), np.int8)
    np.testing.assert_array_equal(got[:, :cols], ref.quantize_activation(x, scale))
    assert not got[:, cols:].any()


def test_quantize_nchw_to_nhwc(cuda_device):
    K, DB = _k()
    rng = np.random.default_rng(5)
    n, c, h, w = 3, 3, 9, 11
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    scale = 0.0271
    cp = K.conv_channels(c)
    xb, qb = DB.from_array(x), DB(n * h * w * cp)
    K.quantize_nchw_to_nhwc(xb, n, c, h, w, scale, qb, cp)
    got = qb.download((n, h, w, cp), np.int8)
    want = ref.quantize_activation(x, scale).transpose(0, 2, 3, 1)
    np.testing.assert_array_equal(got[..., :c], want)
    assert not got[..., c:].any()


# ------------------------------------------------------------------------------ qgemm

def _run_qgemm(M, N, K_, steps_spec, seed, want_i8=True, rowcol=False, splitk=False):
    K, DB = _k()
    rng = np.random.default_rng(seed)
    x_scale = float(rng.uniform(0.005, 0.05))
    xq = rng.integers(-127, 128, (M, K_)).astype(np.int8)
    q = rng.integers(-127, 128, (K_, N)).astype(np.int8)
    w_scale = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    lda = K.round_up(K_, 16)
    A = np.zeros((M, lda), np.int8)
    A[:, :K_] = xq
    Ab, Bb = DB.from_array(A), DB.from_array(K.matmul_weight(q))
    acc = ref.int_matmul(xq, q)
    keep = []
    if rowcol:
        rs = rng.uniform(1e-3, 1e-2, M).astype(np.float32)
        cs = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
        rb, cb = DB.from_array(rs), DB.from_array(cs)
        keep += [rb, cb]
        dq = K.dequant_rowcol(rb, cb)
        y = (acc.astype(np.float64) * (rs.astype(np.float64)[:, None] * cs.astype(np.float64)[None, :])).astype(np.float32)
    else:
        s64, hi, lo = K.scale_arrays(x_scale, w_scale)
        sb, hb, lb = DB.from_array(s64), DB.from_array(hi), DB.from_array(lo)
        keep += [sb, hb, lb]
        dq = K.dequant_channel(sb, hb, lb)
        y = ref.dequant(acc, ref.combined_scale(x_scale, w_scale))
    steps, ref_steps, operands = [], [], []
    for kind in steps_spec:
        if kind == "bias":
            b = rng.standard_normal(N).astype(np.float32)
            bb = DB.from_array(K.pad_channels(b))
            keep.append(bb)
            steps.append(K.Step("add", "channel", ptr=bb))
            ref_steps.append(("add", len(operands), False))
            operands.append(b)
        elif kind == "residual":
            r = rng.standard_normal((M, N)).astype(np.float32)
            rb_ = DB.from_array(r)
            keep.append(rb_)
            steps.append(K.Step("add", "full", ptr=rb_, ld=N))
            ref_steps.append(("add", len(operands), True))
            steps[-1].swapped = True
            operands.append(r)
        elif kind == "scale":            # a per-channel multiply (an unfolded batch norm's scale)
            g = rng.uniform(0.5, 2.0, N).astype(np.float32)
            gb = DB.from_array(K.pad_channels(g))
            keep.append(gb)
            steps.append(K.Step("mul", "channel", ptr=gb))
            ref_steps.append(("mul", len(operands), False))
            operands.append(g)
        elif kind == "rsub":             # 0.25 - y
            steps.append(K.Step("sub", "scalar", scalar=0.25))
            steps[-1].swapped = True
            ref_steps.append(("sub", len(operands), True))
            operands.append(np.float32(0.25))
        elif kind in ("relu", "gelu", "tanh", "sigmoid"):
            steps.append(K.Step(kind))
            ref_steps.append((kind, None, False))
        elif kind == "relu6":
            steps += [K.Step("maximum", "scalar", scalar=0.0), K.Step("minimum", "scalar", scalar=6.0)]
            operands += [np.float32(0.0), np.float32(6.0)]
            ref_steps += [("maximum", len(operands) - 2, False), ("minimum", len(operands) - 1, False)]
    y = ref.epilogue(y, operands, ref_steps).astype(np.float32)
    out_scale = float(np.abs(y).max() / 127.0) or 1.0
    yb = DB(M * N * 4)
    ldi = K.round_up(N, 16)
    qb = DB(M * ldi) if want_i8 else None
    epi = K.Epi(steps, out_f32=yb, ld_f32=N, out_i8=qb, ld_i8=ldi, out_scale=out_scale)
    if splitk:
        nbytes = K.qgemm_workspace(M, N, K_)
        assert nbytes > 0, "shape expected to split"
        ws = DB(nbytes)
        K.qgemm_splitk(M, N, K_, Ab, lda, Bb, lda, dq, epi, ws, nbytes)
    else:
        K.qgemm(M, N, K_, Ab, lda, Bb, lda, dq, epi)
    got = yb.download((M, N), np.float32)
    got_q = qb.download((M, ldi), np.int8) if want_i8 else None
    return got, y, got_q, ref.quantize_activation(y, out_scale)


@pytest.mark.parametrize("M,N,K_", [(128, 64, 128), (1, 10, 16), (37, 100, 100), (256, 512, 784),
                                    (300, 300, 1000), (129, 256, 4096), (1024, 1000, 512)])
def test_qgemm_bias_relu_exact(cuda_device, M, N, K_):
    got, want, got_q, want_q = _run_qgemm(M, N, K_, ["bias", "relu"], seed=M + N + K_)
    _same_f32(got, want)
    np.testing.assert_array_equal(got_q[:, :N], want_q)
    assert not got_q[:, N:].any()


@pytest.mark.parametrize("M,N,K_,rowcol", [(4096, 4096, 4096, False), (4100, 3000, 3200, False),
                                           (2304, 2304, 4096, True), (8192, 2560, 3080, True)])
def test_qgemm_cta_pair_exact(cuda_device, M, N, K_, rowcol):
    """Long reductions with at least one 256 x 256 tile per SM pair run on CTA pairs (tcgen05.mma.cta_group::2):
    bit-exact like every GEMM, including ragged M (a last row tile whose odd CTA is all padding), N
    (a partial column half) and K."""
    spec = ["bias", "relu"] if rowcol else ["bias", "residual", "relu"]
    got, want, got_q, want_q = _run_qgemm(M, N, K_, spec, seed=M + N + K_, want_i8=not rowcol, rowcol=rowcol)
    _same_f32(got, want)
    if not rowcol:
        np.testing.assert_array_equal(got_q[:, :N], want_q)
        assert not got_q[:, N:].any()


@pytest.mark.parametrize("spec", [[], ["relu"], ["bias", "residual", "relu"], ["bias", "relu6"],
                                  ["scale", "bias", "relu"], ["scale", "rsub", "scale", "residual"]])
def test_qgemm_epilogues_exact(cuda_device, spec):
    """Each step rounded on its own; a mul step followed by add/sub must not fuse into one fma."""
    got, want, got_q, want_q = _run_qgemm(200, 192, 576, spec, seed=11)
    _same_f32(got, want)
    np.testing.assert_array_equal(got_q[:, :192], want_q)


@pytest.mark.parametrize("act", ["gelu", "tanh", "sigmoid"])
def test_qgemm_transcendental_epilogue_close(cuda_device, act):
    got, want, _, _ = _run_qgemm(130, 96, 256, ["bias", act], seed=3, want_i8=False)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("M,N,K_", [(256, 256, 256), (100, 130, 4096), (1, 4096, 4096), (16, 4096, 4096)])
def test_qgemm_rowcol_sweep_semantics(cuda_device, M, N, K_):
    got, want, _, _ = _run_qgemm(M, N, K_, ["bias"], seed=7, want_i8=False, rowcol=True)
    _same_f32(got, want)


@pytest.mark.parametrize("M,N,K_", [(1, 4096, 4096), (16, 4096, 4096), (128, 4096, 4096), (200, 300, 2048),
                                    (3, 10, 1024), (64, 768, 3072)])
@pytest.mark.parametrize("rowcol", [False, True])
def test_qgemm_splitk_exact(cuda_device, M, N, K_, rowcol):
    """Split-K (int32 partial sums per K range, added by a second kernel) gives the reference's
    result bit for bit, like the unsplit GEMM."""
    spec = ["bias", "relu"] if rowcol else ["bias", "residual", "relu"]
    got, want, got_q, want_q = _run_qgemm(M, N, K_, spec, seed=M + K_, rowcol=rowcol, splitk=True)
    _same_f32(got, want)
    np.testing.assert_array_equal(got_q[:, :N], want_q)
    assert not got_q[:, N:].any()


@pytest.mark.parametrize("M", [1, 16])
def test_qgemm_splitk_mul_step_exact(cuda_device, M):
    got, want, got_q, want_q = _run_qgemm(M, 4096, 4096, ["scale", "rsub", "bias"], seed=M, splitk=True)
    _same_f32(got, want)
    np.testing.assert_array_equal(got_q[:, :4096], want_q)


def test_qgemm_splitk_shapes_in_sequence(cuda_device):
    """Split-K shapes of different tile counts and splits one after another (a decode step's mix),
    each sharing nothing but the device: all bit-exact."""
    for M, N, K_ in [(64, 768, 768), (64, 3072, 768), (64, 768, 768), (16, 4096, 4096), (64, 768, 3072),
                     (64, 3072, 768)]:
        got, want, got_q, want_q = _run_qgemm(M, N, K_, ["bias", "residual"], seed=N + K_, splitk=True)
        _same_f32(got, want)
        np.testing.assert_array_equal(got_q[:, :N], want_q)


def test_qgemm_splitk_workspace_rule(cuda_device):
    K, _ = _k()
    assert K.qgemm_workspace(65536, 768, 3072) == 0          # enough output tiles
    assert K.qgemm_workspace(300, 4096, 512) == 0            # taller shapes: reduction too short to split
    assert K.qgemm_workspace(1, 4096, 4096) > 0
    # one row tile (a decode step's projections): 64-column tiles, K split down to one K-block
    assert K.qgemm_workspace(64, 768, 768) == 6 * 64 * 768 * 4


# ------------------------------------------------------------------------------ qconv2d

def _run_qconv(n, c, h, w, o, kh, kw, stride, pad, dil=(1, 1), spec=("bias", "relu"), seed=0):
    K, DB = _k()
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    x_scale = float(np.abs(x).max() / 127.0)
    wt = (rng.standard_normal((o, c, kh, kw)) / np.sqrt(c * kh * kw)).astype(np.float32)
    q, w_scale = ref.quantize_array(wt, 0)
    bias = rng.standard_normal((o, 1, 1)).astype(np.float32)
    ref_steps, operands, steps, keep = [], [], [], []
    if "bias" in spec:
        bb = DB.from_array(K.pad_channels(bias))
        keep.append(bb)
        steps.append(K.Step("add", "channel", ptr=bb))
        ref_steps.append(("add", 1, False))
        operands.append(bias)
    if "relu" in spec:
        steps.append(K.Step("relu"))
        ref_steps.append(("relu", None, False))
    xq, acc, y = ref.qconv2d(x, q, w_scale, x_scale, stride, pad, dil, steps=ref_steps, operands=operands)
    wq, cp = K.conv_weight(q)
    xn = np.zeros((n, h, w, cp), np.int8)
    xn[..., :c] = xq.transpose(0, 2, 3, 1)
    oh, ow = y.shape[2:]
    M = n * oh * ow
    s64, hi, lo = K.scale_arrays(x_scale, w_scale)
    sb, hb, lb = DB.from_array(s64), DB.from_array(hi), DB.from_array(lo)
    xb, wb = DB.from_array(xn), DB.from_array(wq)
    yb = DB(M * o * 4)
    ldi = K.round_up(o, 16)
    qb = DB(M * ldi)
    out_scale = float(np.abs(y).max() / 127.0) or 1.0
    K.qconv2d(n, h, w, cp, xb, o, kh, kw, wb, wq.shape[1], stride, pad, dil, K.dequant_channel(sb, hb, lb),
              K.Epi(steps, out_f32=yb, ld_f32=o, out_i8=qb, ld_i8=ldi, out_scale=out_scale))
    got = yb.download((n, oh, ow, o), np.float32).transpose(0, 3, 1, 2)
    got_q = qb.download((n, oh, ow, ldi), np.int8)[..., :o].transpose(0, 3, 1, 2)
    return got, y, got_q, ref.quantize_activation(y, out_scale)


@pytest.mark.parametrize("case", [
    dict(n=2, c=64, h=14, w=14, o=64, kh=3, kw=3, stride=(1, 1), pad=(1, 1)),
    dict(n=2, c=64, h=15, w=13, o=128, kh=3, kw=3, stride=(2, 2), pad=(1, 1)),
    dict(n=3, c=128, h=8, w=8, o=256, kh=1, kw=1, stride=(2, 2), pad=(0, 0)),
    dict(n=2, c=3, h=32, w=32, o=64, kh=7, kw=7, stride=(2, 2), pad=(3, 3)),
    dict(n=1, c=1, h=28, w=28, o=16, kh=3, kw=3, stride=(1, 1), pad=(1, 1)),
    dict(n=2, c=16, h=14, w=14, o=32, kh=3, kw=3, stride=(1, 1), pad=(1, 1)),
    dict(n=1, c=256, h=7, w=7, o=512, kh=3, kw=3, stride=(1, 1), pad=(1, 1)),
    dict(n=2, c=32, h=10, w=10, o=48, kh=3, kw=3, stride=(1, 1), pad=(2, 2), dil=(2, 2)),
    dict(n=2, c=40, h=9, w=9, o=24, kh=1, kw=1, stride=(1, 1), pad=(0, 0)),
    # TMA im2col path (channels a multiple of 64, square kernels, symmetric padding)
    dict(n=2, c=64, h=12, w=12, o=64, kh=3, kw=3, stride=(1, 1), pad=(2, 2), dil=(2, 2)),
    dict(n=2, c=192, h=9, w=9, o=96, kh=3, kw=3, stride=(1, 1), pad=(1, 1)),
    dict(n=3, c=128, h=11, w=11, o=64, kh=5, kw=5, stride=(2, 2), pad=(2, 2)),
    dict(n=5, c=64, h=9, w=7, o=128, kh=1, kw=1, stride=(1, 1), pad=(0, 0)),
    dict(n=4, c=320, h=7, w=7, o=1280, kh=1, kw=1, stride=(1, 1), pad=(0, 0)),   # 1x1 as a 2-D TMA GEMM
    dict(n=2, c=512, h=7, w=7, o=256, kh=3, kw=3, stride=(2, 2), pad=(1, 1)),
    dict(n=4, c=64, h=20, w=20, o=32, kh=3, kw=3, stride=(1, 1), pad=(0, 0)),
    # non-square kernel with 64 channels: the cp.async gather
    dict(n=2, c=64, h=10, w=10, o=64, kh=1, kw=3, stride=(1, 1), pad=(0, 1)),
])
def test_qconv2d_exact(cuda_device, case):
    got, want, got_q, want_q = _run_qconv(**case, seed=sum(v if isinstance(v, int) else 0 for v in case.values()))
    _same_f32(got, want)
    np.testing.assert_array_equal(got_q, want_q)


# ------------------------------------------------------------------------------ memory-bound ops

def test_maxpool_f32_and_int8(cuda_device):
    K, DB = _k()
    rng = np.random.default_rng(2)
    n, c, h, w = 2, 64, 15, 15
    x = np.maximum(rng.standard_normal((n, c, h, w)), 0).astype(np.float32)
    scale = float(np.abs(x).max() / 127)
    want = ref.maxpool2d(x, 3, 2, 1)
    xn = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    oh = want.shape[2]
    xb = DB.from_array(xn)
    yb, qb = DB(n * oh * oh * c * 4), DB(n * oh * oh * c)
    K.maxpool2d(n, h, w, c, c, 3, 2, 1, -np.inf, x_f32=xb, out_f32=yb, ldc_out_f32=c, out_i8=qb, ldc_out_i8=c,
                out_scale=scale)
    _same_f32(yb.download((n, oh, oh, c), np.float32).transpose(0, 3, 1, 2), want)
    np.testing.assert_array_equal(qb.download((n, oh, oh, c), np.int8).transpose(0, 3, 1, 2),
                                  ref.quantize_activation(want, scale))
    # int8 path: pooling int8 equals quantizing the pooled f32 values
    xq = DB.from_array(ref.quantize_activation(xn, scale))
    q2 = DB(n * oh * oh * c)
    K.maxpool2d(n, h, w, c, c, 3, 2, 1, -np.inf, x_i8=xq, out_i8=q2, ldc_out_i8=c, out_scale=scale)
    np.testing.assert_array_equal(q2.download((n, oh, oh, c), np.int8).transpose(0, 3, 1, 2),
                                  ref.quantize_activation(want, scale))


@pytest.mark.parametrize("hw", [(7, 7), (1, 1), (14, 14), (3, 5)])
def test_mean_hw_bit_exact(cuda_device, hw):
    K, DB = _k()
    rng = np.random.default_rng(hw[0] * 10 + hw[1])
    n, c = 5, 96
    x = (rng.standard_normal((n, c) + hw) * 3).astype(np.float32)
    want = x.mean(axis=(2, 3))
    xb = DB.from_array(np.ascontiguousarray(x.transpose(0, 2, 3, 1)))
    yb, qb = DB(n * c * 4), DB(n * 112)
    scale = float(np.abs(want).max() / 127)
    K.mean_hw(xb, n, hw[0] * hw[1], c, c, out_f32=yb, out_i8=qb, ld_i8=112, out_scale=scale)
    _same_f32(yb.download((n, c), np.float32), want)
    np.testing.assert_array_equal(qb.download((n, 112), np.int8)[:, :c], ref.quantize_activation(want, scale))


@pytest.mark.parametrize("stride,c,inf_weight", [(1, 96, False), (2, 96, False), (1, 30, False), (2, 960, False),
                                                (1, 96, True), (1, 30, True)])
def test_dwconv_bit_exact(cuda_device, stride, c, inf_weight):
    """Four-channel vector kernel (c % 4 == 0, c / 4 above one warp for 960) and the scalar kernel
    (c = 30), with f32 and int8 outputs.  An inf weight makes every output that reads a padded tap
    through it NaN in the zero-padded reference (0 * inf), and the kernels must agree."""
    K, DB = _k()
    rng = np.random.default_rng(stride + c)
    n, h, w = 2, 13, 13
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = rng.standard_normal((c, 1, 3, 3)).astype(np.float32)
    if inf_weight:
        wt[3, 0, 0, 0] = np.inf
        wt[5, 0, 2, 1] = -np.inf
    bias = rng.standard_normal((c, 1, 1)).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        want = ref.dwconv2d(x, wt, (stride, stride), (1, 1), steps=[("add", 2, False), ("maximum", 3, False),
                                                                     ("minimum", 4, False)],
                            operands=[bias, np.float32(0), np.float32(6)])
    if inf_weight:
        assert np.isnan(want).any()
    oh = want.shape[2]
    xb = DB.from_array(np.ascontiguousarray(x.transpose(0, 2, 3, 1)))
    wb = DB.from_array(np.ascontiguousarray(wt[:, 0].reshape(c, 9).T))
    bb = DB.from_array(K.pad_channels(bias))
    yb = DB(n * oh * oh * c * 4)
    ldq = K.round_up(c, 16)
    qb = DB(n * oh * oh * ldq, zero=True)
    scale = 6.0 / 127
    K.dwconv2d(xb, n, h, w, c, wb, 3, 3, (stride, stride), (1, 1), (1, 1),
               K.Epi([K.Step("add", "channel", ptr=bb), K.Step("maximum", "scalar", scalar=0.0),
                      K.Step("minimum", "scalar", scalar=6.0)], out_f32=yb, ld_f32=c, out_i8=qb, ld_i8=ldq,
                     out_scale=scale))
    got = yb.download((n, oh, oh, c), np.float32).transpose(0, 3, 1, 2)
    _same_f32(got, want)
    if not inf_weight:
        q = qb.download((n, oh, oh, ldq), np.int8)[..., :c].transpose(0, 3, 1, 2)
        np.testing.assert_array_equal(q, ref.quantize_activation(want, scale))


@pytest.mark.parametrize("n,c,h,w,k,stride,pad,dil", [
    (2, 64, 11, 9, 5, 1, 2, 1),      # 5x5: the general 4-channel kernel
    (2, 32, 12, 12, 3, 1, 2, 2),     # dilated 3x3: the general 4-channel kernel
    (2, 36, 9, 10, 3, 2, 0, 1),      # unpadded, ragged output width
    (600, 8, 112, 5, 3, 1, 1, 1),    # 67200 output rows: more than one grid row per block
    (1, 1024, 3, 3, 3, 1, 1, 1),     # channels beyond one block's 256 threads
])
def test_dwconv_geometries_bit_exact(cuda_device, n, c, h, w, k, stride, pad, dil):
    K, DB = _k()
    rng = np.random.default_rng(n + c + k)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = rng.standard_normal((c, 1, k, k)).astype(np.float32)
    want = ref.dwconv2d(x, wt, (stride, stride), (pad, pad), (dil, dil))
    oh, ow = want.shape[2:]
    xb = DB.from_array(np.ascontiguousarray(x.transpose(0, 2, 3, 1)))
    wb = DB.from_array(np.ascontiguousarray(wt[:, 0].reshape(c, k * k).T))
    yb = DB(n * oh * ow * c * 4)
    K.dwconv2d(xb, n, h, w, c, wb, k, k, (stride, stride), (pad, pad), (dil, dil), K.Epi([], out_f32=yb, ld_f32=c))
    _same_f32(yb.download((n, oh, ow, c), np.float32).transpose(0, 3, 1, 2), want)


@pytest.mark.parametrize("n,c,h,w,k,stride,pad,dil,epi", [
    (2, 32, 13, 11, 3, 1, 1, 1, "bias_relu6"),     # 3x3 stride 1: 4 columns per thread
    (2, 96, 14, 14, 3, 2, 1, 1, "bias_relu6"),     # 3x3 stride 2: 2 columns per thread
    (1, 960, 7, 7, 3, 1, 1, 1, "bias_relu6"),      # c / 4 above one block of threads
    (3, 144, 9, 17, 3, 2, 1, 1, "bias"),           # odd widths: partial column groups
    (2, 16, 11, 9, 5, 1, 2, 1, "bias_relu6"),      # 5x5: the general kernel
    (1, 8, 10, 10, 3, 1, 2, 2, "none"),            # dilated
    (2, 12, 7, 9, 3, 2, 0, 1, "bias_relu6"),       # no padding, stride 2, general kernel (c not 16k)
])
def test_qdwconv_bit_exact(cuda_device, n, c, h, w, k, stride, pad, dil, epi):
    """The opt-in int8 depthwise conv against the oracle's restatement of the reference's grouped
    qconv2d (itself pinned to the reference's outputs): f32 and int8 outputs bit for bit."""
    K, DB = _k()
    rng = np.random.default_rng(n * 1000 + c + k)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    q, ws = ref.quantize_array(rng.standard_normal((c, 1, k, k)).astype(np.float32), 0)
    x_scale = float(np.abs(x).max() / 127.0)
    bias = rng.standard_normal((c, 1, 1)).astype(np.float32)
    if epi == "bias_relu6":
        steps, operands = [("add", 1, False), ("maximum", 2, False), ("minimum", 3, False)], [bias, np.float32(0),
                                                                                               np.float32(6)]
        ksteps = [K.Step("add", "channel", ptr=DB.from_array(K.pad_channels(bias))),
                  K.Step("maximum", "scalar", scalar=0.0), K.Step("minimum", "scalar", scalar=6.0)]
    elif epi == "bias":
        steps, operands = [("add", 1, False)], [bias]
        ksteps = [K.Step("add", "channel", ptr=DB.from_array(K.pad_channels(bias)))]
    else:
        steps, operands, ksteps = [], [], []
    xq, acc, want = ref.qdwconv2d(x, q, ws, x_scale, (stride, stride), (pad, pad), (dil, dil), steps, operands)
    oh, ow = want.shape[2:]
    ldx = K.round_up(c, 16)
    xh = np.zeros((n, h, w, ldx), np.int8)
    xh[..., :c] = xq.transpose(0, 2, 3, 1)
    xb = DB.from_array(xh)
    wb = DB.from_array(np.ascontiguousarray(q[:, 0].reshape(c, k * k).T))
    keep = [DB.from_array(a) for a in K.scale_arrays(x_scale, ws)]
    yb = DB(n * oh * ow * c * 4)
    qb = DB(n * oh * ow * ldx, zero=True)
    out_scale = float(np.abs(want).max() / 127.0) or 1.0
    K.qdwconv2d(xb, ldx, n, h, w, c, wb, k, k, (stride, stride), (pad, pad), (dil, dil), K.dequant_channel(*keep),
                K.Epi(ksteps, out_f32=yb, ld_f32=c, out_i8=qb, ld_i8=ldx, out_scale=out_scale))
    got = yb.download((n, oh, ow, c), np.float32).transpose(0, 3, 1, 2)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    qgot = qb.download((n, oh, ow, ldx), np.int8)
    np.testing.assert_array_equal(qgot[..., :c].transpose(0, 3, 1, 2), ref.quantize_activation(want, out_scale))
    assert not qgot[..., c:].any()


def test_layout_roundtrip(cuda_device):
    K, DB = _k()
    x = np.random.default_rng(0).standard_normal((3, 70, 9, 13)).astype(np.float32)
    xb, yb, zb = DB.from_array(x), DB(x.nbytes), DB(x.nbytes)
    K.nchw_to_nhwc(xb, 3, 70, 9, 13, yb, 70)
    np.testing.assert_array_equal(yb.download((3, 9, 13, 70), np.float32), x.transpose(0, 2, 3, 1))
    K.nhwc_to_nchw(yb, 3, 9, 13, 70, 70, zb)
    np.testing.assert_array_equal(zb.download(x.shape, np.float32), x)


# ------------------------------------------------------------------------------ fused conv + max pool

@pytest.mark.parametrize("case", [
    dict(n=2, c=3, h=40, w=36, o=64, k=7, s=2, p=3, ps=3, pst=2, pp=1),     # ResNet stem + its pool
    dict(n=3, c=1, h=28, w=28, o=16, k=3, s=1, p=1, ps=2, pst=2, pp=0),     # small CNN block
    dict(n=2, c=16, h=14, w=14, o=32, k=3, s=1, p=1, ps=2, pst=2, pp=0),
    dict(n=1, c=32, h=17, w=15, o=48, k=3, s=1, p=1, ps=3, pst=2, pp=1),
])
def test_qconv2d_maxpool_fused_exact(cuda_device, case):
    K, DB = _k()
    n, c, h, w, o, k = case["n"], case["c"], case["h"], case["w"], case["o"], case["k"]
    rng = np.random.default_rng(n * 100 + c + o)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    x_scale = float(np.abs(x).max() / 127.0)
    q, w_scale = ref.quantize_array(rng.standard_normal((o, c, k, k)).astype(np.float32), 0)
    bias = rng.standard_normal((o, 1, 1)).astype(np.float32)
    xq, _, y = ref.qconv2d(x, q, w_scale, x_scale, (case["s"],) * 2, (case["p"],) * 2,
                           steps=[("add", 1, False), ("relu", None, False)], operands=[bias])
    want = ref.maxpool2d(y, case["ps"], case["pst"], case["pp"], -np.inf)
    wq, cp = K.conv_weight(q)
    xn = np.zeros((n, h, w, cp), np.int8)
    xn[..., :c] = xq.transpose(0, 2, 3, 1)
    s64, hi, lo = K.scale_arrays(x_scale, w_scale)
    bufs = [DB.from_array(a) for a in (xn, wq, s64, hi, lo, K.pad_channels(bias))]
    ph, pw = want.shape[2:]
    ldi = K.round_up(o, 16)
    yb, qb = DB(n * ph * pw * o * 4), DB(n * ph * pw * ldi)
    out_scale = float(np.abs(want).max() / 127.0)
    K.qconv2d_maxpool(n, h, w, cp, bufs[0], o, k, k, bufs[1], wq.shape[1], (case["s"],) * 2, (case["p"],) * 2,
                      (1, 1), case["ps"], case["pst"], case["pp"], -np.inf, K.dequant_channel(*bufs[2:5]),
                      K.Epi([K.Step("add", "channel", ptr=bufs[5]), K.Step("relu")], out_f32=yb, ld_f32=o,
                            out_i8=qb, ld_i8=ldi, out_scale=out_scale))
    _same_f32(yb.download((n, ph, pw, o), np.float32).transpose(0, 3, 1, 2), want)
    got_q = qb.download((n, ph, pw, ldi), np.int8)
    np.testing.assert_array_equal(got_q[..., :o].transpose(0, 3, 1, 2), ref.quantize_activation(want, out_scale))
    assert not got_q[..., o:].any()


# ------------------------------------------------------------------------------ row-expanded inputs

@pytest.mark.parametrize("case", [
    dict(n=2, c=3, h=40, w=36, o=64, k=7, s=2, p=3),     # ResNet stem
    dict(n=2, c=3, h=33, w=31, o=32, k=3, s=2, p=1),     # MobileNetV2 stem
    dict(n=3, c=1, h=28, w=28, o=16, k=3, s=1, p=1),
    dict(n=1, c=4, h=9, w=13, o=24, k=5, s=1, p=0),
    dict(n=2, c=3, h=21, w=30, o=16, k=3, s=4, p=1),     # entries laid out at stride 4
])
@pytest.mark.parametrize("pool", [False, True])
def test_row4_layout_conv_exact(cuda_device, case, pool):
    K, DB = _k()
    n, c, h, w, o, k, s, p = (case[key] for key in ("n", "c", "h", "w", "o", "k", "s", "p"))
    rng = np.random.default_rng(n + c * 10 + o)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    x_scale = float(np.abs(x).max() / 127.0)
    q, w_scale = ref.quantize_array(rng.standard_normal((o, c, k, k)).astype(np.float32), 0)
    bias = rng.standard_normal((o, 1, 1)).astype(np.float32)
    _, _, y = ref.qconv2d(x, q, w_scale, x_scale, (s, s), (p, p), steps=[("add", 1, False), ("relu", None, False)],
                          operands=[bias])
    if pool:
        y = ref.maxpool2d(y, 3, 2, 1, -np.inf)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    entries = K.row4_entries(ow, s)
    xb, xq = DB.from_array(x), DB(n * h * entries * 16)
    K.quantize_nchw_to_row4(xb, n, c, h, w, x_scale, xq, entries, p, s)
    wq = K.conv_weight_row4(q)
    s64, hi, lo = K.scale_arrays(x_scale, w_scale)
    bufs = [DB.from_array(a) for a in (wq, s64, hi, lo, K.pad_channels(bias))]
    ph, pw_ = y.shape[2:]
    ldi = K.round_up(o, 16)
    yb, qb = DB(n * ph * pw_ * o * 4), DB(n * ph * pw_ * ldi)
    out_scale = float(np.abs(y).max() / 127.0)
    epi = K.Epi([K.Step("add", "channel", ptr=bufs[4]), K.Step("relu")], out_f32=yb, ld_f32=o, out_i8=qb, ld_i8=ldi,
                out_scale=out_scale)
    if pool:
        K.qconv2d_maxpool(n, h, w, 4, xq, o, k, k, bufs[0], wq.shape[1], (s, s), (p, p), (1, 1), 3, 2, 1, -np.inf,
                          K.dequant_channel(*bufs[1:4]), epi, layout=1, row_entries=entries)
    else:
        K.qconv2d(n, h, w, 4, xq, o, k, k, bufs[0], wq.shape[1], (s, s), (p, p), (1, 1), K.dequant_channel(*bufs[1:4]),
                  epi, layout=1, row_entries=entries)
    _same_f32(yb.download((n, ph, pw_, o), np.float32).transpose(0, 3, 1, 2), y)
    np.testing.assert_array_equal(qb.download((n, ph, pw_, ldi), np.int8)[..., :o].transpose(0, 3, 1, 2),
                                  ref.quantize_activation(y, out_scale))


@pytest.mark.parametrize("n,c,h,w,o,k,stride,pad,dil", [(2, 3, 17, 15, 16, 3, 1, 1, 1), (1, 64, 14, 14, 32, 3, 2, 1, 1),
                                                       (2, 5, 12, 12, 7, 5, 1, 4, 2), (3, 16, 9, 9, 24, 1, 1, 0, 1)])
def test_f32_conv_im2col_within_error_bound(cuda_device, n, c, h, w, o, k, stride, pad, dil):
    """General f32 convolution = patch matrix (im2col) times [k*k*c, o] weights in the f32 matmul:
    within the f32 error bound of the exact (float64) convolution, bias added in the epilogue."""
    K, DB = _k()
    rng = np.random.default_rng(n + c + k)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = rng.standard_normal((o, c, k, k)).astype(np.float32)
    bias = rng.standard_normal(o).astype(np.float32)
    oh = (h + 2 * pad - dil * (k - 1) - 1) // stride + 1
    ow = (w + 2 * pad - dil * (k - 1) - 1) // stride + 1
    rows, kdim = n * oh * ow, k * k * c
    xb = DB.from_array(np.ascontiguousarray(x.transpose(0, 2, 3, 1)))
    pb = DB(rows * kdim * 4)
    K.im2col_f32(xb, n, h, w, c, c, k, k, (stride, stride), (pad, pad), (dil, dil), pb, kdim)
    patches = pb.download((rows, kdim), np.float32)
    xp = np.pad(x.transpose(0, 2, 3, 1), ((0, 0), (pad, pad), (pad, pad), (0, 0)))
    want_p = np.concatenate([xp[:, i * dil:i * dil + stride * (oh - 1) + 1:stride, j * dil:j * dil + stride * (ow - 1) + 1:stride]
                             for i in range(k) for j in range(k)], axis=-1).reshape(rows, kdim)
    np.testing.assert_array_equal(patches, want_p)
    bmat = np.ascontiguousarray(wt.transpose(2, 3, 1, 0).reshape(kdim, o))
    bb, biasb, yb = DB.from_array(bmat), DB.from_array(bias), DB(rows * o * 4)
    K.bmm_f32(1, 1, rows, o, kdim, K.View(pb, (0, 0, kdim, 1)), K.View(bb, (0, 0, o, 1)),
              K.BmmEpi([K.BmmStep("add", "view", view=K.View(biasb, (0, 0, 0, 1)))], out=K.View(yb, (0, 0, o, 1))))
    got = yb.download((rows, o), np.float32)
    exact = want_p.astype(np.float64) @ bmat.astype(np.float64) + bias.astype(np.float64)
    bound = (np.abs(want_p).astype(np.float64) @ np.abs(bmat).astype(np.float64) + np.abs(bias)) * (kdim + 2) * 2.0 ** -24
    assert np.all(np.abs(got - exact) <= bound + 1e-30)


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "maximum", "minimum", "relu", "gelu", "sigmoid", "tanh"])
def test_elementwise_f32(cuda_device, op):
    """Standalone element-wise op over a transposed view with a broadcast operand: IEEE binary ops
    and relu bit for bit against NumPy, the transcendental ones within f32 tolerance."""
    K, DB = _k()
    rng = np.random.default_rng(len(op))
    a = (rng.standard_normal((2, 3, 7, 40)) * 3).astype(np.float32)
    b = rng.standard_normal((1, 3, 1, 40)).astype(np.float32)
    a_t = np.ascontiguousarray(a.transpose(0, 1, 3, 2))          # stored [.., 40, 7], read as [.., 7, 40]
    ab, bb, ob = DB.from_array(a_t), DB.from_array(b), DB(a.nbytes)
    av = K.View(ab, (3 * 40 * 7, 40 * 7, 1, 7))
    out = K.View(ob, (3 * 7 * 40, 7 * 40, 40, 1))
    unary = op in ("relu", "gelu", "sigmoid", "tanh")
    K.elementwise_f32(op, a.shape, av, out, b=None if unary else K.View(bb, (0, 40, 0, 1)))
    got = ob.download(a.shape, np.float32)
    want = (ref.UNARY[op](a) if unary else ref.BINARY[op](a, b)).astype(np.float32)
    if op in ("gelu", "sigmoid", "tanh"):
        # CUDA's tanhf/expf against NumPy's: relative near 1, absolute where GELU tends to 0
        np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-6)
    else:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # a scalar on the left: 0.75 op a
    if not unary:
        K.elementwise_f32(op, a.shape, av, out, scalar=0.75, swapped=True)
        want = ref.BINARY[op](np.float32(0.75), a).astype(np.float32)
        assert np.array_equal(ob.download(a.shape, np.float32).view(np.uint32), want.view(np.uint32))


def test_qgemm_config2_8192_cubed_exact(cuda_device):
    """The GEMM sweep's headline shape exactly as bench.py times it: M = N = K = 8192 on config-2
    operands (A, B uniform int8 in [-127, 127], row and column scales U(1e-3, 1e-2), bias N(0, 1)),
    which takes the CTA-pair kernel; every output against the oracle's exact restatement
    (float64 sums of int8 products are exact here)."""
    from mira_b200 import _lib
    K, DB = _k()
    n = 8192
    rng = np.random.default_rng(1000 + n)
    a = rng.integers(-127, 128, (n, n), dtype=np.int8)
    b = rng.integers(-127, 128, (n, n), dtype=np.int8)          # K-major: row j holds column j of B
    rs = rng.uniform(1e-3, 1e-2, n).astype(np.float32)
    cs = rng.uniform(1e-3, 1e-2, n).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    Ab, Bb, rb, cb = DB.from_array(a), DB.from_array(b), DB.from_array(rs), DB.from_array(cs)
    biasb, yb = DB.from_array(K.pad_channels(bias)), DB(n * n * 4)
    n0 = _lib.launch_count()
    K.qgemm(n, n, n, Ab, n, Bb, n, K.dequant_rowcol(rb, cb),
            K.Epi([K.Step("add", "channel", ptr=biasb)], out_f32=yb, ld_f32=n))
    assert _lib.launch_count() - n0 == 1
    got = yb.download((n, n), np.float32)
    _, want = ref.qgemm_rowcol(a, b.T, rs, cs, bias)
    _same_f32(got, want)


# ------------------------------------------------------------------------------ chunk-planar convs

def _run_qconv_cp(n, c, h, w, o, seed, out_layout, residual=False, out_f32=True):
    """A 3x3 stride-1 pad-1 conv reading the chunk-planar layout (MIRA_LAYOUT_CP): every output
    against the oracle, int8 output in the chunk-planar or NHWC layout."""
    from mira_b200 import _lib
    K, DB = _k()
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    x_scale = float(np.abs(x).max() / 127.0)
    wt = (rng.standard_normal((o, c, 3, 3)) / np.sqrt(c * 9)).astype(np.float32)
    q, w_scale = ref.quantize_array(wt, 0)
    bias = rng.standard_normal((o, 1, 1)).astype(np.float32)
    res = rng.standard_normal((n, o, h, w)).astype(np.float32)
    steps_ref, operands = [("add", 1, False)], [bias]
    if residual:
        steps_ref.append(("add", 2, False))
        operands.append(res)
    steps_ref.append(("relu", None, False))
    xq, acc, y = ref.qconv2d(x, q, w_scale, x_scale, (1, 1), (1, 1), steps=steps_ref, operands=operands)
    wq, cp = K.conv_weight(q, K.round_up(c, 64))    # the layout's convs read 64k channels
    xn = np.zeros((n, h, w, cp), np.int8)
    xn[..., :c] = xq.transpose(0, 2, 3, 1)
    xb = DB.from_array(K.to_cp(xn))
    assert xb.nbytes == _lib.load().mira_cuda_cp_bytes(n, h, w, cp)
    s64, hi, lo = K.scale_arrays(x_scale, w_scale)
    keep = [DB.from_array(a) for a in (s64, hi, lo)]
    bb = DB.from_array(K.pad_channels(bias))
    steps = [K.Step("add", "channel", ptr=bb)]
    if residual:
        rb = DB.from_array(np.ascontiguousarray(res.transpose(0, 2, 3, 1)))
        steps.append(K.Step("add", "full", ptr=rb, ld=o))
    steps.append(K.Step("relu"))
    ldi = K.round_up(o, 16)
    M = n * h * w
    yb = DB(M * o * 4) if out_f32 else None
    cp_out = out_layout == "cp"
    qb = DB(K.cp_bytes(n, h, w, ldi) if cp_out else M * ldi, zero=True)
    out_scale = float(np.abs(y).max() / 127.0) or 1.0
    wb = DB.from_array(wq)
    K.qconv2d(n, h, w, cp, xb, o, 3, 3, wb, wq.shape[1], (1, 1), (1, 1), (1, 1), K.dequant_channel(*keep),
              K.Epi(steps, out_f32=yb, ld_f32=o, out_i8=qb, ld_i8=ldi, out_scale=out_scale,
                    i8_layout=_lib.LAYOUT_CP if cp_out else _lib.LAYOUT_NHWC),
              layout=_lib.LAYOUT_CP)
    if out_f32:
        _same_f32(yb.download((n, h, w, o), np.float32).transpose(0, 3, 1, 2), y)
    raw = qb.download((qb.nbytes,), np.int8)
    got_q = K.from_cp(raw, n, h, w, ldi) if cp_out else raw.reshape(n, h, w, ldi)
    np.testing.assert_array_equal(got_q[..., :o].transpose(0, 3, 1, 2), ref.quantize_activation(y, out_scale))
    assert not got_q[..., o:].any()
    if cp_out:   # the padding ring and the guards stay zero
        assert np.array_equal(K.to_cp(got_q), raw)


@pytest.mark.parametrize("case", [
    dict(n=2, c=64, h=56, w=56, o=64),          # ResNet layer 1 (resident weights)
    dict(n=3, c=64, h=9, w=13, o=64),           # tiles spanning several images
    dict(n=1, c=64, h=5, w=5, o=100),           # partial column tile
    dict(n=2, c=64, h=20, w=20, o=256),
    dict(n=2, c=128, h=28, w=28, o=128),        # layer 2
    dict(n=2, c=128, h=11, w=7, o=64),
    dict(n=2, c=128, h=6, w=6, o=256),
    dict(n=3, c=256, h=14, w=14, o=256),        # layer 3
    dict(n=2, c=256, h=9, w=9, o=128),
    dict(n=4, c=512, h=7, w=7, o=512),          # layer 4
    dict(n=1, c=48, h=8, w=8, o=32),            # 64 padded channels
])
@pytest.mark.parametrize("out_layout", ["cp", "nhwc"])
def test_qconv2d_chunk_planar_exact(cuda_device, case, out_layout):
    _run_qconv_cp(**case, seed=case["h"] * 7 + case["o"], out_layout=out_layout)


@pytest.mark.parametrize("case", [dict(n=2, c=64, h=56, w=56, o=64), dict(n=3, c=128, h=28, w=28, o=128),
                                  dict(n=2, c=512, h=7, w=7, o=512)])
def test_qconv2d_chunk_planar_residual_exact(cuda_device, case):
    """The block's second conv: bias + residual (full f32 operand read per pixel) + relu, f32 and int8 out."""
    _run_qconv_cp(**case, seed=5, out_layout="cp", residual=True)


def test_qconv2d_chunk_planar_int8_only(cuda_device):
    _run_qconv_cp(2, 64, 56, 56, 64, seed=9, out_layout="cp", out_f32=False)


def test_qconv2d_nhwc_input_chunk_planar_output(cuda_device):
    """A stride-2 im2col conv writing its int8 output in the chunk-planar layout (the next layer's
    3x3 convs read it)."""
    from mira_b200 import _lib
    K, DB = _k()
    rng = np.random.default_rng(3)
    n, c, h, w, o = 2, 64, 15, 13, 128
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    x_scale = float(np.abs(x).max() / 127.0)
    q, w_scale = ref.quantize_array(rng.standard_normal((o, c, 3, 3)).astype(np.float32), 0)
    xq, _, y = ref.qconv2d(x, q, w_scale, x_scale, (2, 2), (1, 1), steps=[("relu", None, False)])
    wq, cp = K.conv_weight(q)
    xb = DB.from_array(np.ascontiguousarray(xq.transpose(0, 2, 3, 1)))
    keep = [DB.from_array(a) for a in K.scale_arrays(x_scale, w_scale)]
    oh, ow = y.shape[2:]
    qb = DB(K.cp_bytes(n, oh, ow, o), zero=True)
    out_scale = float(np.abs(y).max() / 127.0)
    K.qconv2d(n, h, w, cp, xb, o, 3, 3, DB.from_array(wq), wq.shape[1], (2, 2), (1, 1), (1, 1),
              K.dequant_channel(*keep), K.Epi([K.Step("relu")], out_i8=qb, ld_i8=o, out_scale=out_scale,
                                             i8_layout=_lib.LAYOUT_CP))
    got = K.from_cp(qb.download((qb.nbytes,), np.int8), n, oh, ow, o)
    np.testing.assert_array_equal(got.transpose(0, 3, 1, 2), ref.quantize_activation(y, out_scale))


def test_maxpool_chunk_planar_int8_output(cuda_device):
    """ResNet's stem pool writing the first block's int8 input in the chunk-planar layout."""
    from mira_b200 import _lib
    K, DB = _k()
    rng = np.random.default_rng(4)
    for n, c, h, w in ((2, 64, 15, 15), (3, 48, 9, 12)):
        x = np.maximum(rng.standard_normal((n, c, h, w)), 0).astype(np.float32)
        scale = float(np.abs(x).max() / 127)
        want = ref.maxpool2d(x, 3, 2, 1)
        oh, ow = want.shape[2:]
        cp = K.round_up(c, 16)
        xb = DB.from_array(np.ascontiguousarray(x.transpose(0, 2, 3, 1)))
        qb = DB(K.cp_bytes(n, oh, ow, cp), zero=True)
        K.maxpool2d(n, h, w, c, c, 3, 2, 1, -np.inf, x_f32=xb, out_i8=qb, ldc_out_i8=cp, out_scale=scale,
                    i8_layout=_lib.LAYOUT_CP)
        got = K.from_cp(qb.download((qb.nbytes,), np.int8), n, oh, ow, cp)
        np.testing.assert_array_equal(got[..., :c].transpose(0, 3, 1, 2), ref.quantize_activation(want, scale))
        assert not got[..., c:].any()


@pytest.mark.parametrize("case", [
    dict(n=2, h=224, w=224, o=64, act="relu", cp_out=True),      # the ResNet-18 stem (layer-1 int8 layout)
    dict(n=5, h=224, w=224, o=64, act="relu", cp_out=False),     # units beyond one wave, NHWC int8
    dict(n=3, h=57, w=61, o=32, act="relu6", cp_out=False),      # odd sizes: ragged bands, odd conv rows
    dict(n=1, h=30, w=20, o=12, act="relu", cp_out=True),        # few channels (padded int8 chunk)
    dict(n=4, h=225, w=254, o=64, act="none", cp_out=False),     # conv rows of 127 pixels, plain bias
])
def test_stem_pool_kernel_exact(cuda_device, case):
    """The stem + pool kernel (7x7/2 conv over the row-expanded input, -inf pad, 3x3/2 max pool,
    pooled values through the epilogue) against the oracle's qconv2d then maxpool2d, bit for bit."""
    from mira_b200 import _lib
    K, DB = _k()
    n, h, w, o = case["n"], case["h"], case["w"], case["o"]
    rng = np.random.default_rng(n * 7 + w)
    x = rng.standard_normal((n, 3, h, w)).astype(np.float32)
    x_scale = float(np.abs(x).max() / 127.0)
    q, w_scale = ref.quantize_array(rng.standard_normal((o, 3, 7, 7)).astype(np.float32), 0)
    bias = rng.standard_normal((o, 1, 1)).astype(np.float32)
    steps, ops = [("add", 1, False)], [bias]
    if case["act"] == "relu":
        steps.append(("relu", None, False))
    elif case["act"] == "relu6":
        steps += [("maximum", 2, False), ("minimum", 3, False)]
        ops += [np.float32(0.0), np.float32(6.0)]
    _, _, y = ref.qconv2d(x, q, w_scale, x_scale, (2, 2), (3, 3), steps=steps, operands=ops)
    y = ref.maxpool2d(y, 3, 2, 1, -np.inf)
    oh, ow = (h + 6 - 7) // 2 + 1, (w + 6 - 7) // 2 + 1
    entries = K.row4_entries(ow, 2)
    xb, xq = DB.from_array(x), DB(n * h * entries * 16)
    K.quantize_nchw_to_row4(xb, n, 3, h, w, x_scale, xq, entries, 3, 2)
    wq = K.conv_weight_row4(q)
    bufs = [DB.from_array(a) for a in (wq, *K.scale_arrays(x_scale, w_scale), K.pad_channels(bias))]
    ph, pw_ = y.shape[2:]
    ldi = K.round_up(o, 16)
    yb = DB(n * ph * pw_ * o * 4)
    qb = DB(K.cp_bytes(n, ph, pw_, ldi) if case["cp_out"] else n * ph * pw_ * ldi, zero=True)
    out_scale = float(np.abs(y).max() / 127.0)
    es = [K.Step("add", "channel", ptr=bufs[4])]
    if case["act"] == "relu":
        es.append(K.Step("relu"))
    elif case["act"] == "relu6":
        es += [K.Step("maximum", "scalar", scalar=0.0), K.Step("minimum", "scalar", scalar=6.0)]
    epi = K.Epi(es, out_f32=yb, ld_f32=o, out_i8=qb, ld_i8=ldi, out_scale=out_scale,
                i8_layout=_lib.LAYOUT_CP if case["cp_out"] else _lib.LAYOUT_NHWC)
    n0 = _lib.launch_count()
    K.qconv2d_maxpool(n, h, w, 4, xq, o, 7, 7, bufs[0], wq.shape[1], (2, 2), (3, 3), (1, 1), 3, 2, 1, -np.inf,
                      K.dequant_channel(*bufs[1:4]), epi, layout=_lib.LAYOUT_ROW4, row_entries=entries)
    assert _lib.launch_count() - n0 == 1
    _same_f32(yb.download((n, ph, pw_, o), np.float32).transpose(0, 3, 1, 2), y)
    raw = qb.download((qb.nbytes,), np.int8)
    got_q = K.from_cp(raw, n, ph, pw_, ldi) if case["cp_out"] else raw.reshape(n, ph, pw_, ldi)
    np.testing.assert_array_equal(got_q[..., :o].transpose(0, 3, 1, 2), ref.quantize_activation(y, out_scale))
    assert not got_q[..., o:].any()
