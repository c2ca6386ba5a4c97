"""The transformer path on the GPU: the sequence kernels against the CPU oracle on identical inputs
(layernorm, embedding and view copies bit for bit; softmax within a few units in the last place;
the f32 matmul within the f32 error bound of the exact product), and the decoder-only transformer
compiled W8A8 for `cuda` against MIRA's cpu target.

End-to-end the transformer cannot be bit-exact: NumPy's float32 exp/tanh are not correctly
rounded and its BLAS sums in an order of its own, so a few activations land on the other side of
an int8 rounding boundary.  The end-to-end test therefore bounds the logit error and reports the
share of logits that agree to 1e-5."""
import numpy as np
import pytest

from oracle import w8a8 as ref

pytestmark = pytest.mark.gpu


def _k():
    from mira_b200 import kernels as K
    from mira_b200.device import DeviceBuffer
    return K, DeviceBuffer


def _bits_equal(got, want):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    bad = got.view(np.uint32) != want.view(np.uint32)
    assert not bad.any(), f"{int(bad.sum())} of {bad.size} values differ; first at {np.argwhere(bad)[:3].tolist()}"


def _ulps(a, b):
    a, b = np.asarray(a, np.float32).view(np.int32).astype(np.int64), np.asarray(b, np.float32).view(np.int32)
    return np.abs(a - b)


# d = 768, 96, 256, 512, 1024 and 2048 take layernorm_tree_kernel (NumPy's pairwise tree over 8, 1, 2,
# 4, 8 and 16 leaves), with rows that leave lanes of the last warp idle; the others the general kernels
@pytest.mark.parametrize("rows,d", [(1, 768), (37, 768), (1000, 768), (5, 100), (9, 5), (3, 8), (17, 3072),
                                    (4, 8192), (3, 96), (70, 256), (33, 512), (9, 1024), (5, 2048)])
def test_layernorm_rows_bit_exact(cuda_device, rows, d):
    K, DB = _k()
    rng = np.random.default_rng(rows * 31 + d)
    x = (rng.standard_normal((rows, d)) * rng.uniform(0.05, 20, (rows, 1)) + rng.normal(0, 3, (rows, 1)))
    x = x.astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.1 * rng.standard_normal(d)).astype(np.float32)
    scale = 0.031
    ld_i8 = K.round_up(d, 16)
    xb, gb, bb = DB.from_array(x), DB.from_array(g), DB.from_array(b)
    yb, qb = DB(rows * d * 4), DB(rows * ld_i8, zero=True)
    K.layernorm_rows(xb, rows, d, d, gb, bb, 1e-5, out_f32=yb, ld_f32=d, out_i8=qb, ld_i8=ld_i8, out_scale=scale)
    want = ref.layernorm(x, g, b)
    _bits_equal(yb.download((rows, d), np.float32), want)
    np.testing.assert_array_equal(qb.download((rows, ld_i8), np.int8)[:, :d], ref.quantize_activation(want, scale))


@pytest.mark.parametrize("ld_x", [768, 770])
def test_layernorm_int8_only(cuda_device, ld_x):
    """The prefill form: int8 output only; a row stride that is not a multiple of 4 floats takes the
    general kernel, the aligned one the tree kernel, with the same bytes."""
    K, DB = _k()
    rng = np.random.default_rng(ld_x)
    rows, d = 301, 768
    full = (rng.standard_normal((rows, ld_x)) * 2 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.1 * rng.standard_normal(d)).astype(np.float32)
    xb, gb, bb, qb = DB.from_array(full), DB.from_array(g), DB.from_array(b), DB(rows * d)
    K.layernorm_rows(xb, rows, d, ld_x, gb, bb, 1e-5, out_i8=qb, ld_i8=d, out_scale=0.02)
    want = ref.quantize_activation(ref.layernorm(full[:, :d], g, b), 0.02)
    np.testing.assert_array_equal(qb.download((rows, d), np.int8), want)


def test_layernorm_strided_rows(cuda_device):
    """Rows read with a row stride larger than d (a column slice of a wider buffer)."""
    K, DB = _k()
    rng = np.random.default_rng(3)
    full = rng.standard_normal((50, 300)).astype(np.float32)
    g, b = np.ones(128, np.float32), np.zeros(128, np.float32)
    xb, gb, bb, yb = DB.from_array(full), DB.from_array(g), DB.from_array(b), DB(50 * 128 * 4)
    from mira_b200.device import DeviceSlice
    K.layernorm_rows(DeviceSlice(xb, 64 * 4), 50, 128, 300, gb, bb, 1e-5, out_f32=yb, ld_f32=128)
    _bits_equal(yb.download((50, 128), np.float32), ref.layernorm(full[:, 64:192], g, b))


@pytest.mark.parametrize("rows,n", [(1, 1024), (300, 1024), (7, 77), (5, 5), (3, 8192), (64, 16)])
def test_softmax_rows_close(cuda_device, rows, n):
    K, DB = _k()
    rng = np.random.default_rng(rows + n)
    x = (rng.standard_normal((rows, n)) * 4).astype(np.float32)
    mask = np.triu(np.ones((rows, n), bool), 1 + n // 2)
    x[mask] -= np.float32(10000)
    xb, yb = DB.from_array(x), DB(rows * n * 4)
    K.softmax_rows(xb, rows, n, n, yb, n)
    got = yb.download((rows, n), np.float32)
    want = ref.softmax(x)
    # NumPy's exp is within 3 ulp of the correctly rounded value and CUDA's expf within 2; the
    # pairwise sum and the final divide add a few more
    assert _ulps(got, want).max() <= 8, _ulps(got, want).max()
    assert np.array_equal(got == 0, want == 0)


def _bmm_case(K, DB, b0, b1, m, n, k, seed, steps=(), operands=(), a_t=False, b_t=False):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((b0, b1, m, k)).astype(np.float32)
    b = rng.standard_normal((b0, b1, k, n)).astype(np.float32)
    # device copies stored transposed when asked (strided views with a unit stride on the other axis)
    a_store = np.ascontiguousarray(a.transpose(0, 1, 3, 2)) if a_t else a
    b_store = np.ascontiguousarray(b.transpose(0, 1, 3, 2)) if b_t else b
    ab, bb = DB.from_array(a_store), DB.from_array(b_store)
    ast = (b1 * m * k, m * k, 1, m) if a_t else (b1 * m * k, m * k, k, 1)
    bst = (b1 * k * n, k * n, 1, k) if b_t else (b1 * k * n, k * n, n, 1)
    yb = DB(b0 * b1 * m * n * 4)
    epi = K.BmmEpi(list(steps), out=K.View(yb, (b1 * m * n, m * n, n, 1)))
    K.bmm_f32(b0, b1, m, n, k, K.View(ab, ast), K.View(bb, bst), epi)
    return a, b, yb.download((b0, b1, m, n), np.float32)


@pytest.mark.parametrize("shape", [(1, 1, 1, 1, 1), (2, 3, 16, 16, 8), (1, 12, 200, 64, 64), (2, 2, 130, 70, 1000),
                                   (1, 1, 257, 129, 33), (1, 1, 5, 3, 0)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False)])
def test_bmm_f32_within_error_bound(cuda_device, shape, a_t, b_t):
    K, DB = _k()
    b0, b1, m, n, k = shape
    a, b, got = _bmm_case(K, DB, b0, b1, m, n, k, sum(shape), a_t=a_t, b_t=b_t)
    exact, bound = ref.matmul_error_bound(a, b)
    assert np.all(np.abs(got - exact) <= bound + 1e-30)
    blas = ref.matmul_f32(a, b)
    assert np.all(np.abs(got - blas) <= 2 * bound + 1e-30)


@pytest.mark.parametrize("b0,b1,m,n,k", [(1, 1, 64, 300, 200), (2, 3, 17, 96, 64), (1, 1, 1, 4096, 768),
                                         (1, 1, 130, 10, 1000)])
def test_bmm_f32_w8_equals_f32_bmm_on_dequantized_weights(cuda_device, b0, b1, m, n, k):
    """Weight-only int8 B (one [K, N] weight broadcast over the batch, per-column scales): the
    staged weights are the reference's dequantized values exactly, so the product is bit-identical
    to the f32 bmm over those values, and within the f32 error bound of the exact product."""
    K, DB = _k()
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((b0, b1, m, k)).astype(np.float32)
    q, scale = ref.quantize_array((rng.standard_normal((k, n)) * rng.uniform(0.01, 2, (1, n))).astype(np.float32), 1)
    w = ref.dequantize(q, scale, 1)
    ab, qb, sb, wb = DB.from_array(a), DB.from_array(q), DB.from_array(scale), DB.from_array(w)
    bias = rng.standard_normal(n).astype(np.float32)
    biasb = DB.from_array(bias)
    av = K.View(ab, (b1 * m * k, m * k, k, 1))
    outs = []
    for w8 in (True, False):
        yb = DB(b0 * b1 * m * n * 4)
        epi = K.BmmEpi([K.BmmStep("add", "view", view=K.View(biasb, (0, 0, 0, 1)))],
                       out=K.View(yb, (b1 * m * n, m * n, n, 1)))
        if w8:
            K.bmm_f32_w8(b0, b1, m, n, k, av, K.View(qb, (0, 0, n, 1), itemsize=1), sb, epi)
        else:
            K.bmm_f32(b0, b1, m, n, k, av, K.View(wb, (0, 0, n, 1)), epi)
        outs.append(yb.download((b0, b1, m, n), np.float32))
    _bits_equal(outs[0], outs[1])
    exact, bound = ref.matmul_error_bound(a, np.broadcast_to(w, (b0, b1, k, n)))
    assert np.all(np.abs(outs[0] - (exact + bias)) <= bound + np.abs(exact + bias) * 2 ** -23 + 1e-30)


def test_bmm_attention_scores_epilogue(cuda_device):
    """q @ k^T * (1/8) + causal mask, the mask broadcast over batch and heads (stride-0 view)."""
    K, DB = _k()
    b0, b1, t, dh = 2, 3, 48, 64
    mask = np.where(np.arange(t)[:, None] >= np.arange(t)[None, :], 0.0, -10000.0).astype(np.float32)
    mb = DB.from_array(mask)
    steps = [K.BmmStep("mul", "scalar", scalar=0.125), K.BmmStep("add", "view", view=K.View(mb, (0, 0, t, 1)))]
    a, b, got = _bmm_case(K, DB, b0, b1, t, t, dh, 11, steps=steps, b_t=True)
    want = ref.matmul_f32(a, b, (("mul", 0, False), ("add", 1, False)), (np.float32(0.125), mask))
    exact, bound = ref.matmul_error_bound(a, b)
    assert np.all(np.abs(got - want) <= 0.125 * 2 * bound + np.abs(want) * 2 ** -22)


def test_embed_rows_with_positions(cuda_device):
    K, DB = _k()
    rng = np.random.default_rng(8)
    table = rng.standard_normal((256, 96)).astype(np.float32)
    pos = rng.standard_normal((40, 96)).astype(np.float32)
    idx = rng.integers(-256, 256, (3, 40)).astype(np.int32)
    tb, pb, ib, yb = DB.from_array(table), DB.from_array(pos), DB.from_array(idx), DB(3 * 40 * 96 * 4)
    K.embed_rows(tb, 256, 96, ib, 120, yb, 96, addend=pb, addend_rows=40)
    _bits_equal(yb.download((3, 40, 96), np.float32), ref.embed(table, idx, pos))


def test_embed_index_out_of_range_is_reported(cuda_device):
    """An id outside [-vocab, vocab) writes 0 and fails the next sync (the reference raises
    IndexError); the device stays usable."""
    from mira_b200 import _lib
    K, DB = _k()
    table = np.ones((4, 8), np.float32)
    idx = np.array([0, 3, 4, -5], np.int32)
    tb, ib, yb = DB.from_array(table), DB.from_array(idx), DB(4 * 8 * 4)
    K.embed_rows(tb, 4, 8, ib, 4, yb, 8)
    with pytest.raises(_lib.CudaError) as e:
        _lib.call("mira_cuda_sync")
    assert e.value.code == _lib.EKERNEL and "index" in str(e.value)
    got = yb.download((4, 8), np.float32)
    np.testing.assert_array_equal(got[:2], 1.0)
    np.testing.assert_array_equal(got[2:], 0.0)


def test_copy_view_transpose(cuda_device):
    K, DB = _k()
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 7, 3, 5)).astype(np.float32)
    xb, yb = DB.from_array(x), DB(x.nbytes)
    src = K.View(xb, (7 * 3 * 5, 5, 3 * 5, 1))            # x.transpose(0, 2, 1, 3) as a view
    K.copy_view((2, 3, 7, 5), src, K.View(yb, (3 * 7 * 5, 7 * 5, 5, 1)))
    _bits_equal(yb.download((2, 3, 7, 5), np.float32), x.transpose(0, 2, 1, 3))


def _attention_case(K, DB, b0, b1, t, dh, seed, amp=1.0, mask=True, skip=True, scale_op="mul", i8_scale=None):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((b0, b1, t, dh)) * amp).astype(np.float32)
    k = (rng.standard_normal((b0, b1, t, dh)) * amp).astype(np.float32)
    v = rng.standard_normal((b0, b1, t, dh)).astype(np.float32)
    m = np.where(np.arange(t)[:, None] >= np.arange(t)[None, :], 0.0, -10000.0).astype(np.float32)
    scale = 0.125 if scale_op == "mul" else 8.0
    qb, kb, vb, mb = (DB.from_array(x) for x in (q, k, v, m))
    st = (b1 * t * dh, t * dh, dh, 1)
    ob = DB(q.nbytes)
    tile_max = kmax = None
    tile_zero = None
    if mask and skip:
        tile_max, kmax = DB.from_array(K.mask_tile_max(m, t, t)), DB(16, zero=True)
        tile_zero = DB.from_array(K.mask_tile_zero(m, t, t))
        K.absmax_f32((b0, b1, t, dh), K.View(kb, st), kmax)
    desc = K.Attn(b0, b1, t, t, dh, K.View(qb, st), K.View(kb, st), K.View(vb, st), scale_op, scale,
                  K.View(mb, (0, 0, t, 1)) if mask else None, tile_max, kmax, tile_zero, out=K.View(ob, st))
    ws = K.attention_workspace(b0, b1, t, t, dh)      # the tensor-core path where it applies
    if ws > 0:
        desc.workspace, desc.workspace_bytes = DB(ws), ws
    qi8 = None
    if i8_scale is not None:
        qi8 = DB(q.size, zero=True)
        desc.out_i8, desc.out_scale = K.View(qi8, st, itemsize=1), i8_scale
    K.attention_f32(desc)
    steps, ops = [(scale_op, 0, False)], [np.float32(scale)]
    if mask:
        steps.append(("add", 1, False))
        ops.append(m)
    want = ref.matmul_f32(ref.softmax(ref.matmul_f32(q, np.swapaxes(k, -1, -2), steps, ops)), v)
    got = ob.download(q.shape, np.float32)
    i8 = qi8.download(q.shape, np.int8) if qi8 is not None else None
    return got, want, v, i8


@pytest.mark.parametrize("b0,b1,t,dh", [(2, 3, 100, 64), (1, 2, 64, 64), (1, 1, 1, 64), (2, 2, 200, 32), (1, 2, 70, 30),
                                        (1, 2, 130, 128), (1, 4, 300, 48)])
@pytest.mark.parametrize("skip", [True, False])
def test_attention_matches_reference_chain(cuda_device, b0, b1, t, dh, skip):
    """softmax(q @ k^T * s + causal mask) @ v against the reference's three ops."""
    K, DB = _k()
    got, want, v, _ = _attention_case(K, DB, b0, b1, t, dh, t + dh, skip=skip)
    np.testing.assert_allclose(got, want, rtol=0, atol=3e-6 * np.abs(v).max())


@pytest.mark.parametrize("b0,b1,tk,dh,scale_op", [(4, 12, 1024, 64, "mul"), (2, 3, 1000, 32, "div"),
                                                 (1, 2, 77, 128, "mul"), (3, 2, 300, 48, "mul"), (1, 1, 5, 64, "div")])
def test_single_query_attention_matches_reference_chain(cuda_device, b0, b1, tk, dh, scale_op):
    """The decode form: one query row per (batch, head) against a key/value cache of tk rows, the
    mask a runtime row (0 up to the position, -10000 after it) shared by every batch and head;
    f32 and int8 outputs."""
    K, DB = _k()
    rng = np.random.default_rng(tk + dh)
    q = rng.standard_normal((b0, b1, 1, dh)).astype(np.float32)
    k = rng.standard_normal((b0, b1, tk, dh)).astype(np.float32)
    v = rng.standard_normal((b0, b1, tk, dh)).astype(np.float32)
    pos = int(rng.integers(0, tk))
    m = np.where(np.arange(tk) <= pos, 0.0, -10000.0).astype(np.float32).reshape(1, tk)
    scale = 0.125 if scale_op == "mul" else 8.0
    qb, kb, vb, mb = (DB.from_array(x) for x in (q, k, v, m))
    kst = (b1 * tk * dh, tk * dh, dh, 1)
    qst = (b1 * dh, dh, dh, 1)
    ob, ib = DB(q.nbytes), DB(q.size, zero=True)
    desc = K.Attn(b0, b1, 1, tk, dh, K.View(qb, qst), K.View(kb, kst), K.View(vb, kst), scale_op, scale,
                  K.View(mb, (0, 0, 0, 1)), None, None, None, out=K.View(ob, qst))
    out_scale = 0.02
    desc.out_i8, desc.out_scale = K.View(ib, qst, itemsize=1), out_scale
    K.attention_f32(desc)
    want = ref.matmul_f32(ref.softmax(ref.matmul_f32(q, np.swapaxes(k, -1, -2), [(scale_op, 0, False), ("add", 1, False)],
                                                     [np.float32(scale), m])), v)
    got = ob.download(q.shape, np.float32)
    np.testing.assert_allclose(got, want, rtol=0, atol=3e-6 * np.abs(v).max())
    np.testing.assert_array_equal(ib.download(q.shape, np.int8), ref.quantize_activation(got, out_scale))


@pytest.mark.parametrize("b0,b1,t", [(1, 12, 1024), (2, 3, 333), (1, 2, 128)])
@pytest.mark.parametrize("skip", [True, False])
def test_tensor_core_attention_matches_reference_and_f32_kernel(cuda_device, monkeypatch, b0, b1, t, skip):
    """The prefill shape of config 5 (d_head 64) runs on the tensor-core path (bf16 three-piece
    split, f32 accumulation); the same tolerance against the reference's three ops as the f32 FMA
    kernel, and both kernels within that tolerance of each other."""
    K, DB = _k()
    assert K.attention_workspace(b0, b1, t, t, 64) > 0
    got, want, v, _ = _attention_case(K, DB, b0, b1, t, 64, t + 1, skip=skip)
    tol = 3e-6 * np.abs(v).max()
    np.testing.assert_allclose(got, want, rtol=0, atol=tol)
    monkeypatch.setenv("MIRA_CUDA_ATTENTION", "simt")
    assert K.attention_workspace(b0, b1, t, t, 64) == 0
    got_simt, _, _, _ = _attention_case(K, DB, b0, b1, t, 64, t + 1, skip=skip)
    np.testing.assert_allclose(got, got_simt, rtol=0, atol=tol)
    print(f"max |tc - ref| {np.abs(got - want).max():.3g}, max |simt - ref| {np.abs(got_simt - want).max():.3g}, "
          f"max|v| {np.abs(v).max():.3g}")


def test_attention_large_scores_are_not_skipped(cuda_device):
    """With scores far beyond the mask (|q.k| * scale >> 10000) the masked entries do count in the
    reference; the skip test must fail and every tile be processed."""
    K, DB = _k()
    got, want, v, _ = _attention_case(K, DB, 1, 2, 160, 64, 5, amp=60.0)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5 * np.abs(v).max())


def test_attention_div_scale_no_mask(cuda_device):
    K, DB = _k()
    got, want, v, _ = _attention_case(K, DB, 2, 3, 90, 64, 6, mask=False, scale_op="div")
    np.testing.assert_allclose(got, want, rtol=0, atol=3e-6 * np.abs(v).max())


def test_attention_int8_output(cuda_device):
    """The fused requantization equals quantize_activation of the kernel's own f32 output."""
    K, DB = _k()
    got, want, v, i8 = _attention_case(K, DB, 2, 2, 96, 64, 7, i8_scale=0.0123)
    np.testing.assert_array_equal(i8, ref.quantize_activation(got, 0.0123))
    assert np.abs(i8.astype(int) - ref.quantize_activation(want, 0.0123).astype(int)).max() <= 1


# ------------------------------------------------------------------------------ end to end

mira_missing = False
try:
    from mira_b200 import configs
    from mira_b200.plugin import install
    install()
    from mira import compiler
except ImportError:  # the host framework package is not on this machine
    mira_missing = True


@pytest.mark.skipif(mira_missing, reason="MIRA host framework (package `mira`) not importable")
@pytest.mark.parametrize("kw,batch", [(dict(seq=16, layers=2, d_model=64, heads=4, d_mlp=128, vocab=32, max_seq=16), 2),
                                      (dict(seq=128, layers=2), 2)])
def test_transformer_prefill_matches_cpu(cuda_device, kw, batch):
    g_cpu, g_cuda = configs.transformer(batch, **kw), configs.transformer(batch, **kw)
    cal = [configs.random_inputs(g_cpu, 100 + i) for i in range(2)]
    cpu = compiler.compile_ir(g_cpu, "cpu", quantize="w8a8", calibration=cal, precision=None)
    cuda = compiler.compile_ir(g_cuda, "cuda", quantize="w8a8", calibration=cal)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    feeds = configs.random_inputs(g_cpu, 1)
    want = cpu.run(feeds)
    for _ in range(2):                   # eager first run, then CUDA-graph replay
        got = cuda.run(feeds)
        assert got.shape == want.shape and got.dtype == want.dtype
        err = np.abs(got - want)
        scale = np.abs(want).max()
        close = np.isclose(got, want, rtol=1e-5, atol=1e-5 * scale)
        print(f"logits within 1e-5: {close.mean():.4%}; max |d| {err.max():.3g} of max |logit| {scale:.3g}")
        # a flipped int8 activation moves a logit by about one quantization step of one input
        assert err.max() <= 0.05 * scale
        assert close.mean() >= 0.5


@pytest.mark.skipif(mira_missing, reason="MIRA host framework (package `mira`) not importable")
@pytest.mark.parametrize("name,batch,kw", [("mlp", 64, {}),
                                           ("transformer", 2, dict(seq=64, layers=2, d_model=128, heads=4,
                                                                   d_mlp=256, vocab=64, max_seq=64))])
def test_weight_only_int8_matches_cpu(cuda_device, name, batch, kw):
    """`quantize="int8"`: int8 weights on the device, f32 activations; against the reference cpu
    target within f32 tolerance (no int8 activation rounding to flip)."""
    g_cpu, g_cuda = configs.BUILDERS[name](batch, **kw), configs.BUILDERS[name](batch, **kw)
    cpu = compiler.compile_ir(g_cpu, "cpu", quantize="int8", precision=None)
    cuda = compiler.compile_ir(g_cuda, "cuda", quantize="int8")
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    feeds = configs.random_inputs(g_cpu, 1)
    want = cpu.run(feeds)
    for _ in range(2):
        got = cuda.run(feeds)
        assert got.shape == want.shape and got.dtype == want.dtype
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max())
