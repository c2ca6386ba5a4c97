"""The CPU oracle pinned against the reference's own outputs (tests/golden/*.npz, produced by
tests/golden/make_golden.py from myramay/MIRA itself).  Everything must match bit for bit."""
from pathlib import Path

import numpy as np
import pytest

from oracle import w8a8 as ref

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    return np.load(GOLDEN / f"{name}.npz")


def _steps(z, i):
    return [(str(f), None if int(k) < 0 else int(k), bool(s))
            for f, k, s in zip(z[f"c{i}_fns"], z[f"c{i}_idx"], z[f"c{i}_sw"])]


def _same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype
    assert np.array_equal(a, b, equal_nan=True), f"{int((a != b).sum())} values differ"


def test_quantize_activation_golden():
    z = _load("quantize_activation")
    for s, x, q in zip(z["scales"], z["x"], z["q"]):
        _same(ref.quantize_activation(x, float(s)), q)


def test_quantize_array_golden():
    z = _load("quantize_array")
    q, s = ref.quantize_array(z["w"], 1)
    _same(q, z["q_axis1"])
    _same(s, z["s_axis1"])
    q, s = ref.quantize_array(z["wc"], 0)
    _same(q, z["q_axis0"])
    _same(s, z["s_axis0"])


@pytest.mark.parametrize("i", range(5))
def test_qmatmul_golden(i):
    z = _load("qmatmul")
    ops = [z[f"c{i}_op{j}"] for j in range(int(z[f"c{i}_n_operands"]))]
    _, _, y = ref.qmatmul(z[f"c{i}_x"], z[f"c{i}_q"], z[f"c{i}_w_scale"], float(z[f"c{i}_x_scale"]),
                          steps=_steps(z, i), operands=ops)
    _same(y, z[f"c{i}_y"])


@pytest.mark.parametrize("i", range(5))
def test_qconv2d_golden(i):
    z = _load("qconv2d")
    s, p, d = (int(v) for v in z[f"c{i}_geom"])
    ops = [z[f"c{i}_op{j}"] for j in range(int(z[f"c{i}_n_operands"]))]
    xq, acc, y = ref.qconv2d(z[f"c{i}_x"], z[f"c{i}_q"], z[f"c{i}_w_scale"], float(z[f"c{i}_x_scale"]), (s, s),
                             (p, p), (d, d), steps=_steps(z, i), operands=ops)
    assert ref.conv_sums_exact_in_f32(xq, z[f"c{i}_q"])
    _same(y, z[f"c{i}_y"])


@pytest.mark.parametrize("i", range(5))
def test_qdwconv2d_golden(i):
    """The opt-in int8 depthwise op: the reference's own qconv2d with groups == channels."""
    z = _load("qdwconv2d")
    s, p, d = (int(v) for v in z[f"c{i}_geom"])
    ops = [z[f"c{i}_op{j}"] for j in range(int(z[f"c{i}_n_operands"]))]
    xq, acc, y = ref.qdwconv2d(z[f"c{i}_x"], z[f"c{i}_q"], z[f"c{i}_w_scale"], float(z[f"c{i}_x_scale"]), (s, s),
                               (p, p), (d, d), steps=_steps(z, i), operands=ops)
    assert np.abs(acc).max() < 2 ** 24
    _same(y, z[f"c{i}_y"])


def test_f32_ops_golden():
    z = _load("f32_ops")
    _same(ref.maxpool2d(z["pool_x"], 3, 2, 1, -np.inf), z["pool_pad_3_2"])
    _same(ref.maxpool2d(z["pool_x"], 2, 2), z["pool_2_2"])
    _same(ref.mean_hw(z["mean_x"]), z["mean"])
    _same(ref.mean_hw(z["mean_x2"]).reshape(z["mean2"].shape), z["mean2"])
    _same(ref.dwconv2d(z["dw_x"], z["dw_w"], (1, 1), (1, 1)), z["dw_s1"])
    _same(ref.dwconv2d(z["dw_x"], z["dw_w"], (2, 2), (1, 1),
                       steps=[("add", 2, False), ("maximum", 3, False), ("minimum", 4, False)],
                       operands=[z["dw_b"], np.float32(0), np.float32(6)]), z["dw_s2_relu6"])


@pytest.mark.parametrize("n", [1, 3, 7, 8, 9, 49, 64, 127, 128, 129, 196, 784, 3136])
def test_pairwise_sum_order_matches_numpy(n):
    """NumPy's float32 summation order, restated (the device mean kernel uses the same order)."""
    rng = np.random.default_rng(n)
    for _ in range(20):
        v = (rng.standard_normal(n) * rng.uniform(0.1, 1e3)).astype(np.float32)
        want = np.add.reduce(v)
        got = ref.pairwise_sum_f32(v)
        assert np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32)


def test_int_conv_matches_einsum_definition():
    """The exact integer convolution equals a direct per-pixel definition on a small case."""
    rng = np.random.default_rng(3)
    xq = rng.integers(-127, 128, (1, 3, 6, 5)).astype(np.int8)
    q = rng.integers(-127, 128, (2, 3, 3, 3)).astype(np.int8)
    acc = ref.int_conv2d(xq, q, (2, 2), (1, 1))
    xp = np.pad(xq.astype(np.int64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    for o in range(2):
        for y in range(acc.shape[2]):
            for x in range(acc.shape[3]):
                assert acc[0, o, y, x] == (xp[0, :, 2 * y:2 * y + 3, 2 * x:2 * x + 3] * q[o]).sum()


def test_qgemm_rowcol_reduces_to_qmatmul_with_a_scalar_row_scale():
    """The GEMM sweep's per-row scale restatement equals the reference qmatmul formula (ops.py:618)
    when every row has the same scale."""
    rng = np.random.default_rng(5)
    a = rng.integers(-127, 128, (9, 40)).astype(np.int8)
    b = rng.integers(-127, 128, (40, 11)).astype(np.int8)
    cs = rng.uniform(1e-3, 1e-2, 11).astype(np.float32)
    xs = np.float32(0.02)
    _, y = ref.qgemm_rowcol(a, b, np.full(9, xs, np.float32), cs)
    _, _, y2 = ref.qmatmul(a.astype(np.float32) * xs, b, cs, float(xs))
    # x = a * xs quantizes back to a exactly; the formulas then coincide
    _same(y, y2)


def test_planted_error_is_caught():
    """A test that the checks bite: an oracle with a deliberately wrong rounding (half away from
    zero instead of half to even) disagrees with the golden quantization."""
    z = _load("quantize_activation")
    s, x, q = z["scales"][0], z["x"][0], z["q"][0]
    wrong = np.clip(np.sign(x) * np.floor(np.abs(x / np.float32(s)) + 0.5), -127, 127).astype(np.int8)
    assert not np.array_equal(wrong, q)


@pytest.mark.parametrize("d", [1, 5, 8, 64, 100, 768, 1000])
def test_layernorm_pairwise_restatement_is_numpy(d):
    """The device layernorm's order (pairwise sums, f32 divide by d, IEEE sqrt) is NumPy's."""
    rng = np.random.default_rng(d)
    x = (rng.standard_normal((9, d)) * 3 + 1).astype(np.float32)
    g, b = rng.standard_normal(d).astype(np.float32), rng.standard_normal(d).astype(np.float32)
    a, e = ref.layernorm(x, g, b), ref.layernorm_rows_explicit(x, g, b)
    assert np.array_equal(a.view(np.uint32), e.view(np.uint32))


def test_sequence_ops_match_reference_fixtures():
    """layernorm / gather bit for bit, softmax / f32 matmul to f32 rounding (NumPy's exp and BLAS
    may differ between CPUs), against outputs of the reference's mira.ops.evaluate."""
    z = np.load(GOLDEN / "sequence.npz")
    for d in (768, 100, 5):
        _same(ref.layernorm(z[f"ln{d}_x"], z[f"ln{d}_g"], z[f"ln{d}_b"]), z[f"ln{d}_y"])
        _same(ref.layernorm_rows_explicit(z[f"ln{d}_x"], z[f"ln{d}_g"], z[f"ln{d}_b"]), z[f"ln{d}_y"])
    np.testing.assert_allclose(ref.softmax(z["sm_x"]), z["sm_y"], rtol=1e-6, atol=1e-12)
    y = ref.matmul_f32(z["mm_a"], z["mm_b"], (("mul", 0, False), ("add", 1, False)), (np.float32(0.125), z["mm_mask"]))
    np.testing.assert_allclose(y, z["mm_y"], rtol=1e-6, atol=1e-5)
    _same(ref.embed(z["ga_table"], z["ga_idx"]), z["ga_y"])


def test_weight_only_dequantize_golden():
    """quantize_array along both axes (an all-zero column gets scale 1) and the dequantize constant,
    bit for bit against the reference's own quantize_array and ops.evaluate("dequantize")."""
    z = _load("weight_only")
    w = z["w_axis1"]
    for axis in (0, 1):
        q, s = z[f"q_axis{axis}"], z[f"s_axis{axis}"]
        d = ref.dequantize(q, s, axis)
        assert d.dtype == np.float32
        assert np.array_equal(d.view(np.uint32), z[f"w_axis{axis}"].view(np.uint32))
    assert z["s_axis0"].shape == (96,) and z["s_axis1"].shape == (40,) and z["s_axis1"][7] == 1.0
    assert not z["q_axis1"][:, 7].any()
    assert w.shape == (96, 40)
