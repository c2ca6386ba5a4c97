"""CPU checks of the arithmetic two kernels rely on, restated with NumPy integer/bit operations (no GPU):

- the tensor-core attention's operand split (mira_b200/csrc/attention_tc.cuh, atc_pack8): an f32 value
  x is x0 + x1 + x2 exactly, x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1) with round to
  nearest even, and the remainder after x1 is itself a bf16 value (so nothing is lost);
- the int8 depthwise kernel's tap layout (mira_b200/csrc/memory_bound.cuh, qdwconv3x3_kernel): the byte
  permutes that turn pixel words (4 channels each) into per-channel byte streams, the funnel shift
  that picks a column's three taps and the weight word (w0, w1, w2, 0), so that one dp4a per row adds
  exactly the row's three products.  __byte_perm, __funnelshift_r and __dp4a are restated from their
  documented semantics."""
import numpy as np

RNG = np.random.default_rng(12345)


# ---------------------------------------------------------------- bf16 three-piece split

def _bf16_rn(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32 (finite inputs)."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32).view(np.float32)


def _random_f32(n: int) -> np.ndarray:
    mant = RNG.integers(0, 1 << 23, n, dtype=np.uint32)
    expo = RNG.integers(1 + 30, 254 - 30, n, dtype=np.uint32)     # away from overflow and subnormals
    sign = RNG.integers(0, 2, n, dtype=np.uint32) << 31
    return (sign | (expo << 23) | mant).view(np.float32)


def test_three_bf16_pieces_are_exact():
    x = np.concatenate([_random_f32(200000), RNG.standard_normal(50000).astype(np.float32),
                        RNG.uniform(0, 1, 50000).astype(np.float32)])
    x0 = _bf16_rn(x)
    r0 = (x - x0).astype(np.float32)
    assert np.array_equal(r0.astype(np.float64), x.astype(np.float64) - x0.astype(np.float64))   # exact in f32
    x1 = _bf16_rn(r0)
    r1 = (r0 - x1).astype(np.float32)
    assert np.array_equal(r1.astype(np.float64), r0.astype(np.float64) - x1.astype(np.float64))
    x2 = _bf16_rn(r1)
    assert np.array_equal(x2, r1)                       # the last remainder is a bf16 value
    total = x0.astype(np.float64) + x1.astype(np.float64) + x2.astype(np.float64)
    assert np.array_equal(total, x.astype(np.float64))


def test_dropped_piece_products_are_below_2_pow_minus_24():
    """x * y = sum of x_i * y_j; the kernel drops the three terms with i + j > 2."""
    x = _random_f32(100000)
    y = _random_f32(100000)
    px = [_bf16_rn(x)]
    px.append(_bf16_rn((x - px[0]).astype(np.float32)))
    px.append((x - px[0] - px[1]).astype(np.float32))
    py = [_bf16_rn(y)]
    py.append(_bf16_rn((y - py[0]).astype(np.float32)))
    py.append((y - py[0] - py[1]).astype(np.float32))
    pxd = [p.astype(np.float64) for p in px]
    pyd = [p.astype(np.float64) for p in py]
    dropped = pxd[1] * pyd[2] + pxd[2] * pyd[1] + pxd[2] * pyd[2]
    exact = x.astype(np.float64) * y.astype(np.float64)
    assert np.all(np.abs(dropped) <= 2.0 ** -24 * np.abs(exact))


# ---------------------------------------------------------------- dp4a tap layout

def _byte_perm(x: int, y: int, s: int) -> int:
    b = [(x >> (8 * i)) & 255 for i in range(4)] + [(y >> (8 * i)) & 255 for i in range(4)]
    return sum(b[(s >> (4 * n)) & 7] << (8 * n) for n in range(4))


def _funnelshift_r(lo: int, hi: int, sh: int) -> int:
    return (((hi << 32) | lo) >> (sh & 31)) & 0xFFFFFFFF


def _s8(v: int) -> int:
    return v - 256 if v >= 128 else v


def _dp4a(a: int, b: int, c: int) -> int:
    return c + sum(_s8((a >> (8 * i)) & 255) * _s8((b >> (8 * i)) & 255) for i in range(4))


def _word(bs) -> int:
    return sum((int(v) & 255) << (8 * i) for i, v in enumerate(bs))


def _row_sums(xr, w0, w1, w2, S, OXT):
    """One input row of the kernel: per column t and channel c the dp4a of the tap word and the
    weight word, in the kernel's order of byte permutes."""
    wr = []
    for c in range(4):
        t01 = _byte_perm(w0, w1, c | ((4 + c) << 4))
        wr.append(_byte_perm(t01, w2, 0x0010 | ((4 + c) << 8)) & 0x00FFFFFF)
    a01l, a01h = _byte_perm(xr[0], xr[1], 0x5140), _byte_perm(xr[0], xr[1], 0x7362)
    a23l, a23h = _byte_perm(xr[2], xr[3], 0x5140), _byte_perm(xr[2], xr[3], 0x7362)
    lo = [_byte_perm(a01l, a23l, 0x5410), _byte_perm(a01l, a23l, 0x7632),
          _byte_perm(a01h, a23h, 0x5410), _byte_perm(a01h, a23h, 0x7632)]
    if len(xr) == 6:
        b45l, b45h = _byte_perm(xr[4], xr[5], 0x5140), _byte_perm(xr[4], xr[5], 0x7362)
        hi = [b45l, b45l >> 16, b45h, b45h >> 16]
    else:
        hi = [xr[4], xr[4] >> 8, xr[4] >> 16, xr[4] >> 24]
    out = np.zeros((OXT, 4), np.int64)
    for t in range(OXT):
        for c in range(4):
            taps = lo[c] if t == 0 else _funnelshift_r(lo[c], hi[c], 8 * S * t)
            out[t, c] = _dp4a(taps, wr[c], 0)
    return out


def test_int8_depthwise_dp4a_taps_equal_direct_sums():
    for S, OXT in ((1, 4), (2, 2)):
        nin = (OXT - 1) * S + 3
        for _ in range(1500):
            x = RNG.integers(-128, 128, (nin, 4))          # pixel, channel
            w = RNG.integers(-128, 128, (3, 4))            # tap j, channel
            got = _row_sums([_word(px) for px in x], *(_word(w[j]) for j in range(3)), S, OXT)
            want = np.array([[sum(int(x[S * t + j, c]) * int(w[j, c]) for j in range(3)) for c in range(4)]
                             for t in range(OXT)])
            np.testing.assert_array_equal(got, want)


def test_int8_depthwise_dp4a_extreme_values():
    """All-(-128) and all-127 bytes: the largest products and the sign handling of every byte."""
    for S, OXT in ((1, 4), (2, 2)):
        nin = (OXT - 1) * S + 3
        for xv, wv in ((-128, -128), (-128, 127), (127, 127), (127, -128)):
            x = np.full((nin, 4), xv)
            w = np.full((3, 4), wv)
            got = _row_sums([_word(px) for px in x], *(_word(w[j]) for j in range(3)), S, OXT)
            assert np.all(got == 3 * xv * wv)
