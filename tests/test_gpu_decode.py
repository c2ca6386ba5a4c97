"""Host-driven W8A8 decode on the GPU: the runtime-position slice kernels against NumPy (clamped
starts included), and the transformer step program with device-resident caches against the
reference cpu target running the same quantized step graph."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _k():
    from mira_b200 import kernels as K
    from mira_b200.device import DeviceBuffer
    return K, DeviceBuffer


def _clamped(start, dims, n):
    return tuple(slice(min(max(int(s), 0), d - k), min(max(int(s), 0), d - k) + k) for s, d, k in zip(start, dims, n))


@pytest.mark.parametrize("dims,size,start,dtype", [
    ((16, 64), (1, 64), (5, 0), np.float32),
    ((16, 64), (1, 64), (40, 0), np.float32),             # clamped to the last row
    ((2, 3, 16, 8), (2, 3, 4, 8), (0, 0, -3, 0), np.float32),   # negative start clamps to 0
    ((7, 9, 11), (3, 2, 5), (2, 6, 4), np.int32),
    ((100,), (17,), (90,), np.int32),
])
def test_dynamic_slice_clamped(cuda_device, dims, size, start, dtype):
    K, DB = _k()
    rng = np.random.default_rng(len(dims))
    x = (rng.standard_normal(dims) * 100).astype(dtype)
    xb, sb, ob = DB.from_array(x), DB.from_array(np.array(start, np.int32)), DB(int(np.prod(size)) * 4)
    r = len(dims)
    K.dynamic_slice(K.View(xb, (0,) * (4 - r) + tuple(np.array(x.strides) // 4)), dims, sb, r, size,
                    K.View(ob, (0,) * (4 - r) + tuple(np.array(np.empty(size, dtype).strides) // 4)))
    np.testing.assert_array_equal(ob.download(size, dtype), x[_clamped(start, dims, size)])


@pytest.mark.parametrize("dims,upd_shape,start", [
    ((2, 3, 16, 8), (2, 3, 1, 8), (0, 0, 5, 0)),
    ((2, 3, 16, 8), (2, 3, 1, 8), (0, 0, 99, 0)),         # clamped to row 15
    ((4, 32), (2, 32), (-1, 0)),
])
def test_dynamic_update_slice_in_place_from_a_strided_view(cuda_device, dims, upd_shape, start):
    K, DB = _k()
    rng = np.random.default_rng(7)
    x = rng.standard_normal(dims).astype(np.float32)
    u = rng.standard_normal(upd_shape).astype(np.float32)
    r = len(dims)
    # the update is read through a transposed view (its last two axes stored swapped)
    ut = np.ascontiguousarray(np.swapaxes(u, -1, -2))
    st = list(np.array(ut.strides) // 4)
    st[-1], st[-2] = st[-2], st[-1]
    xb, ub, sb = DB.from_array(x), DB.from_array(ut), DB.from_array(np.array(start, np.int32))
    K.dynamic_update_slice(K.View(xb, (0,) * (4 - r) + tuple(np.array(x.strides) // 4)), dims,
                           K.View(ub, (0,) * (4 - r) + tuple(st)), upd_shape, sb, r)
    want = x.copy()
    want[_clamped(start, dims, upd_shape)] = u
    np.testing.assert_array_equal(xb.download(dims, np.float32), want)


mira_missing = False
try:
    from mira_b200 import configs, decode
    from mira_b200.plugin import install
    install()
    from mira import compiler
except ImportError:  # the host framework package is not on this machine
    mira_missing = True

SMALL = dict(layers=2, d_model=128, heads=4, d_mlp=256, vocab=64, max_seq=64)


def _programs(batch):
    g = configs.transformer(batch, seq=64, **SMALL)
    cal = [configs.random_inputs(g, 100 + i) for i in range(2)]
    pre = compiler.compile_ir(g, "cpu", quantize="w8a8", calibration=cal, precision=None)
    cpu = decode.compile_step(configs.transformer_step(batch, **SMALL), pre, "cpu")
    cuda = decode.compile_step(configs.transformer_step(batch, **SMALL), pre, "cuda")
    return cpu, cuda


@pytest.mark.skipif(mira_missing, reason="MIRA host framework (package `mira`) not importable")
def test_decoder_matches_cpu_step_program(cuda_device):
    """Greedy decode with resident caches (eager first step, CUDA-graph replays after it) against
    the reference cpu step program fed the same tokens, caches through the host.  Like the prefill,
    the f32 attention and GELU are not bit-exact, so logits are compared to a bound."""
    batch = 4
    cpu, cuda = _programs(batch)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    dec = decode.Decoder(cuda)
    prompt = np.random.default_rng(5).integers(0, 64, (batch, 8)).astype(np.int32)
    toks, logits = dec.generate(prompt, 24)
    names = [v.name for v in cpu.graph.inputs[3:]]
    caches = {n: np.zeros(v.type.shape, np.float32) for n, v in zip(names, cpu.graph.inputs[3:])}
    close = []
    for p in range(logits.shape[0]):
        out = cpu.run({"tok": toks[:, p:p + 1], "pos2": np.array([p, 0], np.int32),
                       "pos4": np.array([0, 0, p, 0], np.int32), **caches})
        caches = dict(zip(names, out[1:]))
        want = out[0][:, 0]
        scale = np.abs(want).max()
        assert np.abs(logits[p] - want).max() <= 0.05 * scale
        close.append(np.isclose(logits[p], want, rtol=1e-5, atol=1e-5 * scale).mean())
    assert np.mean(close) >= 0.5
    k0 = dec.read_cache(0)
    np.testing.assert_allclose(k0, caches[names[0]], rtol=1e-3, atol=1e-3 * np.abs(caches[names[0]]).max())
    assert not k0[:, :, logits.shape[0]:].any()          # rows past the last position untouched
