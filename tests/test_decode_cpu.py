"""Host-driven W8A8 decode on the CPU: the transformer step graph (runtime-position slices, key/value
caches) planned for `cuda` and executed by the host-side stand-in device, against the reference cpu
target running the same quantized step graph."""
import numpy as np
import pytest

from fake_device import FakeDevice
from mira_b200 import configs, decode
from mira_b200.plugin import install

mira = install()
from mira import compiler  # noqa: E402

TINY = dict(layers=2, d_model=64, heads=4, d_mlp=128, vocab=32, max_seq=16)


def _prefill(batch, seq, **kw):
    g = configs.transformer(batch, seq=seq, **{**TINY, **kw})
    cal = [configs.random_inputs(g, 100 + i) for i in range(2)]
    return compiler.compile_ir(g, "cpu", quantize="w8a8", calibration=cal, precision=None)


def _steps(batch, prefill, **kw):
    """(reference cpu step program, cuda step program on the fake device, the fake device)."""
    cpu = decode.compile_step(configs.transformer_step(batch, **{**TINY, **kw}), prefill, "cpu")
    dev = FakeDevice()
    cuda = decode.compile_step(configs.transformer_step(batch, **{**TINY, **kw}), prefill, "cuda", executor=dev)
    return cpu, cuda, dev


def _feeds(g, tok, p, caches):
    return {"tok": tok.reshape(-1, 1), "pos2": np.array([p, 0], np.int32), "pos4": np.array([0, 0, p, 0], np.int32),
            **caches}


def test_step_scales_come_from_prefill():
    pre = _prefill(2, 16)
    cpu, _, _ = _steps(2, pre)
    want = [op.attrs["x_scale"] for op in pre.graph.ops if op.kind == "qmatmul"]
    got = [op.attrs["x_scale"] for op in cpu.graph.ops if op.kind == "qmatmul"]
    assert len(got) == len(want) == 6 * 2 + 1          # q, k, v, out, two MLP per layer; LM head
    assert got == want


def test_step_plan_updates_caches_in_place():
    pre = _prefill(2, 16)
    _, cuda, dev = _steps(2, pre)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    exe = cuda.segments[0].executable
    pairs = exe.state_pairs()
    assert sorted(x.name for x, _ in pairs) == ["k0", "k1", "v0", "v1"]
    kinds = [l.kind for l in exe.plan.launches]
    assert kinds.count("dyn_update") == 4 and kinds.count("dyn_slice") == 2          # position row, mask row
    assert "copy_view" not in kinds                         # no cache is copied
    assert kinds.count("qgemm") == 4 * 2 + 1 and kinds.count("attention") == 2


def test_step_program_matches_cpu_with_host_caches():
    """Standard protocol (every cache in and out through the host), several positions."""
    pre = _prefill(2, 16)
    cpu, cuda, _ = _steps(2, pre)
    rng = np.random.default_rng(3)
    names = [v.name for v in cpu.graph.inputs[3:]]
    caches_c = {n: np.zeros(v.type.shape, np.float32) for n, v in zip(names, cpu.graph.inputs[3:])}
    caches_g = dict(caches_c)
    for p in range(6):
        tok = rng.integers(0, 32, 2).astype(np.int32)
        want = cpu.run(_feeds(cpu.graph, tok, p, caches_c))
        got = cuda.run(_feeds(cuda.graph, tok, p, caches_g))
        for w, g_ in zip(want, got):
            assert w.shape == g_.shape
            np.testing.assert_array_equal(g_, w)
        caches_c = dict(zip(names, want[1:]))
        caches_g = dict(zip(names, got[1:]))


def test_decoder_with_resident_caches_matches_host_loop():
    pre = _prefill(2, 16)
    cpu, cuda, _ = _steps(2, pre)
    dec = decode.Decoder(cuda)
    prompt = np.random.default_rng(5).integers(0, 32, (2, 4)).astype(np.int32)
    toks, logits = dec.generate(prompt, 6)
    assert toks.shape == (2, 10) and logits.shape == (9, 2, 32)
    np.testing.assert_array_equal(toks[:, :4], prompt)
    # the same tokens through the reference cpu step program, caches through the host
    names = [v.name for v in cpu.graph.inputs[3:]]
    caches = {n: np.zeros(v.type.shape, np.float32) for n, v in zip(names, cpu.graph.inputs[3:])}
    for p in range(9):
        out = cpu.run(_feeds(cpu.graph, toks[:, p], p, caches))
        np.testing.assert_array_equal(logits[p], out[0][:, 0])
        caches = dict(zip(names, out[1:]))
        if p >= 3:
            assert np.array_equal(toks[:, p + 1], out[0][:, 0].argmax(axis=1))
    for i, n in enumerate(names):
        np.testing.assert_array_equal(dec.read_cache(i), caches[n])


def test_decoder_position_limit():
    pre = _prefill(1, 16)
    _, cuda, _ = _steps(1, pre)
    dec = decode.Decoder(cuda)
    with pytest.raises(ValueError):
        dec.generate(np.zeros((1, 10), np.int32), 8)


def test_w8a8_decode_rows_track_prefill_rows():
    """Decode at position p sees the same int8 activations as prefill row p up to rounding of the
    f32 attention sums, so the logits agree closely (reference cpu target on both sides)."""
    B, T = 2, 16
    pre = _prefill(B, T)
    cpu, _, _ = _steps(B, pre)
    tok = np.random.default_rng(1).integers(0, 32, (B, T)).astype(np.int32)
    want = pre.run({"tok": tok})
    names = [v.name for v in cpu.graph.inputs[3:]]
    caches = {n: np.zeros(v.type.shape, np.float32) for n, v in zip(names, cpu.graph.inputs[3:])}
    scale = np.abs(want).max()
    for p in range(T):
        out = cpu.run(_feeds(cpu.graph, tok[:, p], p, caches))
        caches = dict(zip(names, out[1:]))
        assert np.abs(out[0][:, 0] - want[:, p]).max() <= 0.05 * scale
