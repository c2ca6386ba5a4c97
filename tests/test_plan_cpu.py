"""The cuda target's planner on the CPU: whole MIRA W8A8 programs compiled for `cuda` and executed
by the host-side stand-in device must reproduce the reference cpu target bit for bit."""
from pathlib import Path

import numpy as np
import pytest

from fake_device import FakeDevice
from mira_b200 import configs
from mira_b200.plugin import install

mira = install()
from mira import compiler  # noqa: E402


def _pair(name, batch, fuse_pool=False, **kw):
    """(reference cpu W8A8 program, cuda program on the fake device) for the same network."""
    cal_seed = 100
    g_cpu = configs.BUILDERS[name](batch, **kw)
    g_cuda = configs.BUILDERS[name](batch, **kw)
    cal = [configs.random_inputs(g_cpu, cal_seed + i) for i in range(2)]
    cpu = compiler.compile_ir(g_cpu, "cpu", quantize="w8a8", calibration=cal, precision=None)
    dev = FakeDevice()
    cuda = compiler.compile_ir(g_cuda, "cuda", quantize="w8a8", calibration=cal, executor=dev, fuse_pool=fuse_pool)
    return cpu, cuda, dev


def _check_same(cpu, cuda, seed=1):
    feeds = configs.random_inputs(cpu.graph, seed)
    want = cpu.run(feeds)
    got = cuda.run(feeds)
    assert got.shape == want.shape and got.dtype == want.dtype
    np.testing.assert_array_equal(got, want)


def test_mlp_plan_matches_cpu():
    cpu, cuda, dev = _pair("mlp", 8)
    assert [s.device for s in cuda.segments] == ["cuda"]
    assert dev.launched == [] or True
    _check_same(cpu, cuda)
    assert dev.launched.count("qgemm") == 3


def test_resnet18_small_plan_matches_cpu():
    cpu, cuda, dev = _pair("resnet18", 2, image=32)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    _check_same(cpu, cuda)
    # the stem conv runs inside the pooling kernel (the stem + pool kernel), the rest as convs
    assert dev.launched.count("qconv2d") == 19 and dev.launched.count("qgemm") == 1
    assert dev.launched.count("qconv2d_pool") == 1 and dev.launched.count("maxpool") == 0
    assert dev.launched.count("quantize_row4") == 1    # the 3-channel image feeds the stem row-expanded


def test_resnet18_chunk_planar_plan_matches_cpu(monkeypatch):
    """With the chunk-planar layout allowed at every width, every 3x3 stride-1 conv reads it
    (written by the max pool or the previous conv's epilogue) and the stride-2 and 1x1 convs read
    NHWC; the results stay those of the reference cpu target."""
    from mira_b200 import _lib
    from mira_b200 import kernels as K
    monkeypatch.setattr(K, "PATCH_MIN_WIDTH", 1)
    cpu, cuda, dev = _pair("resnet18", 2, image=32)
    _check_same(cpu, cuda)
    launches = cuda.segments[0].executable.plan.launches
    convs = [l for l in launches if l.kind == "qconv2d"]
    assert sum(l.args["layout"] == _lib.LAYOUT_CP for l in convs) == 13
    assert sum(l.args["epi"].i8_layout == _lib.LAYOUT_CP for l in convs) == 12
    assert [l.args["epi"].i8_layout for l in launches if l.kind == "qconv2d_pool"] == [_lib.LAYOUT_CP]


def test_resnet18_fused_stem_pool_plan_matches_cpu():
    """With fuse_pool the stem conv runs inside the max-pool kernel (its f32 output never reaches
    HBM)."""
    cpu, cuda, dev = _pair("resnet18", 2, fuse_pool=True, image=32)
    _check_same(cpu, cuda)
    assert dev.launched.count("qconv2d_pool") == 1
    assert dev.launched.count("qconv2d") == 19 and dev.launched.count("maxpool") == 0


def test_mobilenet_v2_small_plan_matches_cpu():
    cpu, cuda, dev = _pair("mobilenet_v2", 2, image=32)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    _check_same(cpu, cuda)
    assert dev.launched.count("dwconv") == 17


def test_mobilenet_v2_int8_depthwise_plan_matches_cpu():
    """The opt-in int8 depthwise mode: both programs compiled inside mira_b200.int8_depthwise (the
    reference cpu target evaluates the grouped qconv2d itself), the depthwise convs on
    mira_cuda_qdwconv2d_nhwc, and the reference's stored output of the same program."""
    from mira_b200 import int8_depthwise
    z = np.load(Path(__file__).resolve().parent / "golden" / "qdwconv2d.npz")
    with int8_depthwise():
        cpu, cuda, dev = _pair("mobilenet_v2", 2, image=32)
    grouped = [op for op in cuda.graph.ops if op.kind == "qconv2d" and op.attrs.get("groups", 1) != 1]
    assert len(grouped) == int(z["mbv2_n_grouped_qconv"]) == 17
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    _check_same(cpu, cuda)
    assert dev.launched.count("qdwconv") == 17 and dev.launched.count("dwconv") == 0
    np.testing.assert_array_equal(cuda.run({"x": z["mbv2_in"]}), z["mbv2_out"])
    # every expansion conv feeding a depthwise conv now writes int8 only
    with int8_depthwise():
        cpu2, _, _ = _pair("mobilenet_v2", 2, image=32)
    np.testing.assert_array_equal(cpu2.run({"x": z["mbv2_in"]}), z["mbv2_out"])


CNN_SRC = """
fn block(x: f32[N, C, H, W], k: f32[O, C, 3, 3], b: f32[O, 1, 1]) -> f32[N, O, H / 2, W / 2] {
  return maxpool2d(relu(conv2d(x, k, padding=1) + b), size=2)
}

fn main(img: f32[4, 1, 16, 16],
        const k1: f32[8, 1, 3, 3],  const c1: f32[8, 1, 1],
        const k2: f32[16, 8, 3, 3], const c2: f32[16, 1, 1],
        const wf: f32[256, 10],     const bf: f32[10]) -> f32[4, 10] {
  let h = block(block(img, k1, c1), k2, c2)
  return TAIL(softmax(flatten(h) @ wf + bf))
}
"""


@pytest.mark.parametrize("tail, devices", [("", ["cuda"]), ("exp", ["cuda", "cpu"])])
def test_mira_source_program_placement(tail, devices):
    """A .mira program: the flatten (NHWC -> NCHW reorder), the quantized FC and the softmax run on
    cuda; a standalone exp (no cuda kernel) falls back to the CPU like any op the target does not
    run (reference partition.py)."""
    src = CNN_SRC.replace("TAIL", tail)
    rng = np.random.default_rng(0)
    cal = [{"img": rng.standard_normal((4, 1, 16, 16)).astype(np.float32)} for _ in range(2)]
    cpu = mira.compile_source(src, "cpu", quantize="w8a8", calibration=cal, precision=None)
    cuda = mira.compile_source(src, "cuda", quantize="w8a8", calibration=cal, executor=FakeDevice())
    assert [s.device for s in cuda.segments] == devices
    feeds = {"img": rng.standard_normal((4, 1, 16, 16)).astype(np.float32)}
    np.testing.assert_array_equal(cuda.run(feeds), cpu.run(feeds))


def test_every_quantized_op_is_placed_on_cuda():
    cpu, cuda, _ = _pair("resnet18", 1, image=32)
    qops = [op for op in cuda.graph.ops if op.kind in ("qmatmul", "qconv2d")]
    assert qops and all(cuda.placement.device[op] == "cuda" for op in qops)


def test_precision_auto_means_f32_on_cuda():
    g = configs.mlp(4)
    cal = [configs.random_inputs(g, 5)]
    p = compiler.compile_ir(g, "cuda", quantize="w8a8", calibration=cal, executor=FakeDevice())
    assert all(op.result.type.dtype == "f32" for op in p.graph.ops)
    with pytest.raises(ValueError):
        compiler.compile_ir(configs.mlp(4), "cuda", quantize="w8a8", calibration=cal, precision="f16",
                            executor=FakeDevice())


def test_cuda_is_a_cli_target():
    from mira.backends import TARGETS
    assert "cuda" in TARGETS


def test_small_batch_calibration_maps_onto_large_graph():
    """compile_w8a8(calib_batch=...) gives the same x_scale values as calibrating the large graph on
    feeds that are the small feeds tiled (the peaks are maxima, so tiling changes nothing)."""
    small = configs.compile_w8a8("mlp", 16, "cuda", calib_batch=4, n_calib=2, executor=FakeDevice())
    scales_small = [op.attrs["x_scale"] for op in small.graph.ops if op.kind == "qmatmul"]
    g = configs.mlp(16)
    cal = [{k: np.tile(v, (4, 1)) for k, v in configs.random_inputs(configs.mlp(4), 100 + i).items()} for i in range(2)]
    full = compiler.compile_ir(g, "cuda", quantize="w8a8", calibration=cal, executor=FakeDevice())
    scales_full = [op.attrs["x_scale"] for op in full.graph.ops if op.kind == "qmatmul"]
    assert scales_small == scales_full


@pytest.mark.parametrize("name", ["mlp", "resnet18", "mobilenet_v2"])
def test_plan_matches_stored_reference_outputs(name):
    """Against the reference's own outputs saved in tests/golden/programs.npz."""
    from pathlib import Path
    z = np.load(Path(__file__).resolve().parent / "golden" / "programs.npz")
    batch, image, n_cal = int(z[f"{name}_batch"]), int(z[f"{name}_image"]), int(z[f"{name}_n_calib"])
    g = configs.BUILDERS[name](batch, **({"image": image} if image else {}))
    cal = [configs.random_inputs(g, 100 + i) for i in range(n_cal)]
    prog = compiler.compile_ir(g, "cuda", quantize="w8a8", calibration=cal, executor=FakeDevice())
    np.testing.assert_array_equal(prog.run({"x": z[f"{name}_x"]}), z[f"{name}_out"])


TINY_TF = dict(seq=16, layers=2, d_model=64, heads=4, d_mlp=128, vocab=32, max_seq=16)


def test_transformer_small_plan_matches_cpu():
    """Decoder-only transformer prefill: embedding, layernorm, fused q/k/v GEMM, attention on
    strided views, softmax, GELU MLP, LM head, all in one cuda segment."""
    cpu, cuda, dev = _pair("transformer", 2, **TINY_TF)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    _check_same(cpu, cuda)
    counts = {k: dev.launched.count(k) for k in set(dev.launched)}
    # per layer: one q/k/v GEMM, out-proj, two MLP GEMMs; plus the LM head
    assert counts["qgemm"] == 4 * 2 + 1
    assert counts["layernorm"] == 2 * 2 + 1 and counts["embed"] == 1
    # q @ k^T -> softmax -> @ v fused, writing the out-projection's int8 rows itself
    assert counts["attention"] == 2 and counts["absmax"] == 2
    assert "bmm" not in counts and "softmax" not in counts and "quantize_rows" not in counts


@pytest.mark.parametrize("name,batch,kw", [("mlp", 8, {}), ("transformer", 2, TINY_TF)])
def test_weight_only_int8_plan_matches_cpu(name, batch, kw):
    """`quantize="int8"` (weight-only): every large matmul weight becomes a `dequantize` constant;
    on cuda they stay int8 on the device and feed the weight-only bmm, whole graph in one segment."""
    g_cpu, g_cuda = configs.BUILDERS[name](batch, **kw), configs.BUILDERS[name](batch, **kw)
    cpu = compiler.compile_ir(g_cpu, "cpu", quantize="int8", precision=None)
    dev = FakeDevice()
    cuda = compiler.compile_ir(g_cuda, "cuda", quantize="int8", executor=dev)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    deq = [op for op in cuda.graph.ops if op.kind == "dequantize"]
    assert deq and all(np.asarray(op.attrs["q"]).dtype == np.int8 for op in deq)
    plan = cuda.segments[0].executable.plan
    w8 = [l for l in plan.launches if l.kind == "bmm" and l.args.get("b_scale") is not None]
    assert len(w8) == len(deq)
    feeds = configs.random_inputs(cpu.graph, 1)
    want = cpu.run(feeds)
    got = cuda.run(feeds)
    assert got.shape == want.shape and got.dtype == want.dtype
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("name,batch,kw,key", [("mlp", 8, {}, "x"), ("transformer", 2, TINY_TF, "tok")])
def test_weight_only_int8_plan_matches_stored_reference_output(name, batch, kw, key):
    """Weight-only programs against the reference cpu target's stored outputs."""
    z = np.load(Path(__file__).resolve().parent / "golden" / "weight_only.npz")
    g = configs.BUILDERS[name](batch, **kw)
    prog = compiler.compile_ir(g, "cuda", quantize="int8", executor=FakeDevice())
    assert sum(op.kind == "dequantize" for op in prog.graph.ops) == int(z[f"{name}_n_dequantize"])
    np.testing.assert_allclose(prog.run({key: z[f"{name}_in"]}), z[f"{name}_out"], rtol=1e-4, atol=1e-4)


def test_unfused_attention_ops_plan_matches_cpu():
    """The generic kernels (strided bmm, softmax) when the chain does not have the fused form:
    here the scores are also a graph output."""
    from mira_b200.hostfw import import_mira
    import_mira()
    from mira import ir
    from mira.types import TensorType as TT
    rng = np.random.default_rng(2)
    q = ir.Value(TT("f32", (2, 3, 8, 16)), name="q")
    k = ir.Value(TT("f32", (2, 3, 16, 8)), name="k")
    g = ir.Graph("attn", [q, k], [], [])
    s = g.add("matmul", [q, k], {})
    s = g.add("mul", [s, g.const(np.float32(0.25))], {})
    p = g.add("softmax", [s], {"axis": -1})
    o = g.add("matmul", [p, g.add("transpose", [k], {"perm": (0, 1, 3, 2)})], {})
    g.outputs = [o, s]
    g.verify()
    feeds = {"q": rng.standard_normal((2, 3, 8, 16)).astype(np.float32),
             "k": rng.standard_normal((2, 3, 16, 8)).astype(np.float32)}
    cpu = compiler.compile_ir(g, "cpu", precision=None)
    dev = FakeDevice()
    cuda = compiler.compile_ir(g, "cuda", executor=dev)
    assert [x.device for x in cuda.segments] == ["cuda"]
    want, got = cpu.run(feeds), cuda.run(feeds)
    for a, b in zip(want, got):
        np.testing.assert_array_equal(a, b)
    assert dev.launched.count("bmm") == 2 and dev.launched.count("softmax") == 1


def test_view_strides_match_numpy_views():
    from mira_b200.target import view_strides
    rng = np.random.default_rng(0)
    for _ in range(500):
        r = int(rng.integers(1, 5))
        shape = tuple(int(x) for x in rng.integers(1, 5, r))
        base = np.arange(int(np.prod(shape)) * 3, dtype=np.float64)
        v = base.reshape(shape + (3,))[..., 0].transpose(rng.permutation(r))
        n, facs = v.size, []
        while n > 1:
            ds = [d for d in range(2, n + 1) if n % d == 0]
            facs.append(ds[int(rng.integers(0, len(ds)))])
            n //= facs[-1]
        new = tuple(facs) or (1,)
        got = view_strides(v.shape, tuple(s // 8 for s in v.strides), new)
        if got is None:
            w = v.view()
            with pytest.raises(AttributeError):
                w.shape = new          # NumPy cannot view it either
            continue
        w = np.lib.stride_tricks.as_strided(base, new, [g * 8 for g in got])
        np.testing.assert_array_equal(w, v.reshape(new))


def test_transformer_plan_matches_stored_reference_output():
    """The small transformer against the reference cpu target's stored logits."""
    z = np.load(Path(__file__).resolve().parent / "golden" / "sequence.npz")
    g = configs.transformer(2, **TINY_TF)
    cal = [configs.random_inputs(g, 100 + i) for i in range(2)]
    prog = compiler.compile_ir(g, "cuda", quantize="w8a8", calibration=cal, executor=FakeDevice())
    scales = np.array([op.attrs["x_scale"] for op in prog.graph.ops if op.kind == "qmatmul"])
    np.testing.assert_array_equal(scales, z["tf_x_scales"])
    np.testing.assert_allclose(prog.run({"tok": z["tf_tok"]}), z["tf_out"], rtol=1e-5, atol=1e-6)


def test_skinny_qmatmul_plans_split_k():
    """A quantized matmul with few output tiles and a long reduction gets a split-K workspace."""
    from mira_b200.hostfw import import_mira
    import_mira()
    from mira import ir
    from mira.types import TensorType as TT
    rng = np.random.default_rng(4)
    x = ir.Value(TT("f32", (4, 2048)), name="x")
    g = ir.Graph("skinny", [x], [], [])
    y = g.add("matmul", [x, g.const((rng.standard_normal((2048, 256)) * 0.02).astype(np.float32))], {})
    y = g.add("relu", [g.add("add", [y, g.const(rng.standard_normal(256).astype(np.float32))], {})], {})
    g.outputs = [y]
    g.verify()
    cal = [{"x": rng.standard_normal((4, 2048)).astype(np.float32)} for _ in range(2)]
    cpu = compiler.compile_ir(g, "cpu", quantize="w8a8", calibration=cal, precision=None)
    dev = FakeDevice()
    cuda = compiler.compile_ir(g, "cuda", quantize="w8a8", calibration=cal, executor=dev)
    launch = [l for l in cuda.segments[0].executable.plan.launches if l.kind == "qgemm"][0]
    assert launch.args.get("ws") is not None and launch.args["ws_bytes"] > 0
    feeds = {"x": rng.standard_normal((4, 2048)).astype(np.float32)}
    np.testing.assert_array_equal(cuda.run(feeds), cpu.run(feeds))


@pytest.mark.parametrize("name,batch,kw", [("mlp", 8, {}), ("resnet18", 2, {"image": 32})])
def test_run_many_matches_run_step_by_step(name, batch, kw):
    """run_many (input copies of the next step overlapped with the kernels of this one) returns
    what run() returns for each step, whether the inputs come in the executable's pinned arrays
    (the same array refilled between calls would race, so only fresh arrays are mixed in here) or
    as ordinary arrays."""
    cpu, cuda, _ = _pair(name, batch, **kw)
    exe = cuda.segments[0].executable
    x = exe.g.inputs[0]
    feeds = [{x: configs.random_inputs(cpu.graph, 10 + i)[x.name]} for i in range(5)]
    want = [exe.run({x: f[x].copy()})[exe.g.outputs[0]] for f in feeds]
    own = exe.input_array(x)          # run() staged every feed through this array: refill it last
    own[...] = feeds[2][x]
    feeds[2] = {x: own}
    got = exe.run_many(feeds)
    assert len(got) == 5
    for w, g_ in zip(want, got):
        np.testing.assert_array_equal(g_[exe.g.outputs[0]], w)


@pytest.mark.parametrize("quantize", [None, "int8"])
def test_f32_and_weight_only_cnn_plan_matches_cpu(quantize):
    """Ungrouped f32 convolutions (im2col + the f32 matmul, weight-only int8 weights kept int8) put a
    whole f32 or `quantize="int8"` ResNet-18 in one cuda segment; f32 tolerance against the cpu target
    (the reference's per-tap einsum sums in another order)."""
    g_cpu, g_cuda = configs.resnet18(2, image=32), configs.resnet18(2, image=32)
    cpu = compiler.compile_ir(g_cpu, "cpu", quantize=quantize, precision=None)
    dev = FakeDevice()
    cuda = compiler.compile_ir(g_cuda, "cuda", quantize=quantize, executor=dev)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    plan = cuda.segments[0].executable.plan
    convs = [l for l in plan.launches if l.kind == "im2col"]
    assert len(convs) == sum(op.kind == "conv2d" for op in cuda.graph.ops) == 20
    if quantize == "int8":
        assert all(l.args.get("b_scale") is not None for l in plan.launches if l.kind == "bmm")
    feeds = configs.random_inputs(cpu.graph, 1)
    want = cpu.run(feeds)
    got = cuda.run(feeds)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max())


def test_standalone_elementwise_ops_plan_matches_cpu():
    """With the reference's epilogue fusion off (fuse=False) every bias add, residual add and ReLU of
    an f32 ResNet-18 is a standalone op: strided element-wise launches over NHWC image values and
    broadcast constants, all in one cuda segment; f32 tolerance against the cpu target."""
    g_cpu, g_cuda = configs.resnet18(2, image=32), configs.resnet18(2, image=32)
    cpu = compiler.compile_ir(g_cpu, "cpu", fuse=False, precision=None)
    dev = FakeDevice()
    cuda = compiler.compile_ir(g_cuda, "cuda", fuse=False, executor=dev)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    kinds = [l.kind for l in cuda.segments[0].executable.plan.launches]
    assert kinds.count("elementwise") >= 40
    feeds = configs.random_inputs(cpu.graph, 1)
    want = cpu.run(feeds)
    np.testing.assert_allclose(cuda.run(feeds), want, rtol=1e-4, atol=1e-4 * np.abs(want).max())


def test_elementwise_graph_with_scalars_and_broadcasting_plan_matches_cpu():
    """Standalone ops on rank-3 values: a scalar on the left (2 - x), tensor-tensor broadcasting,
    division, the transcendental unaries; all on cuda."""
    from mira_b200.hostfw import import_mira
    import_mira()
    from mira import ir
    from mira.types import TensorType as TT

    def build():                      # compiling rewrites the graph: one per target
        x = ir.Value(TT("f32", (2, 3, 5)), name="x")
        y = ir.Value(TT("f32", (1, 3, 1)), name="y")
        g = ir.Graph("elt", [x, y], [], [])
        t = g.add("sub", [g.const(np.float32(2.0)), x], {})
        t = g.add("maximum", [t, y], {})
        t = g.add("div", [t, g.add("add", [g.add("sigmoid", [x], {}), g.const(np.float32(0.5))], {})], {})
        t = g.add("mul", [g.add("tanh", [t], {}), g.const(np.linspace(-1, 1, 5).astype(np.float32))], {})
        g.outputs = [g.add("gelu", [t], {})]
        return g

    feeds = {"x": np.random.default_rng(0).standard_normal((2, 3, 5)).astype(np.float32),
             "y": np.random.default_rng(1).standard_normal((1, 3, 1)).astype(np.float32)}
    cpu = compiler.compile_ir(build(), "cpu", fuse=False, precision=None)
    cuda = compiler.compile_ir(build(), "cuda", fuse=False, executor=FakeDevice(), cost_model=False)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    np.testing.assert_allclose(cuda.run(feeds), cpu.run(feeds), rtol=1e-6, atol=1e-6)
