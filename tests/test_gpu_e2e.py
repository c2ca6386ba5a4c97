"""End-to-end parity on the GPU: MIRA programs compiled W8A8 for the `cuda` target against the same
programs on the reference `cpu` target (MIRA's NumPy golden model), identical seeded inputs and
calibration.  The outputs must be bit-identical (tolerance 0): every op on these paths is exact on
the device (see the per-kernel tests), including the global mean (NumPy's summation order)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

mira_missing = False
try:
    from mira_b200 import configs
    from mira_b200.plugin import install
    mira = install()
    from mira import compiler
except ImportError:  # the host framework package is not on this machine
    mira_missing = True

needs_mira = pytest.mark.skipif(mira_missing, reason="MIRA host framework (package `mira`) not importable")


def _pair(name, batch, n_calib=2, fuse_pool=False, **kw):
    g_cpu = configs.BUILDERS[name](batch, **kw)
    g_cuda = configs.BUILDERS[name](batch, **kw)
    cal = [configs.random_inputs(g_cpu, 100 + i) for i in range(n_calib)]
    cpu = compiler.compile_ir(g_cpu, "cpu", quantize="w8a8", calibration=cal, precision=None)
    cuda = compiler.compile_ir(g_cuda, "cuda", quantize="w8a8", calibration=cal, fuse_pool=fuse_pool)
    return cpu, cuda


def _assert_same(cpu, cuda, seeds=(1, 2)):
    for s in seeds:
        feeds = configs.random_inputs(cpu.graph, s)
        want = cpu.run(feeds)
        for _ in range(2):              # eager first run, then CUDA-graph replays
            got = cuda.run(feeds)
            assert got.dtype == want.dtype and got.shape == want.shape
            bad = got != want
            assert not bad.any(), f"{int(bad.sum())} of {bad.size} outputs differ (max |d| {np.abs(got - want).max()})"


@needs_mira
def test_config1_mlp_batch256_bit_exact(cuda_device):
    """Config 1: x[256, 784], 784-512-512-10, 8 calibration batches."""
    cpu, cuda = _pair("mlp", 256, n_calib=8)
    assert [s.device for s in cuda.segments] == ["cuda"]
    _assert_same(cpu, cuda)


@needs_mira
@pytest.mark.parametrize("batch,image", [(2, 64), (1, 224)])
def test_resnet18_bit_exact(cuda_device, batch, image):
    cpu, cuda = _pair("resnet18", batch, image=image)
    assert [s.device for s in cuda.segments] == ["cuda"]
    _assert_same(cpu, cuda, seeds=(1,))


@needs_mira
def test_resnet18_fused_stem_pool_bit_exact(cuda_device):
    cpu, cuda = _pair("resnet18", 2, fuse_pool=True, image=64)
    _assert_same(cpu, cuda, seeds=(1,))


@needs_mira
@pytest.mark.parametrize("batch,image", [(2, 64), (1, 224)])
def test_mobilenet_v2_bit_exact(cuda_device, batch, image):
    cpu, cuda = _pair("mobilenet_v2", batch, image=image)
    assert [s.device for s in cuda.segments] == ["cuda"]
    _assert_same(cpu, cuda, seeds=(1,))


CNN_SRC = """
fn block(x: f32[N, C, H, W], k: f32[O, C, 3, 3], b: f32[O, 1, 1]) -> f32[N, O, H / 2, W / 2] {
  return maxpool2d(relu(conv2d(x, k, padding=1) + b), size=2)
}

fn main(img: f32[16, 1, 28, 28],
        const k1: f32[16, 1, 3, 3],  const c1: f32[16, 1, 1],
        const k2: f32[32, 16, 3, 3], const c2: f32[32, 1, 1],
        const wf: f32[1568, 10],     const bf: f32[10]) -> f32[16, 10] {
  let h = block(block(img, k1, c1), k2, c2)
  return softmax(flatten(h) @ wf + bf)
}
"""


@needs_mira
def test_mira_source_cnn_matches_cpu(cuda_device):
    """A .mira CNN through compile_source: convs, pools, the flatten, the FC and the final softmax
    all on cuda.  Everything up to the softmax is exact; the softmax's exp is CUDA's expf against
    NumPy's float32 exp (neither is correctly rounded), so the probabilities agree to a few ulp."""
    rng = np.random.default_rng(0)
    cal = [{"img": rng.standard_normal((16, 1, 28, 28)).astype(np.float32)} for _ in range(2)]
    cpu = mira.compile_source(CNN_SRC, "cpu", quantize="w8a8", calibration=cal, precision=None)
    cuda = mira.compile_source(CNN_SRC, "cuda", quantize="w8a8", calibration=cal)
    feeds = {"img": rng.standard_normal((16, 1, 28, 28)).astype(np.float32)}
    got, want = cuda.run(feeds), cpu.run(feeds)
    ulps = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32))
    assert ulps.max() <= 8, int(ulps.max())
    assert [s.device for s in cuda.segments] == ["cuda"]


@needs_mira
def test_w8a8_accuracy_against_f32_like_reference_test(cuda_device):
    """Reference tests/test_control_dynamic_quant.py:205-213 applied to the cuda target: W8A8 logits
    agree with the unquantized f32 cpu program in argmax >= 0.9 and max error < 0.1 max|ref|."""
    g32 = configs.mlp(64)
    feeds = {"x": np.random.default_rng(0).standard_normal((64, 784)).astype(np.float32)}
    ref = compiler.compile_ir(g32, "cpu", precision=None).run(feeds)
    cal = [configs.random_inputs(configs.mlp(64), 100 + i) for i in range(4)]
    got = compiler.compile_ir(configs.mlp(64), "cuda", quantize="w8a8", calibration=cal).run(feeds)
    assert (got.argmax(1) == ref.argmax(1)).mean() >= 0.9
    assert np.abs(got - ref).max() < 0.1 * np.abs(ref).max()


@needs_mira
def test_run_many_overlapped_copies_bit_exact(cuda_device):
    """run_many (each step's input copy on the copy stream overlapping the previous step's kernels,
    a second device input buffer, a two-slot output ring) against the reference cpu target step by
    step, with the executable's own pinned input array and with ordinary arrays."""
    cpu, cuda = _pair("resnet18", 4, image=64)
    exe = cuda.segments[0].executable
    x = exe.g.inputs[0]
    feeds = [configs.random_inputs(cpu.graph, 20 + i) for i in range(6)]
    want = [cpu.run(f) for f in feeds]
    own = exe.input_array(x)
    own[...] = feeds[3]["x"]
    steps = [{x: own} if i == 3 else {x: f["x"]} for i, f in enumerate(feeds)]
    for _ in range(2):                  # the first call captures the CUDA graph on its second step
        got = exe.run_many(steps)
        for w, g_ in zip(want, got):
            out = g_[exe.g.outputs[0]]
            assert out.shape == w.shape and not (out != w).any()


@needs_mira
@pytest.mark.parametrize("quantize", [None, "int8"])
def test_f32_and_weight_only_resnet18_close_to_cpu(cuda_device, quantize):
    """f32 (no quantization) and weight-only int8 ResNet-18: ungrouped convolutions through im2col and
    the f32 matmul, all on the device; f32 tolerance against the reference cpu target."""
    g_cpu, g_cuda = configs.resnet18(2, image=64), configs.resnet18(2, image=64)
    cpu = compiler.compile_ir(g_cpu, "cpu", quantize=quantize, precision=None)
    cuda = compiler.compile_ir(g_cuda, "cuda", quantize=quantize)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    feeds = configs.random_inputs(g_cpu, 1)
    want = cpu.run(feeds)
    for _ in range(2):
        got = cuda.run(feeds)
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max())


@needs_mira
def test_unfused_f32_resnet18_close_to_cpu(cuda_device):
    """fuse=False: every bias add, residual add and ReLU a standalone element-wise launch over NHWC
    image values; f32 tolerance against the reference cpu target."""
    g_cpu, g_cuda = configs.resnet18(2, image=64), configs.resnet18(2, image=64)
    cpu = compiler.compile_ir(g_cpu, "cpu", fuse=False, precision=None)
    cuda = compiler.compile_ir(g_cuda, "cuda", fuse=False)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    feeds = configs.random_inputs(g_cpu, 1)
    want = cpu.run(feeds)
    np.testing.assert_allclose(cuda.run(feeds), want, rtol=1e-4, atol=1e-4 * np.abs(want).max())
