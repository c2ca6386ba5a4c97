"""Parity at the benchmarked sizes: the programs `bench.py` times (ResNet-18 at batch 256 and 64,
MobileNetV2 at batch 256, 224 x 224, calibrated on 4 seeded batches of 8 images) against the
reference cpu target, bit for bit.

Every op of these networks is independent per image and the activation scales are calibration
constants, so a batch-1 cpu program compiled with the same calibration (`configs.compile_w8a8`
shares the calibration peaks between the two compiles) computes exactly image i's row of the large
program's output.  The reference takes about a second per ResNet-18 image on the host, so a spread of
images is compared: the first and last rows, the rows on both sides of the middle (where tile and
wave boundaries of the larger launches fall), and seeded random ones.  Oracle: the reference's
_qconv2d_ref / _qmatmul_ref (mira/ops.py:616-634) through CPUExecutable.run (mira/backends/cpu.py:28-36)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

mira_missing = False
try:
    from mira_b200 import configs
    from mira_b200.plugin import install
    install()
except ImportError:  # the host framework package is not on this machine
    mira_missing = True

needs_mira = pytest.mark.skipif(mira_missing, reason="MIRA host framework (package `mira`) not importable")

CALIB = dict(calib_batch=8, n_calib=4)     # bench.py's calibration for the image workloads


def _images(batch: int, n_random: int, seed: int) -> list[int]:
    fixed = {0, 1, batch // 2 - 1, batch // 2, batch - 2, batch - 1}
    rng = np.random.default_rng(seed)
    rest = [int(i) for i in rng.permutation(batch) if int(i) not in fixed][:n_random]
    return sorted(fixed) + sorted(rest)


def _x_scales(prog):
    return [op.attrs["x_scale"] for op in prog.graph.ops if op.kind in ("qconv2d", "qmatmul")]


_CPU = {}


def _cpu_program(name, **kw):
    key = (name, tuple(sorted(kw.items())))
    if key not in _CPU:
        _CPU[key] = configs.compile_w8a8(name, 1, "cpu", **CALIB, **kw)
    return _CPU[key]


def _check_rows(name: str, batch: int, n_random: int, seed: int, **kw):
    cpu = _cpu_program(name, **kw)
    cuda = configs.compile_w8a8(name, batch, "cuda", **CALIB, **kw)
    assert [s.device for s in cuda.segments] == ["cuda"], cuda.summary()
    assert _x_scales(cuda) == _x_scales(cpu), "the two compiles must share their activation scales"
    x = np.random.default_rng(seed).standard_normal((batch, 3, 224, 224), dtype=np.float32)
    runs = [cuda.run({"x": x}).copy() for _ in range(2)]     # eager, then a CUDA-graph replay
    assert np.array_equal(runs[0], runs[1])
    got = runs[1]
    idx = _images(batch, n_random, seed)
    bad = []
    for i in idx:
        want = cpu.run({"x": x[i:i + 1]})
        assert want.shape == (1, got.shape[1]) and want.dtype == got.dtype
        if not np.array_equal(got[i:i + 1], want):
            bad.append((i, int((got[i:i + 1] != want).sum())))
    print(f"{name} batch {batch} {kw}: {len(idx)} images compared bit for bit, mismatching images: {bad}")
    assert not bad, f"images with differing logits (image, values): {bad}"


@needs_mira
def test_resnet18_batch256_rows_bit_exact(cuda_device):
    """The headline program: ResNet-18 W8A8 at batch 256."""
    _check_rows("resnet18", 256, n_random=10, seed=11)


@needs_mira
def test_resnet18_batch64_rows_bit_exact(cuda_device):
    _check_rows("resnet18", 64, n_random=4, seed=12)


@needs_mira
def test_mobilenet_v2_batch256_rows_bit_exact(cuda_device):
    """MobileNetV2 W8A8 at batch 256: int8 convs, f32 depthwise, global mean."""
    _check_rows("mobilenet_v2", 256, n_random=26, seed=13)


@needs_mira
def test_mobilenet_v2_int8_depthwise_batch256_rows_bit_exact(cuda_device):
    """The opt-in int8 depthwise mode at the benchmarked size: both programs compiled inside
    mira_b200.int8_depthwise, the reference cpu target evaluating its grouped qconv2d itself."""
    _check_rows("mobilenet_v2", 256, n_random=6, seed=14, int8_depthwise=True)
