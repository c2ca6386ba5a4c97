"""The cuda target against the reference's own stored outputs (tests/golden/programs.npz, written by
running myramay/MIRA's cpu W8A8 path), plus the device-side failure path of the bounded waits."""
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"

try:
    from mira_b200 import configs
    from mira_b200.plugin import install
    install()
    from mira import compiler
    HAVE_MIRA = True
except ImportError:
    HAVE_MIRA = False


@pytest.mark.skipif(not HAVE_MIRA, reason="MIRA host framework (package `mira`) not importable")
@pytest.mark.parametrize("name", ["mlp", "resnet18", "mobilenet_v2"])
def test_program_matches_stored_reference_output(cuda_device, name):
    z = np.load(GOLDEN / "programs.npz")
    batch, image, n_cal = int(z[f"{name}_batch"]), int(z[f"{name}_image"]), int(z[f"{name}_n_calib"])
    kw = {"image": image} if image else {}
    g = configs.BUILDERS[name](batch, **kw)
    cal = [configs.random_inputs(g, 100 + i) for i in range(n_cal)]
    prog = compiler.compile_ir(g, "cuda", quantize="w8a8", calibration=cal)
    scales = np.array([op.attrs["x_scale"] for op in prog.graph.ops if op.kind in ("qmatmul", "qconv2d")])
    np.testing.assert_array_equal(scales, z[f"{name}_x_scales"])
    got = prog.run({"x": z[f"{name}_x"]})
    np.testing.assert_array_equal(got, z[f"{name}_out"])


def test_expired_bounded_wait_is_reported_and_device_stays_usable(cuda_device):
    """A kernel whose barrier never completes gives up after its bound, records an error that
    mira_cuda_sync turns into MIRA_CUDA_EKERNEL, and the device keeps working afterwards."""
    from mira_b200 import _lib
    from mira_b200 import kernels as K
    from mira_b200.device import DeviceBuffer
    _lib.call("mira_cuda_selftest_wait_timeout", 20000)
    with pytest.raises(_lib.CudaError) as e:
        _lib.call("mira_cuda_sync")
    assert e.value.code == _lib.EKERNEL
    _lib.call("mira_cuda_sync")   # the record was cleared
    x = DeviceBuffer.from_array(np.arange(32, dtype=np.float32))
    q = DeviceBuffer(32)
    K.quantize_rows(x, 1, 32, 32, 0.25, q, 32)
    np.testing.assert_array_equal(q.download((32,), np.int8), np.clip(np.round(np.arange(32) / 0.25), -127, 127))
