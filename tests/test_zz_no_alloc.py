"""mira_cuda_qgemm_splitk_static (split-K GEMM whose partial sums live in the library's fixed 8 MiB
scratch array) against mira_cuda_qgemm_splitk with a caller workspace: two calls in a row with
different inputs and shapes, bit for bit.  Kept in its own file, collected last, so it also runs
after every other GPU test in the same process."""
import ctypes as C

import numpy as np
import pytest

from oracle import w8a8 as ref

pytestmark = pytest.mark.gpu


def _case(K, DB, M, N, Kd, seed):
    rng = np.random.default_rng(seed)
    xq = rng.integers(-127, 128, (M, Kd)).astype(np.int8)
    q = rng.integers(-127, 128, (Kd, N)).astype(np.int8)
    x_scale = float(rng.uniform(0.005, 0.05))
    w_scale = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    lda = K.round_up(Kd, 16)
    a = np.zeros((M, lda), np.int8)
    a[:, :Kd] = xq
    bufs = dict(A=DB.from_array(a), B=DB.from_array(K.matmul_weight(q)), bias=DB.from_array(K.pad_channels(bias)))
    s64, hi, lo = K.scale_arrays(x_scale, w_scale)
    bufs.update(s64=DB.from_array(s64), hi=DB.from_array(hi), lo=DB.from_array(lo))
    want = ref.epilogue(ref.dequant(ref.int_matmul(xq, q), ref.combined_scale(x_scale, w_scale)), [bias],
                        [("add", 0, False), ("relu", None, False)]).astype(np.float32)
    out_scale = float(np.abs(want).max() / 127.0) or 1.0
    return bufs, lda, want, out_scale


def _run(K, DB, bufs, M, N, Kd, lda, out_scale, static):
    from mira_b200 import _lib
    y, yq = DB(M * N * 4), DB(M * K.round_up(N, 16), zero=True)
    dq = K.dequant_channel(bufs["s64"], bufs["hi"], bufs["lo"])
    epi = K.Epi([K.Step("add", "channel", ptr=bufs["bias"]), K.Step("relu")], out_f32=y, ld_f32=N, out_i8=yq,
                ld_i8=K.round_up(N, 16), out_scale=out_scale).struct()
    if static:
        _lib.call("mira_cuda_qgemm_splitk_static", M, N, Kd, C.c_void_p(bufs["A"].ptr), lda, C.c_void_p(bufs["B"].ptr),
                  lda, C.byref(dq), C.byref(epi))
    else:
        nbytes = K.qgemm_workspace(M, N, Kd)
        ws = DB(max(nbytes, 16))
        _lib.call("mira_cuda_qgemm_splitk", M, N, Kd, C.c_void_p(bufs["A"].ptr), lda, C.c_void_p(bufs["B"].ptr), lda,
                  C.byref(dq), C.byref(epi), C.c_void_p(ws.ptr), nbytes)
    _lib.call("mira_cuda_sync")
    return y.download((M, N), np.float32), yq.download((M, K.round_up(N, 16)), np.int8)


def test_static_scratch_splitk_matches_workspace_splitk_twice_in_a_row(cuda_device):
    from mira_b200 import kernels as K
    from mira_b200.device import DeviceBuffer as DB
    # two different shapes back to back: the second call must not see anything of the first
    for M, N, Kd, seed in ((16, 4096, 4096, 1), (3, 1000, 2048, 2)):
        assert 0 < K.qgemm_workspace(M, N, Kd) <= 8 << 20
        bufs, lda, want, out_scale = _case(K, DB, M, N, Kd, seed)
        got_s, q_s = _run(K, DB, bufs, M, N, Kd, lda, out_scale, static=True)
        got_w, q_w = _run(K, DB, bufs, M, N, Kd, lda, out_scale, static=False)
        assert np.array_equal(got_s.view(np.uint32), got_w.view(np.uint32))
        np.testing.assert_array_equal(q_s, q_w)
        assert np.array_equal(got_s.view(np.uint32), want.view(np.uint32))


def test_static_scratch_call_leaves_free_device_memory_unchanged(cuda_device):
    """The property these callers need: after the first call on a device (which looks up the scratch
    array's address), a call takes no device memory, so the device's free bytes stay the same."""
    import torch
    from mira_b200 import kernels as K
    from mira_b200.device import DeviceBuffer as DB
    M, N, Kd = 16, 4096, 4096
    bufs, lda, _, out_scale = _case(K, DB, M, N, Kd, 4)
    y, yq = DB(M * N * 4), DB(M * K.round_up(N, 16), zero=True)
    dq = K.dequant_channel(bufs["s64"], bufs["hi"], bufs["lo"])
    epi = K.Epi([K.Step("add", "channel", ptr=bufs["bias"]), K.Step("relu")], out_f32=y, ld_f32=N, out_i8=yq,
                ld_i8=K.round_up(N, 16), out_scale=out_scale).struct()
    from mira_b200 import _lib

    def call():
        _lib.call("mira_cuda_qgemm_splitk_static", M, N, Kd, C.c_void_p(bufs["A"].ptr), lda, C.c_void_p(bufs["B"].ptr),
                  lda, C.byref(dq), C.byref(epi))
        _lib.call("mira_cuda_sync")

    call()
    free0 = torch.cuda.mem_get_info(cuda_device)[0]
    for _ in range(3):
        call()
    assert torch.cuda.mem_get_info(cuda_device)[0] == free0


def test_static_scratch_rejects_shapes_beyond_its_size(cuda_device):
    from mira_b200 import _lib
    from mira_b200 import kernels as K
    from mira_b200.device import DeviceBuffer as DB
    M, N, Kd = 256, 1024, 8192           # 16 K ranges x 256 x 1024 int32 = 16 MiB of partial sums
    assert K.qgemm_workspace(M, N, Kd) > 8 << 20
    bufs, lda, _, out_scale = _case(K, DB, M, N, Kd, 3)
    with pytest.raises(_lib.CudaError) as e:
        _run(K, DB, bufs, M, N, Kd, lda, out_scale, static=True)
    assert e.value.code == _lib.EINVAL and "8 MiB" in str(e.value)
