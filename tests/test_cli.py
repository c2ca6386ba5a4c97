"""MIRA's own command line with the cuda target registered (`python -m mira_b200`, which is mira/cli.py
main): `run -t cuda --quantize w8a8` must save the same bytes as `run -t cpu --quantize w8a8`, `--check`
must pass against the f32 cpu program, and `bench --targets cpu,cuda` must report one row per target
with the same error against the f32 reference (cli.py:87-112, 202-231).  A program that ends in a
softmax agrees to a few ulp on the device (CUDA's expf against NumPy's exp).

The CPU tests run the cuda plan on the host-side stand-in device; the gpu tests run the CLI as a
subprocess on the real device, the way a user types it."""
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from fake_device import FakeDevice

ROOT = Path(__file__).resolve().parents[1]
PROGRAMS = sorted((Path(__file__).parent / "programs").glob("*.mira"))
TOL = "0.05"      # --check compares W8A8 against f32; these small nets lose up to ~2.5% to quantization


def _bench_rows(text):
    """{target: (rel err, segments)} from `mira bench` output."""
    rows = {}
    for line in text.splitlines():
        m = re.match(r"^(\S+)\s+[\d.]+s\s+[\d.]+ms\s+[\d.]+ms\s+(\S+)\s+(\S+)$", line)
        if m:
            rows[m.group(1)] = (m.group(2), m.group(3))
    return rows


@pytest.fixture
def cli(monkeypatch):
    import mira_b200.target as T
    from mira_b200.__main__ import main
    monkeypatch.setattr(T, "CudaDevice", lambda index: FakeDevice())
    return main


@pytest.mark.parametrize("prog", PROGRAMS, ids=lambda p: p.stem)
def test_cli_run_cuda_matches_cpu_w8a8(cli, prog, tmp_path, capsys):
    assert cli(["run", str(prog), "-t", "cpu", "--quantize", "w8a8", "--save", str(tmp_path / "cpu.npy")]) == 0
    assert cli(["run", str(prog), "-t", "cuda", "--quantize", "w8a8", "--check", "--tol", TOL,
                "--save", str(tmp_path / "cuda.npy")]) == 0
    out = capsys.readouterr().out
    assert "cuda:0 (B200, sm_100a)" in out and "PASS" in out
    np.testing.assert_array_equal(np.load(tmp_path / "cuda.npy"), np.load(tmp_path / "cpu.npy"))


def test_cli_bench_cpu_and_cuda(cli, capsys):
    prog = str(ROOT / "tests" / "programs" / "convnet.mira")
    assert cli(["bench", prog, "--quantize", "w8a8", "--targets", "cpu,cuda", "--iters", "2"]) == 0
    rows = _bench_rows(capsys.readouterr().out)
    assert set(rows) == {"cpu", "cuda"}
    assert rows["cuda"][1] == "cuda"
    assert rows["cuda"][0] == rows["cpu"][0]        # bit-identical outputs give the same error vs f32


def test_cli_lists_cuda_target(cli, capsys):
    with pytest.raises(SystemExit):
        cli(["run", "--help"])
    assert "cuda" in capsys.readouterr().out


def _run_cli(*args):
    env = dict(os.environ, PYTHONPATH=str(ROOT) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    return subprocess.run([sys.executable, "-m", "mira_b200", *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def _assert_same(prog, got, want):
    """Bit-identical, except after a softmax: its exp is CUDA's expf on the device against NumPy's
    float32 exp on the host (neither correctly rounded), so probabilities agree to a few ulp."""
    if "softmax" not in prog.read_text():
        np.testing.assert_array_equal(got, want)
        return
    assert got.shape == want.shape and got.dtype == want.dtype == np.float32
    ulps = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32))
    assert ulps.max() <= 8, int(ulps.max())


@pytest.mark.gpu
@pytest.mark.parametrize("prog", PROGRAMS, ids=lambda p: p.stem)
def test_gpu_cli_run_cuda_matches_cpu_w8a8(prog, tmp_path):
    r = _run_cli("run", str(prog), "-t", "cpu", "--quantize", "w8a8", "--save", str(tmp_path / "cpu.npy"))
    assert r.returncode == 0, r.stderr
    r = _run_cli("run", str(prog), "-t", "cuda", "--quantize", "w8a8", "--check", "--tol", TOL,
                 "--save", str(tmp_path / "cuda.npy"))
    assert r.returncode == 0, r.stdout + r.stderr
    assert "sm_100a" in r.stdout and "PASS" in r.stdout
    _assert_same(prog, np.load(tmp_path / "cuda.npy"), np.load(tmp_path / "cpu.npy"))


@pytest.mark.gpu
def test_gpu_cli_bench_cpu_and_cuda():
    prog = str(ROOT / "tests" / "programs" / "convnet.mira")
    r = _run_cli("bench", prog, "--quantize", "w8a8", "--targets", "cpu,cuda", "--iters", "5")
    assert r.returncode == 0, r.stdout + r.stderr
    rows = _bench_rows(r.stdout)
    assert set(rows) == {"cpu", "cuda"}, r.stdout
    assert rows["cuda"][1] == "cuda"
    # the program ends in a softmax (a few ulp apart): the printed errors agree to about 1e-6 relative
    assert float(rows["cuda"][0]) == pytest.approx(float(rows["cpu"][0]), rel=2e-2)
