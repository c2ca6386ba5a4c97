#!/usr/bin/env python
"""Benchmark of the W8A8 hot path on B200: ResNet-18 W8A8 images/s (batch 256 per GPU, weak
scaling over 1/2/4/8 GPUs, one process per GPU) plus the int8 GEMM throughput at 8192^3.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]
                  [--workload resnet18|mobilenet_v2|mlp|transformer|decode]

The default workload is the headline (ResNet-18); the others are the remaining configurations of
the same path (MobileNetV2 images/s, the MLP's samples/s, the transformer prefill's tokens/s) with
the same JSON line.

A step is one forward pass of a batch through the compiled MIRA program.  `value` times K steps
on device-resident inputs (CUDA events on the library stream, max over ranks); `e2e` times the
same K steps through the public API (`CompiledProgram.run` with pinned host inputs: host->device
copy of the batch, the kernels, device->host copy of the logits).  `--impl reference` times the
reference's own cpu W8A8 path (MIRA's NumPy golden model) on a bounded sample.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# name -> metric, unit, config name, default batch, calibration (batch, count), items per batch row,
# and the bounded sample the reference cpu path is timed on (builder options, batch, and the factor
# that scales its rate to the full network: the transformer sample runs 1 of the 12 layers)
WORKLOADS = {
    "resnet18": dict(metric="w8a8 ResNet-18 img/s", unit="img/s", config="resnet18-w8a8-224", batch=256,
                     calib_batch=8, n_calib=4, items_per_row=1, build_kw={}, cpu_batch=1, cpu_build_kw={},
                     cpu_scale=1.0, cpu_note="one image per step"),
    "mobilenet_v2": dict(metric="w8a8 MobileNetV2 img/s", unit="img/s", config="mobilenet_v2-w8a8-224", batch=256,
                         calib_batch=8, n_calib=4, items_per_row=1, build_kw={}, cpu_batch=1, cpu_build_kw={},
                         cpu_scale=1.0, cpu_note="one image per step"),
    "mlp": dict(metric="w8a8 MLP samples/s", unit="samples/s", config="mlp-784-512-512-10", batch=256,
                calib_batch=256, n_calib=8, items_per_row=1, build_kw={}, cpu_batch=256, cpu_build_kw={},
                cpu_scale=1.0, cpu_note="one batch of 256 per step"),
    "transformer": dict(metric="w8a8 transformer prefill tokens/s", unit="tokens/s",
                        config="decoder-12x768-h12-mlp3072-vocab256-seq1024", batch=64, calib_batch=1, n_calib=4,
                        items_per_row=1024, build_kw={}, cpu_batch=1, cpu_build_kw=dict(layers=1, seq=128),
                        cpu_scale=1.0 / 12,
                        cpu_note="one sequence of 128 tokens through 1 of the 12 layers per step; tokens/s "
                                 "divided by 12 (layers; attention cost per token grows with the sequence, so "
                                 "this overestimates the reference at 1024)"),
}
WORKLOAD = "resnet18"
METRIC = WORKLOADS[WORKLOAD]["metric"]

# config-5 decode: one new token for each of `batch` sequences per step, key/value caches of max_seq
# positions resident on the device (mira_b200.decode); the reference cpu sample runs the same
# quantized step graph at batch 1
DECODE = dict(metric="w8a8 transformer decode tokens/s", unit="tokens/s",
              config="decoder-12x768-h12-mlp3072-vocab256-kv1024-step", batch=64, max_seq=1024, vocab=256)


def _env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops"), d.get("hbm_gbs"), "MEASURED_PEAKS.json"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region: NVML read every 5 ms from a
    thread (read-only queries, so regions of a few ms still get samples), else nvidia-smi every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []
        self.nvml_samples: list[tuple[float, int]] = []
        self.nvml_max = None
        self._stop = None

    def _poll_nvml(self, nv, h):
        while True:
            try:
                self.nvml_samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                          int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
            except Exception:
                return
            if self._stop.wait(0.005):
                return

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.nvml_max = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._nv = nv
            self._stop = threading.Event()
            self.t = threading.Thread(target=self._poll_nvml, args=(nv, h), daemon=True)
            self.t.start()
            return self
        except Exception:
            self._stop = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self.t.join(timeout=5)
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self._stop is not None:
            nv = self._nv
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            sm = [c for c, _ in self.nvml_samples]
            if not sm:
                return {"sm_mhz": None, "sm_max_mhz": self.nvml_max, "reasons": [], "samples": 0, "source": "nvml"}
            reasons = sorted(n for n, b in bits.items() if any(r & b for _, r in self.nvml_samples))
            under_load = [c for c in sm if c > 0.3 * (self.nvml_max or 1)] or sm
            return {"sm_mhz": statistics.median(under_load), "sm_max_mhz": self.nvml_max, "reasons": reasons,
                    "samples": len(sm), "source": "nvml, every 5 ms"}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        under_load = [s for s in sm if s > 0.3 * (mx or 1)] or sm
        return {"sm_mhz": statistics.median(under_load), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def conv_work(graph) -> tuple[int, int]:
    """(int8 ops of the convolutions, int8 ops of all quantized ops) per batch of the compiled graph."""
    conv = total = 0
    for op in graph.ops:
        if op.kind == "qconv2d":
            o, c, kh, kw = op.attrs["q"].shape
            n, _, oh, ow = op.result.type.shape
            w = 2 * n * oh * ow * o * c * kh * kw
            conv += w
            total += w
        elif op.kind == "qmatmul":
            k, nn = op.attrs["q"].shape
            m = int(np.prod(op.inputs[0].type.shape[:-1]))
            total += 2 * m * k * nn
    return conv, total


def time_kernels(exe, kinds, iters: int = 3) -> tuple[float, int]:
    """(average summed duration in ms, count) of the plan's launches of the given kinds, each
    bracketed by CUDA events on the library stream (one event pair per launch, eager launches)."""
    from mira_b200 import _lib
    idx = [i for i, l in enumerate(exe.plan.launches) if l.kind in kinds]
    if not idx:
        return 0.0, 0

    def ev():
        p = C.c_void_p()
        _lib.call("mira_cuda_event_create", C.byref(p))
        return p

    pairs = [(ev(), ev()) for _ in idx]
    total = 0.0
    for _ in range(iters):
        j = 0
        for i, t in enumerate(exe.thunks):
            if j < len(idx) and idx[j] == i:
                _lib.call("mira_cuda_event_record", pairs[j][0])
                t()
                _lib.call("mira_cuda_event_record", pairs[j][1])
                j += 1
            else:
                t()
        for a, b in pairs:
            ms = C.c_float()
            _lib.call("mira_cuda_event_elapsed", a, b, C.byref(ms))
            total += ms.value
    for a, b in pairs:
        _lib.call("mira_cuda_event_destroy", a)
        _lib.call("mira_cuda_event_destroy", b)
    return total / iters, len(idx)


GEMM_SQUARE = (1024, 2048, 4096, 8192, 16384)
GEMM_SKINNY = (1, 16, 128)
GEMM_ITERS = 50
ROTATE_BYTES = 320e6     # operands + output cycled between timed GEMMs: more than twice the 126 MB L2


def gemm_operands(m: int, n: int, k: int, seed: int):
    """Config 2's operands: A int8 [m, k] and B int8 [n, k] (K-major, the transposed [k, n] weight)
    uniform in [-127, 127], row and column scales f32 U(1e-3, 1e-2), bias f32 N(0, 1)."""
    rng = np.random.default_rng(seed)
    return (rng.integers(-127, 128, (m, k), dtype=np.int8), rng.integers(-127, 128, (n, k), dtype=np.int8),
            rng.uniform(1e-3, 1e-2, m).astype(np.float32), rng.uniform(1e-3, 1e-2, n).astype(np.float32),
            rng.standard_normal(n).astype(np.float32))


def _rotation(m: int, n: int, k: int) -> int:
    """Operand sets to cycle through so consecutive timed GEMMs never find their inputs in L2."""
    return max(1, int(np.ceil(ROTATE_BYTES / (m * k + n * k + 4 * m * n))))


def _graph_us(fns, iters: int) -> float:
    """Device time per call of `iters` calls cycling over fns: captured into one CUDA graph on the
    library stream, replayed once untimed, then once between CUDA events."""
    from mira_b200 import _lib
    for f in fns:
        f()
    _lib.call("mira_cuda_sync")
    _lib.call("mira_cuda_graph_begin")
    try:
        for i in range(iters):
            fns[i % len(fns)]()
    finally:
        g = C.c_void_p()
        _lib.call("mira_cuda_graph_end", C.byref(g))
    try:
        _lib.call("mira_cuda_graph_launch", g)
        _lib.call("mira_cuda_sync")
        a, b = C.c_void_p(), C.c_void_p()
        _lib.call("mira_cuda_event_create", C.byref(a))
        _lib.call("mira_cuda_event_create", C.byref(b))
        _lib.call("mira_cuda_event_record", a)
        _lib.call("mira_cuda_graph_launch", g)
        _lib.call("mira_cuda_event_record", b)
        _lib.call("mira_cuda_sync")
        ms = C.c_float()
        _lib.call("mira_cuda_event_elapsed", a, b, C.byref(ms))
        _lib.call("mira_cuda_event_destroy", a)
        _lib.call("mira_cuda_event_destroy", b)
    finally:
        _lib.call("mira_cuda_graph_destroy", g)
    return ms.value / iters * 1e3


def _ours_gemm(m: int, n: int, k: int, seed: int, splitk: bool):
    """Device buffers and launch closures of mira_cuda_qgemm (or _splitk) on config-2 operand sets."""
    from mira_b200 import _lib, kernels as K
    from mira_b200.device import DeviceBuffer as DB
    keep, fns = [], []
    lib = _lib.load()
    for s in range(_rotation(m, n, k)):
        A, B, rs, cs, bias = gemm_operands(m, n, k, seed + s)
        bufs = [DB.from_array(A), DB.from_array(B), DB.from_array(rs), DB.from_array(cs),
                DB.from_array(K.pad_channels(bias)), DB(m * n * 4)]
        dq = K.dequant_rowcol(bufs[2], bufs[3])
        e = K.Epi([K.Step("add", "channel", ptr=bufs[4])], out_f32=bufs[5], ld_f32=n).struct()
        keep += bufs + [dq, e]
        if splitk:
            ws_bytes = K.qgemm_workspace(m, n, k)
            ws = DB(max(ws_bytes, 16))
            keep.append(ws)
            args = (m, n, k, C.c_void_p(bufs[0].ptr), k, C.c_void_p(bufs[1].ptr), k, C.byref(dq), C.byref(e),
                    C.c_void_p(ws.ptr), ws_bytes)
            fn = lib.mira_cuda_qgemm_splitk
        else:
            args = (m, n, k, C.c_void_p(bufs[0].ptr), k, C.c_void_p(bufs[1].ptr), k, C.byref(dq), C.byref(e))
            fn = lib.mira_cuda_qgemm

        def call(fn=fn, args=args):
            rc = fn(*args)
            if rc != _lib.OK:
                raise _lib.CudaError(rc, _lib.last_error())
        fns.append(call)
    return keep, fns


def cublaslt_us(m: int, n: int, k: int, seed: int, iters: int = GEMM_ITERS) -> float | None:
    """torch._int_mm (cuBLASLt int8 x int8 -> int32) on the same operand sets and rotation, for
    context: device time per call of `iters` calls replayed from a CUDA graph."""
    try:
        import torch
        sets = []
        for s in range(_rotation(m, n, k)):
            A, B, *_ = gemm_operands(m, n, k, seed + s)
            sets.append((torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda().t()))
        for a, b in sets:
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(iters):
                a, b = sets[i % len(sets)]
                torch._int_mm(a, b)
        g.replay()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        g.replay()
        s1.record()
        torch.cuda.synchronize()
        us = s0.elapsed_time(s1) / iters * 1e3
        del g, sets
        torch.cuda.empty_cache()
        return us
    except Exception:
        return None


def gemm_sweep(peak_tops: float | None) -> dict:
    """Config 2 (the int8 GEMM sweep) through mira_cuda_qgemm: square M = N = K in GEMM_SQUARE and
    skinny M x 4096 x 4096 (split-K), row x column scales + bias, f32 out; operands per config 2,
    cycled so no timed GEMM finds its inputs in L2; GEMM_ITERS calls replayed from a CUDA graph.
    cuBLASLt's int8 GEMM (int32 out, no epilogue) on the same data beside each square size."""
    square = {}
    for n in GEMM_SQUARE:
        keep, fns = _ours_gemm(n, n, n, 1000 + n, splitk=False)
        us = _graph_us(fns, GEMM_ITERS)
        del keep, fns
        tops = 2.0 * n ** 3 / (us * 1e-6) / 1e12
        lt = cublaslt_us(n, n, n, 1000 + n)
        lt_tops = 2.0 * n ** 3 / (lt * 1e-6) / 1e12 if lt else None
        square[str(n)] = {"us": us, "tops": tops, "frac_of_2x_bf16": tops / peak_tops if peak_tops else None,
                          "cublaslt_tops": lt_tops, "frac_of_cublaslt": tops / lt_tops if lt_tops else None,
                          "operand_sets": _rotation(n, n, n)}
    skinny = {}
    for m in GEMM_SKINNY:
        n = k = 4096
        keep, fns = _ours_gemm(m, n, k, 2000 + m, splitk=True)
        us = _graph_us(fns, GEMM_ITERS)
        del keep, fns
        nbytes = m * k + k * n + 4 * m * n + 4 * (m + 2 * n)
        skinny[str(m)] = {"us": us, "gb_s": nbytes / (us * 1e-6) / 1e9, "algorithmic_bytes": nbytes}
    return {"square": square, "skinny_mx4096x4096": skinny, "iters": GEMM_ITERS,
            "data": "config 2: A, B int8 uniform [-127, 127], row/col scales U(1e-3, 1e-2), bias N(0, 1), "
                    "seeded; operand sets cycled (more than twice L2 between reuses)"}


PROFILE_CASES = ("gemm8192", "conv_l1", "conv_l1_cp", "dwconv_l1", "qdwconv_l1", "attention_q1", "quantize_rows", "stem", "stem_pool",
                 "maxpool_stem",
                 "decode_step", "attention_prefill", "layernorm_decode", "layernorm_prefill")


def profile_case(name: str, reps: int = 3, timed: bool = False) -> None:
    """One kernel on a bounded, seeded case, launched `reps` times, for ncu captures (the inputs are
    larger than L2 where the kernel is HBM-bound; a few hundred MB on the device):
      gemm8192      mira_cuda_qgemm 8192^3 on config-2 operands, row/col scales + bias, f32 out
      conv_l1       ResNet-18 layer-1 3x3 conv, batch 256, 56x56x64 -> 64, bias + relu, int8 + f32 out
      conv_l1_cp    the same conv reading and writing int8 in the chunk-planar layout (MIRA_LAYOUT_CP)
      dwconv_l1     MobileNetV2's first depthwise layer, batch 96, 112x112x32, bias + relu6, int8 out
      qdwconv_l1    the same layer in the opt-in int8 depthwise mode (int8 in, exact sums), int8 out
      attention_q1  a decode step's attention: 64 sequences x 12 heads, 1024 cached rows, d_head 64
      quantize_rows the transformer's activation quantization, 65536 x 768 f32 -> int8
      stem          ResNet-18's stem: NCHW f32 64 x 3 x 224 x 224 quantized into the row-expanded layout,
                    then the 7x7/2 conv to 64 channels, bias + relu, f32 out (205 MB)
      stem_pool     ResNet-18's stem conv fused with its max pool (one kernel), 64 images, pooled f32 and
                    chunk-planar int8 out
      maxpool_stem  ResNet-18's -inf pad + 3x3/2 max pool on the stem output, 64 x 112 x 112 x 64 f32,
                    f32 and int8 out
      decode_step   `reps` eager steps of the config-5 decode (batch 64, 1024-row caches): every
                    launch of a step, for a launch list
      attention_prefill  the prefill's fused attention: 8 sequences x 12 heads x 1024 tokens, d_head 64,
                    causal mask with exact tile skipping (tensor-core kernel and its piece pass;
                    MIRA_CUDA_ATTENTION=simt selects the f32 FMA kernel)
      layernorm_decode  a decode step's layernorm: 64 rows x 768, f32 and int8 out
      layernorm_prefill a prefill layernorm: 65536 rows x 768 (201 MB), int8 out"""
    from mira_b200 import _lib, kernels as K
    from mira_b200.device import DeviceBuffer as DB
    rng = np.random.default_rng(0)
    if name == "gemm8192":
        n = 8192
        a, b, r, c, bi = gemm_operands(n, n, n, 1000 + n)
        A, B, Y = DB.from_array(a), DB.from_array(b), DB(n * n * 4)
        rs, cs = DB.from_array(r), DB.from_array(c)
        bias = DB.from_array(K.pad_channels(bi))
        epi = K.Epi([K.Step("add", "channel", ptr=bias)], out_f32=Y, ld_f32=n)
        for _ in range(reps):
            K.qgemm(n, n, n, A, n, B, n, K.dequant_rowcol(rs, cs), epi)
    elif name == "conv_l1":
        n, h, c, o = 256, 56, 64, 64
        x = DB.from_array(rng.integers(-127, 128, (n, h, h, c)).astype(np.int8))
        wq, cp = K.conv_weight(rng.integers(-127, 128, (o, c, 3, 3)).astype(np.int8))
        s64, hi, lo = K.scale_arrays(0.02, rng.uniform(1e-3, 1e-2, o).astype(np.float32))
        keep = [DB.from_array(a) for a in (s64, hi, lo)]
        bias = DB.from_array(K.pad_channels(rng.standard_normal(o).astype(np.float32)))
        y, yq = DB(n * h * h * o * 4), DB(n * h * h * o)
        epi = K.Epi([K.Step("add", "channel", ptr=bias), K.Step("relu")], out_f32=y, ld_f32=o, out_i8=yq, ld_i8=o,
                    out_scale=0.05)
        wb = DB.from_array(wq)
        for _ in range(reps):
            K.qconv2d(n, h, h, cp, x, o, 3, 3, wb, wq.shape[1], (1, 1), (1, 1), (1, 1), K.dequant_channel(*keep), epi,
                      layout=0)
    elif name == "conv_l1_cp":
        n, h, c, o = 256, 56, 64, 64
        xq = rng.integers(-127, 128, (n, h, h, c)).astype(np.int8)
        x = DB.from_array(K.to_cp(xq))
        wq, cp = K.conv_weight(rng.integers(-127, 128, (o, c, 3, 3)).astype(np.int8))
        s64, hi, lo = K.scale_arrays(0.02, rng.uniform(1e-3, 1e-2, o).astype(np.float32))
        keep = [DB.from_array(a) for a in (s64, hi, lo)]
        bias = DB.from_array(K.pad_channels(rng.standard_normal(o).astype(np.float32)))
        y, yq = DB(n * h * h * o * 4), DB(K.cp_bytes(n, h, h, o), zero=True)
        epi = K.Epi([K.Step("add", "channel", ptr=bias), K.Step("relu")], out_f32=y, ld_f32=o, out_i8=yq, ld_i8=o,
                    out_scale=0.05, i8_layout=_lib.LAYOUT_CP)
        wb = DB.from_array(wq)
        for _ in range(reps):
            K.qconv2d(n, h, h, cp, x, o, 3, 3, wb, wq.shape[1], (1, 1), (1, 1), (1, 1), K.dequant_channel(*keep), epi,
                      layout=_lib.LAYOUT_CP)
    elif name == "dwconv_l1":
        n, h, c = 96, 112, 32
        x = DB.from_array(rng.standard_normal((n, h, h, c), dtype=np.float32))
        wt = DB.from_array(rng.standard_normal((9, c)).astype(np.float32))
        bias = DB.from_array(K.pad_channels(rng.standard_normal(c).astype(np.float32)))
        q = DB(n * h * h * K.round_up(c, 16))
        epi = K.Epi([K.Step("add", "channel", ptr=bias), K.Step("maximum", "scalar", scalar=0.0),
                     K.Step("minimum", "scalar", scalar=6.0)], out_i8=q, ld_i8=K.round_up(c, 16), out_scale=6.0 / 127)
        for _ in range(reps):
            K.dwconv2d(x, n, h, h, c, wt, 3, 3, (1, 1), (1, 1), (1, 1), epi)
    elif name == "qdwconv_l1":
        n, h, c = 96, 112, 32
        x = DB.from_array(rng.integers(-127, 128, (n, h, h, c)).astype(np.int8))
        wq = DB.from_array(rng.integers(-127, 128, (9, c)).astype(np.int8))
        keep = [DB.from_array(a) for a in K.scale_arrays(0.02, rng.uniform(1e-3, 1e-2, c).astype(np.float32))]
        bias = DB.from_array(K.pad_channels(rng.standard_normal(c).astype(np.float32)))
        q = DB(n * h * h * K.round_up(c, 16))
        epi = K.Epi([K.Step("add", "channel", ptr=bias), K.Step("maximum", "scalar", scalar=0.0),
                     K.Step("minimum", "scalar", scalar=6.0)], out_i8=q, ld_i8=K.round_up(c, 16), out_scale=6.0 / 127)
        for _ in range(reps):
            K.qdwconv2d(x, c, n, h, h, c, wq, 3, 3, (1, 1), (1, 1), (1, 1), K.dequant_channel(*keep), epi)
    elif name == "attention_q1":
        b, hd, tk, dh = 64, 12, 1024, 64
        q = DB.from_array(rng.standard_normal((b, hd, 1, dh), dtype=np.float32))
        k = DB.from_array(rng.standard_normal((b, hd, tk, dh), dtype=np.float32))
        v = DB.from_array(rng.standard_normal((b, hd, tk, dh), dtype=np.float32))
        m = DB.from_array(np.where(np.arange(tk) <= 700, 0.0, -10000.0).astype(np.float32))
        out = DB(b * hd * dh * 4)
        st, qst = (hd * tk * dh, tk * dh, dh, 1), (hd * dh, dh, dh, 1)
        desc = K.Attn(b, hd, 1, tk, dh, K.View(q, qst), K.View(k, st), K.View(v, st), "mul", 0.125,
                      K.View(m, (0, 0, 0, 1)), out=K.View(out, qst))
        for _ in range(reps):
            K.attention_f32(desc)
    elif name == "quantize_rows":
        rows, cols = 65536, 768
        x = DB.from_array(rng.standard_normal((rows, cols), dtype=np.float32))
        xq = DB(rows * cols)
        for _ in range(reps):
            K.quantize_rows(x, rows, cols, cols, 0.03, xq, cols)
    elif name == "stem":
        n, h, o = 64, 224, 64
        x = DB.from_array(rng.standard_normal((n, 3, h, h), dtype=np.float32))
        ow = (h + 2 * 3 - 7) // 2 + 1
        entries = K.row4_entries(ow, 2)
        xq = DB(n * h * entries * 16)
        wq = K.conv_weight_row4(rng.integers(-127, 128, (o, 3, 7, 7)).astype(np.int8))
        s64, hi, lo = K.scale_arrays(0.03, rng.uniform(1e-3, 1e-2, o).astype(np.float32))
        keep = [DB.from_array(a) for a in (s64, hi, lo)]
        bias = DB.from_array(K.pad_channels(rng.standard_normal(o).astype(np.float32)))
        y = DB(n * ow * ow * o * 4)
        epi = K.Epi([K.Step("add", "channel", ptr=bias), K.Step("relu")], out_f32=y, ld_f32=o)
        wb = DB.from_array(wq)
        for _ in range(reps):
            K.quantize_nchw_to_row4(x, n, 3, h, h, 0.03, xq, entries, 3, 2)
            K.qconv2d(n, h, h, 4, xq, o, 7, 7, wb, wq.shape[1], (2, 2), (3, 3), (1, 1), K.dequant_channel(*keep), epi,
                      layout=_lib.LAYOUT_ROW4, row_entries=entries)
    elif name == "stem_pool":
        n, h, o = 64, 224, 64
        x = DB.from_array(rng.standard_normal((n, 3, h, h), dtype=np.float32))
        ow = (h + 2 * 3 - 7) // 2 + 1
        ph = (ow + 2 - 3) // 2 + 1
        entries = K.row4_entries(ow, 2)
        xq = DB(n * h * entries * 16)
        wq = K.conv_weight_row4(rng.integers(-127, 128, (o, 3, 7, 7)).astype(np.int8))
        keep = [DB.from_array(a) for a in K.scale_arrays(0.03, rng.uniform(1e-3, 1e-2, o).astype(np.float32))]
        bias = DB.from_array(K.pad_channels(rng.standard_normal(o).astype(np.float32)))
        y, yq = DB(n * ph * ph * o * 4), DB(K.cp_bytes(n, ph, ph, o), zero=True)
        epi = K.Epi([K.Step("add", "channel", ptr=bias), K.Step("relu")], out_f32=y, ld_f32=o, out_i8=yq, ld_i8=o,
                    out_scale=0.05, i8_layout=_lib.LAYOUT_CP)
        wb = DB.from_array(wq)
        K.quantize_nchw_to_row4(x, n, 3, h, h, 0.03, xq, entries, 3, 2)
        for _ in range(reps):
            K.qconv2d_maxpool(n, h, h, 4, xq, o, 7, 7, wb, wq.shape[1], (2, 2), (3, 3), (1, 1), 3, 2, 1, -np.inf,
                              K.dequant_channel(*keep), epi, layout=_lib.LAYOUT_ROW4, row_entries=entries)
    elif name == "attention_prefill":
        b0, b1, t, dh = 8, 12, 1024, 64
        q, k, v = (DB.from_array(rng.standard_normal((b0, b1, t, dh), dtype=np.float32)) for _ in range(3))
        m = np.where(np.arange(t)[:, None] >= np.arange(t)[None, :], 0.0, -10000.0).astype(np.float32)
        mb = DB.from_array(m)
        st = (b1 * t * dh, t * dh, dh, 1)
        out = DB(b0 * b1 * t * dh * 4)
        tm, km, tz = DB.from_array(K.mask_tile_max(m, t, t)), DB(16, zero=True), DB.from_array(K.mask_tile_zero(m, t, t))
        K.absmax_f32((b0, b1, t, dh), K.View(k, st), km)
        desc = K.Attn(b0, b1, t, t, dh, K.View(q, st), K.View(k, st), K.View(v, st), "mul", 0.125,
                      K.View(mb, (0, 0, t, 1)), tm, km, tz, out=K.View(out, st))
        # the planner's workspace selects the tensor-core kernel (MIRA_CUDA_ATTENTION=simt: the f32 one)
        nws = K.attention_workspace(b0, b1, t, t, dh)
        if nws > 0:
            ws = DB(nws)
            desc.workspace, desc.workspace_bytes = ws, nws
        for _ in range(reps):
            K.attention_f32(desc)
        if timed:   # CUDA events around 20 calls on the library stream, after the calls above
            a, b = C.c_void_p(), C.c_void_p()
            _lib.call("mira_cuda_event_create", C.byref(a))
            _lib.call("mira_cuda_event_create", C.byref(b))
            _lib.call("mira_cuda_sync")
            _lib.call("mira_cuda_event_record", a)
            for _ in range(20):
                K.attention_f32(desc)
            _lib.call("mira_cuda_event_record", b)
            _lib.call("mira_cuda_sync")
            ms = C.c_float()
            _lib.call("mira_cuda_event_elapsed", a, b, C.byref(ms))
            print(json.dumps({"case": name, "us_per_call": ms.value / 20 * 1e3, "calls": 20, "warmup": reps,
                              "kernel": "simt" if os.environ.get("MIRA_CUDA_ATTENTION") == "simt" else
                              ("tensor-core" if nws > 0 else "simt")}))
    elif name in ("layernorm_decode", "layernorm_prefill"):
        rows, d = (64, 768) if name == "layernorm_decode" else (65536, 768)
        x = DB.from_array(rng.standard_normal((rows, d), dtype=np.float32))
        g = DB.from_array((1 + 0.02 * rng.standard_normal(d)).astype(np.float32))
        bta = DB.from_array((0.02 * rng.standard_normal(d)).astype(np.float32))
        y = DB(rows * d * 4) if name == "layernorm_decode" else None
        yq = DB(rows * d)
        for _ in range(reps):
            K.layernorm_rows(x, rows, d, d, g, bta, 1e-5, out_f32=y, ld_f32=d if y is not None else 0, out_i8=yq,
                             ld_i8=d, out_scale=0.03)
    elif name == "decode_step":
        from mira_b200 import decode
        _, step = _decode_programs(DECODE["batch"], "cuda")
        exe = step.segments[0].executable
        exe.use_graph = False             # eager launches, so every kernel shows up individually
        dec = decode.Decoder(step)
        dec.reset()
        for i in range(reps):
            dec.step(np.full(DECODE["batch"], i % DECODE["vocab"], np.int32))
        print(f"decode step: {exe.launches_per_run} launches per step", flush=True)
    elif name == "maxpool_stem":
        n, h, c = 64, 112, 64
        x = DB.from_array(np.maximum(rng.standard_normal((n, h, h, c), dtype=np.float32), 0))
        oh = (h + 2 - 3) // 2 + 1
        y, yq = DB(n * oh * oh * c * 4), DB(n * oh * oh * c)
        for _ in range(reps):
            K.maxpool2d(n, h, h, c, c, 3, 2, 1, -np.inf, x_f32=x, out_f32=y, ldc_out_f32=c, out_i8=yq, ldc_out_i8=c,
                        out_scale=0.05)
    else:
        raise SystemExit(f"unknown profile case {name}; one of {', '.join(PROFILE_CASES)}")
    _lib.call("mira_cuda_sync")
    print(f"profile case {name}: {reps} launches ok", flush=True)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of the largest launch of the conv family,
# ResNet-18's layer-1 3x3 conv with an f32 and an int8 output at batch 256 (`--profile-case
# conv_l1_cp`, one ncu capture of that kernel: 58.0 MB read, 208.7 MB written), against its 307 MB
# of algorithmic bytes (51 MB int8 in, 205 MB f32 + 51 MB int8 out; some writes are still in L2
# when the kernel ends).  A whole pass at a batch small enough for an ncu capture keeps its
# activations in the 126 MB L2, so its DRAM bytes say nothing about batch 256.
CONV_L1_DRAM_BYTES = 58.0e6 + 208.7e6


def pass_bytes(graph) -> dict:
    """Algorithmic HBM bytes of one forward pass of the compiled graph, in this target's
    representations: every activation is written once per representation it needs (int8, 1 byte
    per element, when a quantized op reads it; f32 otherwise) and read once by each op that uses
    it; weights and the graph input are read once.  Views (reshape/transpose) and the padding that
    the max pool reads through cost nothing."""
    QO = ("qconv2d", "qmatmul")
    FREE = ("reshape", "transpose", "pad", "const")
    users: dict = {}
    for op in graph.ops:
        for i, v in enumerate(op.inputs):
            users.setdefault(v, []).append((op, i))

    def root(v):
        p = v.producer
        while p is not None and p.kind in FREE[:3]:
            v = p.inputs[0]
            p = v.producer
        return v

    def numel(v):
        return int(np.prod(v.type.shape, dtype=np.int64))

    def is_const(v):
        p = v.producer
        return p is not None and p.kind in ("const", "dequantize")

    reads = writes = weights = 0
    reps: dict = {}
    for op in graph.ops:
        if op.kind in FREE or op.is_constant_like:
            continue
        for i, v in enumerate(op.inputs):
            if is_const(v):
                continue
            r = root(v)
            kind = "i8" if (op.kind in QO and i == 0) else "f32"
            reps.setdefault(r, set()).add(kind)
            reads += numel(r) * (1 if kind == "i8" else 4)
        if op.kind in QO:
            weights += int(np.asarray(op.attrs["q"]).nbytes)
    for v, kinds in reps.items():
        if v in graph.inputs:
            continue
        writes += numel(v) * sum(1 if k == "i8" else 4 for k in kinds)
    for v in graph.outputs:
        writes += numel(v) * 4
    x_bytes = sum(numel(v) * 4 for v in graph.inputs)
    reads_no_input = reads - sum(numel(v) * 4 for v in graph.inputs if v in reps)
    total = reads_no_input + x_bytes + writes + weights
    return {"bytes": total, "activation_reads": reads_no_input, "activation_writes": writes,
            "weights": weights, "input": x_bytes}


def parity_check(workload: str, batch: int, out: np.ndarray, x: np.ndarray, calib_batch: int, n_calib: int,
                 n_images: int = 4, **kw) -> dict:
    """The timed program's own output rows against the reference cpu target (MIRA's NumPy golden
    model) run on the same input rows, bit for bit: a batch-1 (MLP: full-batch) cpu program compiled
    with the same calibration, so every activation scale is identical.  Images: first, last and a
    seeded middle pair."""
    from mira_b200 import configs
    if workload == "mlp":
        cpu = configs.compile_w8a8(workload, batch, "cpu", calib_batch=calib_batch, n_calib=n_calib, **kw)
        want = cpu.run({"x": x})
        bad = int((want != out).any(axis=1).sum())
        return {"images": int(batch), "mismatches": bad, "oracle": "reference cpu target, whole batch"}
    cpu = configs.compile_w8a8(workload, 1, "cpu", calib_batch=calib_batch, n_calib=n_calib, **kw)
    rng = np.random.default_rng(7)
    idx = sorted({0, batch - 1, *(int(i) for i in rng.choice(batch, size=max(0, n_images - 2), replace=False))})
    bad = [i for i in idx if not np.array_equal(cpu.run({"x": x[i:i + 1]}), out[i:i + 1])]
    return {"images": len(idx), "mismatches": len(bad), "rows": idx,
            "oracle": "reference cpu target (batch-1 program, same calibration), bit for bit"}


def reference_cpu_sample(steps: int, warmup: int, workload: str = WORKLOAD, max_seconds: float = 60.0) -> dict:
    """The reference's own cpu W8A8 path (mira.compile_ir(..., "cpu", quantize="w8a8") then
    CompiledProgram.run) on the workload's bounded sample: `steps` runs, or fewer when they would
    take longer than `max_seconds` (the rate is over the runs done)."""
    w = WORKLOADS[workload]
    from mira_b200 import configs
    from mira_b200.hostfw import import_mira
    import_mira()
    batch = w["cpu_batch"]
    prog = configs.compile_w8a8(workload, batch, "cpu", n_calib=w["n_calib"], calib_batch=batch,
                                build_kw=w["cpu_build_kw"] or None)
    feeds = configs.random_inputs(prog.graph, 1)
    rows = int(prog.graph.inputs[0].type.shape[0])
    items = rows * (prog.graph.inputs[0].type.shape[1] if w["items_per_row"] > 1 else 1)
    for _ in range(warmup):
        prog.run(feeds)
    t0 = time.perf_counter()
    done = 0
    while done < steps and (done == 0 or time.perf_counter() - t0 < max_seconds):
        prog.run(feeds)
        done += 1
    dt = time.perf_counter() - t0
    return {"value": items * done / dt * w["cpu_scale"], "unit": w["unit"], "cores": os.cpu_count(),
            "kind": "reference", "ms_per_step": dt / done * 1e3, "steps_run": done,
            "sample": f"{done} run(s) after {warmup} warm-up run(s) (at most {steps}, stopped after "
                      f"{max_seconds:.0f} s), {w['cpu_note']}; reference cpu target "
                      f"(NumPy golden model, OpenBLAS on all host cores)"}


def _decode_programs(batch: int, target: str, device: int = 0):
    """(prefill program on the host, used for its activation scales; W8A8 step program for target)."""
    from mira_b200 import configs, decode
    pre = configs.compile_w8a8("transformer", 1, "cpu", n_calib=4, calib_batch=1)
    opts = {"device": device} if target == "cuda" else {}
    return pre, decode.compile_step(configs.transformer_step(batch, max_seq=DECODE["max_seq"]), pre, target, **opts)


def reference_decode_sample(steps: int, warmup: int, max_seconds: float = 60.0) -> dict:
    """The reference cpu target running the quantized step graph (batch 1, caches through the host),
    `steps` steps or as many as fit in `max_seconds`."""
    _, prog = _decode_programs(1, "cpu")
    g = prog.graph
    names = [v.name for v in g.inputs[3:]]
    caches = {n: np.zeros(v.type.shape, np.float32) for n, v in zip(names, g.inputs[3:])}
    tok = np.zeros((1, 1), np.int32)
    dt = 0.0
    done = 0
    for i in range(warmup + steps):
        if i >= warmup and done > 0 and dt > max_seconds:
            break
        t0 = time.perf_counter()
        out = prog.run({"tok": tok, "pos2": np.array([i, 0], np.int32), "pos4": np.array([0, 0, i, 0], np.int32),
                        **caches})
        if i >= warmup:
            dt += time.perf_counter() - t0
            done += 1
        caches = dict(zip(names, out[1:]))
        tok = out[0][:, 0].argmax(axis=1).astype(np.int32).reshape(1, 1)
    return {"value": done / dt, "unit": DECODE["unit"], "cores": os.cpu_count(), "kind": "reference",
            "ms_per_step": dt / done * 1e3, "steps_run": done,
            "sample": f"{done} step(s) after {warmup} warm-up step(s) of one sequence (batch 1) through the W8A8 "
                      f"step graph, caches through the host; reference cpu target (NumPy golden model, OpenBLAS "
                      f"on all host cores)"}


def run_reference(args) -> None:
    rank, world, _ = _env_rank()
    if rank != 0:
        return
    if args.workload == "decode":
        res = reference_decode_sample(args.steps, args.warmup)
        line = {"metric": DECODE["metric"], "value": res["value"], "unit": DECODE["unit"], "impl": "reference",
                "n_gpus": args.gpus, "steps": res["steps_run"], "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic", "config": {"workload": DECODE["config"], "batch_per_step": 1,
                                                "note": "bounded sample: one sequence per step"},
                "cpu_baseline": res, "e2e": {"value": res["value"], "unit": DECODE["unit"], "h2d_bytes_per_step": 0,
                                             "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    w = WORKLOADS[args.workload]
    res = reference_cpu_sample(args.steps, args.warmup, args.workload)
    line = {"metric": w["metric"], "value": res["value"], "unit": w["unit"], "impl": "reference", "n_gpus": args.gpus,
            "steps": res["steps_run"], "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": w["config"], "batch_per_step": w["cpu_batch"],
                       "note": f"bounded sample of the workload: {w['cpu_note']}"},
            "cpu_baseline": res, "e2e": {"value": res["value"], "unit": w["unit"], "h2d_bytes_per_step": 0,
                                         "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_decode(args, rank: int, world: int, local: int, dist) -> None:
    """Config-5 decode: `batch` sequences per GPU, one token each per step, caches resident.

    value: tokens/s over K steps replayed on the device (each step attends over all max_seq cache
    rows, so every position costs the same); e2e: K Decoder.step calls (token ids and start
    vectors to the device, logits back, positions advancing).  HBM-bound: the roofline counts the
    int8 weights and the whole key/value cache read each step."""
    from mira_b200 import _lib, decode

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    batch = args.batch
    if args.warmup + 2 * args.steps > DECODE["max_seq"]:
        raise SystemExit(f"warmup + 2 * steps must stay within the {DECODE['max_seq']} cache positions")
    t0 = time.perf_counter()
    _, step = _decode_programs(batch, "cuda", local)
    compile_s = time.perf_counter() - t0
    dec = decode.Decoder(step)
    exe = dec.exe
    rng = np.random.default_rng(1 + rank)
    toks = rng.integers(0, DECODE["vocab"], (batch, args.warmup + 2 * args.steps)).astype(np.int32)
    dec.reset()
    for i in range(args.warmup):           # eager first step, then the captured CUDA graph
        logits = dec.step(toks[:, i])

    ev_a, ev_b = C.c_void_p(), C.c_void_p()
    _lib.call("mira_cuda_event_create", C.byref(ev_a))
    _lib.call("mira_cuda_event_create", C.byref(ev_b))
    n0 = _lib.launch_count()
    barrier()
    _lib.call("mira_cuda_sync")
    with ClockSampler(local) as clocks:
        _lib.call("mira_cuda_event_record", ev_a)
        for _ in range(args.steps):
            exe.replay()
        _lib.call("mira_cuda_event_record", ev_b)
        _lib.call("mira_cuda_sync")
        ms = C.c_float()
        _lib.call("mira_cuda_event_elapsed", ev_a, ev_b, C.byref(ms))
    barrier()
    dev_ms = max_over_ranks(ms.value)
    gpu_launches = args.steps * exe.launches_per_run + (_lib.launch_count() - n0)

    barrier()
    t1 = time.perf_counter()
    for i in range(args.steps):
        logits = dec.step(toks[:, args.warmup + i])
    e2e_s = max_over_ranks(time.perf_counter() - t1)
    barrier()

    if rank == 0:
        bf16, hbm, src = _peaks()
        g = exe.g
        weight_bytes = sum(np.asarray(op.attrs["q"]).nbytes + 4 * np.asarray(op.attrs["w_scale"]).size
                           for op in g.ops if op.kind == "qmatmul")
        cache_bytes = sum(v.type.numel * 4 for v in dec.caches)
        step_bytes = weight_bytes + cache_bytes
        step_ms = dev_ms / args.steps
        kernels = {}
        for kind in ("attention", "qgemm", "layernorm", "dyn_update", "dyn_slice", "embed"):
            ms_k, n_k = time_kernels(exe, (kind,))
            if n_k:
                kernels[kind] = {"launches": n_k, "ms_per_step": ms_k}
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = reference_decode_sample(3, 1)
        items = batch * world * args.steps
        result = {
            "metric": DECODE["metric"], "value": items / (dev_ms * 1e-3), "unit": DECODE["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": DECODE["config"], "global_batch": batch * world, "batch_per_gpu": batch,
                       "parallelism": f"dp{world} (replicas, no collective)",
                       "l2": f"inputs larger than L2 ({cache_bytes / 1e9:.1f} GB key/value cache read per step)",
                       "calibration": "prefill activation scales (4 seeded sequences of 1024 tokens)",
                       "compile_s": round(compile_s, 1)},
            "e2e": {"value": items / e2e_s, "unit": DECODE["unit"], "h2d_bytes_per_step": batch * 4 + 8 + 16,
                    "d2h_bytes_per_step": int(logits.nbytes)},
            "roofline": {"bound": "hbm", "kernel": "whole step (int8 weights + key/value cache reads)",
                         "achieved": step_bytes / (step_ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": (step_bytes / (step_ms * 1e-3) / 1e9 / hbm) if hbm else None, "traffic": None,
                         "algorithmic_bytes_per_step": step_bytes, "weight_bytes": weight_bytes,
                         "cache_bytes": cache_bytes, "peak_source": f"hbm_gbs of {src}"},
            "kernels": kernels, "gpu_launches": int(gpu_launches), "clocks": clocks.summary(), "cpu_baseline": cpu,
        }
        print(json.dumps(result), flush=True)
    if dist is not None:
        barrier()
        dist.destroy_process_group()


def _init_dist(local: int):
    import datetime

    import torch
    import torch.distributed as dist
    if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
        os.environ["NCCL_DEBUG"] = "WARN"      # keep stdout to the one JSON line
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    return dist


def _device_timed(exe, steps: int, barrier, max_over_ranks, local: int, sample_clocks: bool = True):
    """(max over ranks of the CUDA-event ms of `steps` device-resident replays, launches, clocks)."""
    from mira_b200 import _lib
    ev_a, ev_b = C.c_void_p(), C.c_void_p()
    _lib.call("mira_cuda_event_create", C.byref(ev_a))
    _lib.call("mira_cuda_event_create", C.byref(ev_b))
    n0 = _lib.launch_count()
    barrier()
    _lib.call("mira_cuda_sync")
    with ClockSampler(local) as clocks:
        _lib.call("mira_cuda_event_record", ev_a)
        for _ in range(steps):
            exe.replay()
        _lib.call("mira_cuda_event_record", ev_b)
        _lib.call("mira_cuda_sync")
        ms = C.c_float()
        _lib.call("mira_cuda_event_elapsed", ev_a, ev_b, C.byref(ms))
    barrier()
    launches = steps * exe.launches_per_run + (_lib.launch_count() - n0)
    _lib.call("mira_cuda_event_destroy", ev_a)
    _lib.call("mira_cuda_event_destroy", ev_b)
    return max_over_ranks(ms.value), launches, clocks


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None, help="batch rows per GPU per step (workload default)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=WORKLOAD, choices=sorted(WORKLOADS) + ["decode"])
    ap.add_argument("--calib-batch", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the parity check of the timed output")
    ap.add_argument("--no-gemm", action="store_true", help="skip the config-2 GEMM sweep of the headline line")
    ap.add_argument("--int8-depthwise", action="store_true",
                    help="MobileNetV2 in the opt-in int8 depthwise mode (mira_b200.int8_depthwise); the parity "
                         "check then compares with the reference cpu target compiled in the same mode")
    ap.add_argument("--fuse-pool", action="store_true",
                    help="compute a conv whose only consumer is a max pool inside the pooling kernel")
    ap.add_argument("--profile-case", choices=PROFILE_CASES, default=None,
                    help="launch one kernel on a bounded case a few times (for ncu) and exit")
    ap.add_argument("--time-case", action="store_true",
                    help="with --profile-case attention_prefill: also time 20 calls with CUDA events (not under ncu)")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case, reps=5 if args.time_case else 3, timed=args.time_case)
        return
    args.warmup = max(args.warmup, 3)
    if args.workload == "decode":
        args.batch = args.batch or DECODE["batch"]
        args.steps = min(args.steps, (DECODE["max_seq"] - args.warmup) // 2)
        if args.impl == "reference":
            run_reference(args)
            return
        rank, world, local = _env_rank()
        os.environ["MIRA_CUDA_DEVICE"] = str(local)
        dist = _init_dist(local) if world > 1 else None
        run_decode(args, rank, world, local, dist)
        return
    wl = WORKLOADS[args.workload]
    args.batch = args.batch or wl["batch"]
    args.calib_batch = args.calib_batch or wl["calib_batch"]
    if args.impl == "reference":
        run_reference(args)
        return

    rank, world, local = _env_rank()
    os.environ["MIRA_CUDA_DEVICE"] = str(local)
    dist = _init_dist(local) if world > 1 else None

    from mira_b200 import configs

    t0 = time.perf_counter()
    mode = {"int8_depthwise": True} if args.int8_depthwise else {}
    prog = configs.compile_w8a8(args.workload, args.batch, "cuda", calib_batch=args.calib_batch, device=local,
                                n_calib=wl["n_calib"], build_kw=wl["build_kw"] or None, fuse_pool=args.fuse_pool,
                                **mode)
    compile_s = time.perf_counter() - t0
    segs = [s for s in prog.segments if s.device == "cuda"]
    assert len(prog.segments) == 1 and len(segs) == 1, "the whole network must be one cuda segment"
    exe = segs[0].executable
    x_val = prog.graph.inputs[0]
    host_x = exe.input_array(x_val)          # pinned staging array of the executable

    def fill_input(arr, r):
        rng = np.random.default_rng(1 + r)
        if arr.dtype == np.int32:             # token ids
            arr[...] = rng.integers(0, configs._vocab_of(prog.graph, x_val), arr.shape)
        else:
            arr[...] = rng.standard_normal(arr.shape, dtype=np.float32)

    fill_input(host_x, rank)
    name = x_val.name
    feeds = {name: host_x}

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- warm-up through the public API (also captures the CUDA graph)
    for _ in range(args.warmup):
        out = prog.run(feeds)

    # ---- device-resident timing
    dev_ms, gpu_launches, clocks = _device_timed(exe, args.steps, barrier, max_over_ranks, local)

    # ---- end to end, K steps with host buffers: through the executable's streaming call run_many
    # (each step's input copy overlaps the previous step's kernels; with several GPUs the final
    # gather of the logits to rank 0 runs on the device after each step's kernels) and through the
    # reference's blocking CompiledProgram.run (copy in, kernels, copy out, one step at a time)
    gather = None
    if dist is not None:
        from mira_b200.shard import DeviceGather
        gather = DeviceGather(exe, world, rank)
    exe.run_many([{x_val: host_x}] * 2, gather=gather)   # first use allocates the second buffers, events
    barrier()
    t1 = time.perf_counter()
    outs = exe.run_many([{x_val: host_x}] * args.steps, gather=gather)
    e2e_s = max_over_ranks(time.perf_counter() - t1)
    barrier()
    out_global = outs[-1].get(exe.g.outputs[0]) if outs[-1] else None
    t1 = time.perf_counter()
    for _ in range(args.steps):
        out = prog.run(feeds)
    e2e_blocking_s = max_over_ranks(time.perf_counter() - t1)
    barrier()

    # ---- multi-GPU checks and strong scaling (untimed: after the timed regions)
    multi = None
    if dist is not None:
        check = None
        if rank == 0:
            # another rank's shard, recomputed on this GPU, against the gathered rows of that rank
            other = world - 1
            x_other = np.empty_like(host_x)
            fill_input(x_other, other)
            mine = prog.run({name: x_other})
            rows = out_global[other * args.batch:(other + 1) * args.batch]
            own = out_global[:args.batch]
            check = {"rank_recomputed_on_rank0": other, "rows": int(args.batch),
                     "mismatches": int((rows != mine).any(axis=1).sum()),
                     "rank0_rows_match_local_run": bool(np.array_equal(own, out))}
        strong_batch = max(1, 256 // world) if args.workload in ("resnet18", "mobilenet_v2") else None
        strong = None
        if strong_batch is not None:
            sprog = configs.compile_w8a8(args.workload, strong_batch, "cuda", calib_batch=args.calib_batch,
                                         device=local, n_calib=wl["n_calib"], build_kw=wl["build_kw"] or None, **mode)
            sexe = sprog.segments[0].executable
            sx = sexe.input_array(sprog.graph.inputs[0])
            fill_input(sx, rank)
            for _ in range(args.warmup):
                sprog.run({name: sx})
            s_ms, _, _ = _device_timed(sexe, args.steps, barrier, max_over_ranks, local)
            strong = {"global_batch": strong_batch * world, "batch_per_gpu": strong_batch,
                      "value": strong_batch * world * args.steps / (s_ms * 1e-3), "ms_per_step": s_ms / args.steps}
        multi = {"gather": "NCCL gather of the logits to rank 0 on the device after every e2e step "
                           "(mira_b200.shard.DeviceGather), then one device-to-host copy on rank 0",
                 "check": check, "strong_scaling": strong}

    items = args.batch * wl["items_per_row"] * world * args.steps
    value = items / (dev_ms * 1e-3)
    conv_ops, q_ops = conv_work(prog.graph)
    headline = args.workload == WORKLOAD

    result = None
    if rank == 0:
        bf16, hbm, src = _peaks()
        peak = 2.0 * bf16 if bf16 else None
        # roofline of the int8 tensor-core kernels: the convolutions (ResNet-18, MobileNetV2) or all
        # quantized matmuls (MLP, transformer)
        kinds = ("qconv2d", "qconv2d_pool") if conv_ops else ("qgemm",)
        fam_ops = conv_ops if conv_ops else q_ops
        fam_ms, fam_n = time_kernels(exe, kinds)
        achieved = fam_ops / (fam_ms * 1e-3) / 1e12
        fam_kernels = ("qgemm_sm100_kernel" + (" + stem_pool_kernel" if any(
            l.kind == "qconv2d_pool" for l in exe.plan.launches) else "")) if conv_ops else "qgemm_sm100_kernel"
        other = {}
        for kind in sorted(set(l.kind for l in exe.plan.launches)):
            ms_k, n_k = time_kernels(exe, (kind,))
            if n_k:
                other[kind] = {"launches": n_k, "ms_per_step": ms_k}
        step_ms = dev_ms / args.steps
        pb = pass_bytes(prog.graph)
        hbm_pass = {"bound": "hbm", "kernel": "whole pass (every launch of one step)",
                    "achieved": pb["bytes"] / (step_ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                    "frac": pb["bytes"] / (step_ms * 1e-3) / 1e9 / hbm if hbm else None,
                    "algorithmic_bytes_per_step": pb, "peak_source": f"hbm_gbs of {src}"}
        gemm = None
        if headline and world == 1 and not args.no_gemm:
            gemm = gemm_sweep(peak)
            g8 = gemm["square"]["8192"]
            gemm.update({"shape": "8192^3", "tops": g8["tops"], "frac_of_peak": g8["frac_of_2x_bf16"],
                         "cublaslt_tops": g8["cublaslt_tops"], "frac_of_cublaslt": g8["frac_of_cublaslt"],
                         "frac_of_larger_peak": g8["tops"] / max(peak or 0, g8["cublaslt_tops"] or 0)
                         if (peak or g8["cublaslt_tops"]) else None})
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            try:
                cpu = reference_cpu_sample(3, 1, args.workload)
            except Exception as e:  # the reference package is missing on this machine
                cpu = {"value": None, "unit": wl["unit"], "cores": os.cpu_count(), "kind": "reference",
                       "sample": f"unavailable: {e}"}
        parity = None
        if not args.no_check and args.workload != "transformer":
            try:
                parity = parity_check(args.workload, args.batch, outs[-1][exe.g.outputs[0]][:args.batch],
                                      host_x, args.calib_batch, wl["n_calib"], **mode)
            except ImportError as e:
                parity = {"unavailable": str(e)}
        in_desc = (f"{host_x.nbytes / 1e6:.0f} MB input batch") if host_x.nbytes > 1e6 else "small input batch"
        h2d = int(host_x.nbytes)
        result = {
            "metric": wl["metric"], "value": value, "unit": wl["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": wl["config"], "global_batch": args.batch * world,
                       "batch_per_gpu": args.batch, "parallelism": f"dp{world} (replicas, no collective in "
                                                                   f"the device-timed step)",
                       "l2": (f"inputs larger than L2 ({in_desc}, activations of several GB per step)")
                       if host_x.nbytes > 126e6 or args.workload == "transformer"
                       else f"working set near L2 ({in_desc})",
                       "calibration": f"{wl['n_calib']} seeded batches of {args.calib_batch}",
                       **({"mode": "opt-in int8 depthwise (mira_b200.int8_depthwise)"} if mode else {}),
                       "compile_s": round(compile_s, 1)},
            "e2e": {"value": items / e2e_s, "unit": wl["unit"], "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": int(out.nbytes) * world,
                    "h2d_gb_s_per_gpu": h2d * args.steps / e2e_s / 1e9,
                    "call": "CudaExecutable.run_many: host batch (pinned) copied in and logits read back every "
                            "step, the next step's copy overlapping this step's kernels"
                            + ("; logits gathered to rank 0 on the device every step" if world > 1 else "")},
            "e2e_blocking": {"value": items / e2e_blocking_s, "unit": wl["unit"],
                             "call": "CompiledProgram.run, one step at a time (copy in, kernels, copy out)"},
            "roofline": {"bound": "tensor", "kernel": f"{fam_kernels} ({'/'.join(kinds)}, {fam_n} launches/step)",
                         "achieved": achieved, "peak": peak, "unit": "TOPS",
                         "frac": (achieved / peak) if peak else None,
                         "traffic": CONV_L1_DRAM_BYTES if headline else None,
                         "traffic_unit": "DRAM bytes of one launch of the family's largest kernel (layer-1 3x3 "
                                         "conv, f32 + int8 out, batch 256; 307 MB algorithmic)"
                         if headline else None,
                         "peak_source": f"2 x bf16_tflops of {src} (dense int8 issues at twice the bf16 rate)",
                         "int8_ops_per_step": fam_ops, "ms_per_step": fam_ms},
            "roofline_hbm_pass": hbm_pass,
            "int8_ops_per_step": q_ops, "int8_tops_step": q_ops / (step_ms * 1e-3) / 1e12,
            "gpu_launches": int(gpu_launches), "clocks": clocks.summary(),
            "cpu_baseline": cpu, "kernels": other,
        }
        if parity is not None:
            result["parity"] = parity
        if gemm is not None:
            result["int8_gemm"] = gemm
        if multi is not None:
            result["multi_gpu"] = multi
        print(json.dumps(result), flush=True)
    if dist is not None:
        barrier()
        del gather
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
