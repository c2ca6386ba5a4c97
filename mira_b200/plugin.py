"""Registers the `cuda` target with MIRA through its own target-plugin surface.

Reference hooks (myramay/MIRA):
  * mira/backends/__init__.py:5-22  get_target(name, **options) - an if-chain; wrapped so "cuda"
    returns CudaTarget.  mira/compiler.py:12 imported get_target by name, so that binding is
    replaced as well.
  * mira/backends/__init__.py:25    TARGETS - the CLI's --target choices (mira/cli.py:261); "cuda"
    is appended in place before the CLI builds its parser.
  * mira/compiler.py:293-294        precision "auto" means f16 for every non-cpu target; W8A8 on
    cuda computes in f32 exactly like the cpu golden model, so "auto" becomes None for "cuda".
  * mira/partition.py:73-80         placement asks target.check(op); CudaTarget.check accepts every
    qmatmul/qconv2d, and compile_ir verifies afterwards that none landed on the CPU.
  * mira/compiler.py:134-150        CompiledProgram.run validates the named inputs and converts each
    with astype, which always copies; for cuda programs the same checks run but an input that
    already has the IR dtype is passed on without a copy (the executable copies it to the device).
"""
from __future__ import annotations

import functools

from .hostfw import import_mira

_installed = False


def install():
    """Idempotent: makes "cuda" a MIRA target.  Returns the `mira` module."""
    global _installed
    mira = import_mira()
    if _installed:
        return mira
    import mira.backends as B
    import mira.compiler as Cmp

    original_get_target = B.get_target

    @functools.wraps(original_get_target)
    def get_target(name: str, **options):
        if name in ("cuda", "b200"):
            from .target import CudaTarget
            return CudaTarget(**options)
        return original_get_target(name, **options)

    B.get_target = get_target
    Cmp.get_target = get_target
    if "cuda" not in B.TARGETS:
        B.TARGETS.append("cuda")

    original_compile_ir = Cmp.compile_ir

    @functools.wraps(original_compile_ir)
    def compile_ir(graph, target="cpu", *, precision="auto", **kw):
        if target in ("cuda", "b200"):
            if precision == "auto":
                precision = None
            if precision is not None:
                raise ValueError("the cuda target runs W8A8 in f32 like the cpu golden model; use precision=None "
                                 f"(got {precision!r})")
        prog = original_compile_ir(graph, target, precision=precision, **kw)
        if target in ("cuda", "b200"):
            _check_placement(prog)
        return prog

    Cmp.compile_ir = compile_ir

    original_run = Cmp.CompiledProgram.run

    @functools.wraps(original_run)
    def run(self, inputs):
        if self.target not in ("cuda", "b200"):
            return original_run(self, inputs)
        import numpy as np
        from mira.errors import MiraError
        missing = [v.name for v in self.graph.inputs if v.name not in inputs]
        if missing:
            raise MiraError(f"missing input(s): {', '.join(missing)}")
        extra = set(inputs) - {v.name for v in self.graph.inputs}
        if extra:
            raise MiraError(f"unknown input(s): {', '.join(sorted(extra))}")
        feeds = {}
        for v in self.graph.inputs:
            arr = np.asarray(inputs[v.name])
            if tuple(arr.shape) != v.type.shape:
                raise MiraError(f"input '{v.name}' should have shape {list(v.type.shape)}, got {list(arr.shape)}")
            feeds[v] = np.asarray(arr, dtype=v.type.np_dtype)
        env = self.runner.run_env(feeds)
        outs = [env[v] for v in self.graph.outputs]
        return outs[0] if len(outs) == 1 else tuple(outs)

    Cmp.CompiledProgram.run = run
    _installed = True
    return mira


def _check_placement(prog) -> None:
    """Every quantized op must run on the cuda target (no CPU fallback for the hot path)."""
    on_cpu = [op for op, dev in prog.placement.device.items() if op.kind in ("qmatmul", "qconv2d") and dev != "cuda"]
    if on_cpu:
        raise RuntimeError(f"{len(on_cpu)} quantized op(s) were placed on the CPU: "
                           + ", ".join(sorted({op.kind for op in on_cpu})))
