"""Host-driven W8A8 decode of the config-5 transformer on the cuda target.

The reference compiles one program per graph and rejects W8A8 quantization of programs with
control flow (mira/quantize.py:84-85), so generation cannot be one quantized program.  Decode is
instead a per-step graph (configs.transformer_step: one new token per sequence, a key/value cache
per layer read and written at a runtime position with the reference's dynamic_slice /
dynamic_update_slice, ops.py:533-576) driven by a loop on the host:

  * compile_step quantizes the step graph with the reference's own pipeline (passes.optimize,
    quantize.quantize_w8a8, compiler.compile_graph) and then gives every int8 matmul the
    activation scale of the prefill program's matmul with the same weights, so a decode step
    quantizes exactly like the prefill row at the same position;
  * Decoder keeps the caches resident on the GPU: the plan writes each step's keys and values into
    the cache input's own device buffer (the dynamic_update_slice result aliases the input), and
    the executable copies neither the caches in nor the updated caches out; per step only the
    token ids and the two start vectors go to the device and the logits come back.
"""
from __future__ import annotations

import hashlib
import time
from typing import Optional

import numpy as np

from .hostfw import import_mira
from .plugin import install


def _weight_key(q: np.ndarray) -> tuple:
    q = np.ascontiguousarray(q)
    return q.shape, hashlib.sha1(q.view(np.uint8)).hexdigest()


def quantize_step_like(step_graph, prefill_program, log: Optional[list] = None) -> int:
    """Rewrites `step_graph` (in place) for W8A8 with the prefill program's activation scales.

    The graph is optimized and quantized by the reference (calibrated on one all-zero step, whose
    scales are then replaced); each qmatmul then takes the x_scale of the prefill qmatmul whose
    int8 weights are identical.  Returns the number of int8 matmuls."""
    import_mira()
    from mira import passes
    from mira import quantize as Q
    passes.optimize(step_graph, fuse=True, precision=None, log=log)
    feed = {v.name: np.zeros(v.type.shape, v.type.np_dtype) for v in step_graph.inputs}
    Q.quantize_w8a8(step_graph, [feed], log=log)
    scales = {}
    for op in prefill_program.graph.ops:
        if op.kind == "qmatmul":
            scales.setdefault(_weight_key(op.attrs["q"]), op.attrs["x_scale"])
    n = 0
    for op in step_graph.ops:
        if op.kind != "qmatmul":
            continue
        key = _weight_key(op.attrs["q"])
        if key not in scales:
            raise ValueError("a step matmul has no prefill matmul with the same weights")
        op.attrs["x_scale"] = scales[key]
        n += 1
    return n


def compile_step(step_graph, prefill_program, target: str = "cuda", **target_options):
    """The W8A8 step program (a reference CompiledProgram) with the prefill's activation scales."""
    install()
    from mira.backends import get_target
    from mira.compiler import CompiledProgram, compile_graph
    t0 = time.perf_counter()
    log: list = []
    quantize_step_like(step_graph, prefill_program, log)
    runner = compile_graph(step_graph, get_target(target, **target_options), True)
    return CompiledProgram(target, runner, log, time.perf_counter() - t0)


class Decoder:
    """Greedy decode with device-resident caches around a compiled step program whose graph is
    configs.transformer_step (inputs tok, pos2, pos4, k0, v0, ...; outputs logits, then the caches)."""

    def __init__(self, step_program):
        segs = step_program.segments
        if len(segs) != 1 or segs[0].device != "cuda":
            raise ValueError("the step program must be a single cuda segment")
        self.exe = segs[0].executable
        ins = {v.name: v for v in self.exe.g.inputs}
        self.tok, self.pos2, self.pos4 = ins["tok"], ins["pos2"], ins["pos4"]
        self.caches = [v for v in self.exe.g.inputs if v.name not in ("tok", "pos2", "pos4")]
        pairs = self.exe.state_pairs()
        if sorted(x.name for x, _ in pairs) != sorted(v.name for v in self.caches):
            raise ValueError("every cache input must be updated in place by the step")
        self.exe.keep_resident(pairs)
        self.logits = next(v for v in self.exe.g.outputs if v not in self.exe.resident_out)
        self.batch = int(self.tok.type.shape[0])
        self.max_seq = int(self.caches[0].type.shape[2])
        self.pos = 0
        self._tok = self.exe.input_array(self.tok)
        self._p2 = self.exe.input_array(self.pos2)
        self._p4 = self.exe.input_array(self.pos4)

    def reset(self) -> None:
        """Empty caches, position 0."""
        for v in self.caches:
            self.exe.state_zero(v)
        self.pos = 0

    def step(self, tokens: np.ndarray) -> np.ndarray:
        """Feeds one token per sequence at the current position; returns logits f32[B, vocab]."""
        if self.pos >= self.max_seq:
            raise ValueError(f"the caches hold {self.max_seq} positions")
        self._tok[...] = np.asarray(tokens, np.int32).reshape(self._tok.shape)
        self._p2[...] = (self.pos, 0)
        self._p4[...] = (0, 0, self.pos, 0)
        out = self.exe.run({self.tok: self._tok, self.pos2: self._p2, self.pos4: self._p4})
        self.pos += 1
        return out[self.logits].reshape(self.batch, -1)

    def generate(self, prompt: np.ndarray, new_tokens: int) -> tuple[np.ndarray, np.ndarray]:
        """Runs the prompt int32[B, P] through the step one position at a time, then appends
        `new_tokens` greedy (argmax) tokens.  Returns (tokens int32[B, P + new_tokens], logits
        f32[P + new_tokens - 1, B, vocab]: the logits of every position whose successor was read)."""
        prompt = np.asarray(prompt, np.int32)
        if prompt.shape[1] + new_tokens - 1 > self.max_seq:
            raise ValueError(f"the caches hold {self.max_seq} positions")
        self.reset()
        toks = [prompt[:, i] for i in range(prompt.shape[1])]
        logits = [self.step(t) for t in toks]
        for i in range(new_tokens):
            toks.append(logits[-1].argmax(axis=1).astype(np.int32))
            if i + 1 < new_tokens:
                logits.append(self.step(toks[-1]))
        return np.stack(toks, axis=1), np.stack(logits)

    def read_cache(self, i: int) -> np.ndarray:
        return self.exe.state_read(self.caches[i])
