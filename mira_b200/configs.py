"""The benchmark workloads, built as MIRA IR graphs with the reference's own `ir.Graph` API
(the reference's ONNX importer needs `onnx`, which is not installed; its BatchNorm lowering is
replaced by folding BN into the conv weights and biases before quantization, as the configs ask).

  mlp          784-512-512-10 ReLU MLP, Kaiming-normal weights, zero biases (config 1)
  resnet18     torchvision ResNet-18 topology at 224x224, Kaiming-normal convs, BN folded (config 3)
  mobilenet_v2 torchvision MobileNetV2 (width 1.0, ReLU6, inverted residuals), BN folded (config 4)
  transformer  decoder-only pre-LayerNorm transformer prefill, 12 x (768, 12 heads, MLP 3072 GELU),
               vocabulary 256 (config 5)

Weights depend only on `seed`, not on the batch size, so a network built at two batch sizes is the
same network.  `compile_w8a8` compiles through MIRA's own driver (mira/compiler.py compile_ir:
optimize, fuse_epilogues, quantize_w8a8 with host calibration, partition, target compile).
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np

from .hostfw import import_mira
from .plugin import install


def _ir():
    import_mira()
    from mira import ir
    from mira.types import TensorType
    return ir, TensorType


class _Net:
    def __init__(self, name: str, input_shape: tuple, seed: int):
        ir, TT = _ir()
        self.ir = ir
        self.x = ir.Value(TT("f32", tuple(input_shape)), name="x")
        self.g = ir.Graph(name, [self.x], [], [])
        self.rng = np.random.default_rng(seed)

    def const(self, arr):
        return self.g.const(np.asarray(arr, np.float32))

    def op(self, kind, inputs, attrs=None):
        return self.g.add(kind, list(inputs), attrs or {})

    def bn_fold(self, w: np.ndarray, cout: int, randomize: bool):
        """Fold an inference BatchNorm (eps 1e-5) into conv weights/bias."""
        if randomize:
            gamma = self.rng.uniform(0.7, 1.3, cout)
            beta = self.rng.normal(0.0, 0.1, cout)
            mean = self.rng.normal(0.0, 0.1, cout)
            var = self.rng.uniform(0.7, 1.3, cout)
        else:
            gamma, beta, mean, var = np.ones(cout), np.zeros(cout), np.zeros(cout), np.ones(cout)
        s = gamma / np.sqrt(var + 1e-5)
        return (w * s[:, None, None, None]).astype(np.float32), (beta - mean * s).astype(np.float32)

    def conv_bn(self, x, cin, cout, k, stride, pad, act=None, groups=1, randomize_bn=True):
        fan_out = cout * k * k // groups
        w = (self.rng.standard_normal((cout, cin // groups, k, k)) * np.sqrt(2.0 / fan_out)).astype(np.float32)
        w, b = self.bn_fold(w, cout, randomize_bn)
        attrs = {"stride": (stride, stride), "padding": (pad, pad)}
        if groups != 1:
            attrs["groups"] = groups
        y = self.op("conv2d", [x, self.const(w)], attrs)
        y = self.op("add", [y, self.const(b.reshape(cout, 1, 1))])
        if act == "relu":
            y = self.op("relu", [y])
        elif act == "relu6":
            y = self.op("maximum", [y, self.const(np.float32(0.0))])
            y = self.op("minimum", [y, self.const(np.float32(6.0))])
        return y

    def linear(self, x, fin, fout, bias=True, std=None):
        w = (self.rng.standard_normal((fin, fout)) * (std if std is not None else np.sqrt(2.0 / fin))).astype(np.float32)
        y = self.op("matmul", [x, self.const(w)])
        if bias:
            y = self.op("add", [y, self.const(self.rng.normal(0.0, 0.05, fout).astype(np.float32))])
        return y

    def finish(self, out):
        self.g.outputs = [out]
        self.g.verify()
        return self.g


def mlp(batch: int = 256, seed: int = 0):
    """Config 1: x f32[B, 784] -> 512 -> ReLU -> 512 -> ReLU -> 10, Kaiming-normal, zero biases
    (MIRA's simplify pass deletes the zero-bias adds, reference passes.py:56-57)."""
    n = _Net("mlp", (batch, 784), seed)
    h = n.x
    for fin, fout, act in ((784, 512, True), (512, 512, True), (512, 10, False)):
        w = (n.rng.standard_normal((fin, fout)) * np.sqrt(2.0 / fin)).astype(np.float32)
        h = n.op("matmul", [h, n.const(w)])
        h = n.op("add", [h, n.const(np.zeros(fout, np.float32))])
        if act:
            h = n.op("relu", [h])
    return n.finish(h)


def resnet18(batch: int = 1, seed: int = 0, image: int = 224, num_classes: int = 1000):
    """Config 3: ResNet-18 (BasicBlock x [2, 2, 2, 2]); stem 7x7/2 conv, -inf pad + 3x3/2 max pool,
    global mean, FC.  BN (random inference statistics) folded into each conv."""
    n = _Net("resnet18", (batch, 3, image, image), seed)
    y = n.conv_bn(n.x, 3, 64, 7, 2, 3, act="relu")
    y = n.op("pad", [y], {"pads": ((0, 0), (0, 0), (1, 1), (1, 1)), "value": -np.inf})
    y = n.op("maxpool2d", [y], {"size": 3, "stride": 2})
    cin = 64
    for cout, stride in ((64, 1), (128, 2), (256, 2), (512, 2)):
        for b in range(2):
            s = stride if b == 0 else 1
            out = n.conv_bn(y, cin, cout, 3, s, 1, act="relu")
            out = n.conv_bn(out, cout, cout, 3, 1, 1)
            short = n.conv_bn(y, cin, cout, 1, s, 0) if (s != 1 or cin != cout) else y
            y = n.op("relu", [n.op("add", [out, short])])
            cin = cout
    y = n.op("reduce_mean", [y], {"axes": (2, 3), "keepdims": False})
    y = n.linear(y, 512, num_classes, std=np.sqrt(1.0 / 512))
    return n.finish(y)


MBV2_SETTINGS = ((1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2), (6, 96, 3, 1), (6, 160, 3, 2),
                 (6, 320, 1, 1))


def mobilenet_v2(batch: int = 1, seed: int = 0, image: int = 224, num_classes: int = 1000):
    """Config 4: MobileNetV2 width 1.0: 3x3/2 stem, inverted residual blocks (expand 1x1, depthwise
    3x3, project 1x1; residual when stride 1 and channels match), 1x1 to 1280, mean, FC.  ReLU6 is
    maximum(., 0) then minimum(., 6), which MIRA fuses into the conv epilogues."""
    n = _Net("mobilenet_v2", (batch, 3, image, image), seed)
    y = n.conv_bn(n.x, 3, 32, 3, 2, 1, act="relu6")
    cin = 32
    for t, c, reps, s in MBV2_SETTINGS:
        for r in range(reps):
            stride = s if r == 0 else 1
            hidden = cin * t
            h = y
            if t != 1:
                h = n.conv_bn(h, cin, hidden, 1, 1, 0, act="relu6")
            h = n.conv_bn(h, hidden, hidden, 3, stride, 1, act="relu6", groups=hidden)
            h = n.conv_bn(h, hidden, c, 1, 1, 0)
            y = n.op("add", [y, h]) if (stride == 1 and cin == c) else h
            cin = c
    y = n.conv_bn(y, cin, 1280, 1, 1, 0, act="relu6")
    y = n.op("reduce_mean", [y], {"axes": (2, 3), "keepdims": False})
    y = n.linear(y, 1280, num_classes, std=np.sqrt(1.0 / 1280))
    return n.finish(y)


def transformer(batch: int = 1, seed: int = 0, seq: int = 1024, layers: int = 12, d_model: int = 768,
                heads: int = 12, d_mlp: int = 3072, vocab: int = 256, max_seq: int = 1024):
    """Config 5 prefill: decoder-only, pre-LayerNorm GPT block (the structure of the reference's
    examples/gpt.mira `block`, with heads): token embedding gather + learned positions, per layer
      x = layernorm(h); q, k, v = x @ Wq + bq, ...; heads via reshape/transpose;
      p = softmax(q @ k^T * (1/sqrt(dh)) + causal_mask); h = h + (p @ v) @ Wo + bo;
      h = h + gelu(layernorm(h) @ W1 + b1) @ W2 + b2,
    then a final layernorm and the LM head.  Weights and biases N(0, 0.02), layernorm gains
    1 + N(0, 0.02) and shifts N(0, 0.02); the mask is 0 on and below the diagonal and -10000 above
    (gpt.mira causal_mask).  Tables are drawn at `max_seq` rows so every `seq` sees the same weights."""
    return _gpt(batch, seed, seq, layers, d_model, heads, d_mlp, vocab, max_seq, step=False)


def transformer_step(batch: int = 1, seed: int = 0, layers: int = 12, d_model: int = 768, heads: int = 12,
                     d_mlp: int = 3072, vocab: int = 256, max_seq: int = 1024):
    """One decode step of the config-5 transformer (same weights as `transformer` with the same
    seed): one new token per sequence at a runtime position p, with a key/value cache per layer.

    Inputs: tok i32[B, 1]; pos2 i32[2] = (p, 0) and pos4 i32[4] = (0, 0, p, 0), the start vectors
    of the reference's runtime-position slices (ops.py:533-576); then k0, v0, k1, v1, ... f32[B,
    heads, max_seq, d_head], the caches holding positions < p.  The step reads the position row and
    the causal-mask row p with dynamic_slice, writes the new key and value at row p with
    dynamic_update_slice, and attends over all max_seq cache rows (rows after p are masked to
    -10000 like the prefill's upper triangle).  Outputs: logits f32[B, 1, vocab], then the
    updated caches in input order."""
    return _gpt(batch, seed, 1, layers, d_model, heads, d_mlp, vocab, max_seq, step=True)


def _gpt(batch, seed, seq, layers, d_model, heads, d_mlp, vocab, max_seq, step):
    ir, TT = _ir()
    if d_model % heads:
        raise ValueError("d_model must be a multiple of heads")
    if seq > max_seq:
        raise ValueError("seq must not exceed max_seq")
    dh = d_model // heads
    n = _Net.__new__(_Net)
    n.ir = ir
    n.x = ir.Value(TT("i32", (batch, seq)), name="tok")
    inputs = [n.x]
    if step:
        pos2 = ir.Value(TT("i32", (2,)), name="pos2")
        pos4 = ir.Value(TT("i32", (4,)), name="pos4")
        caches = [ir.Value(TT("f32", (batch, heads, max_seq, dh)), name=f"{kv}{l}")
                  for l in range(layers) for kv in ("k", "v")]
        inputs += [pos2, pos4] + caches
    n.g = ir.Graph("transformer_step" if step else "transformer", inputs, [], [])
    n.rng = np.random.default_rng(seed)
    std = 0.02

    def normal(*shape):
        return (n.rng.standard_normal(shape) * std).astype(np.float32)

    def ln(h):
        g = (1.0 + normal(d_model)).astype(np.float32)
        return n.op("layernorm", [h, n.const(g), n.const(normal(d_model))], {"eps": 1e-5})

    def dense(x, fin, fout, bias=True):
        y = n.op("matmul", [x, n.const(normal(fin, fout))])
        return n.op("add", [y, n.const(normal(fout))]) if bias else y

    emb = normal(vocab, d_model)
    pos_table = normal(max_seq, d_model)
    if step:
        causal = np.where(np.arange(max_seq)[:, None] >= np.arange(max_seq)[None, :], 0.0, -10000.0)
        pos = n.op("dynamic_slice", [n.const(pos_table), pos2], {"size": (1, d_model)})
        mask = n.op("dynamic_slice", [n.const(causal.astype(np.float32)), pos2], {"size": (1, max_seq)})
    else:
        pos = n.const(pos_table[:seq])
        mask = n.const(np.where(np.arange(seq)[:, None] >= np.arange(seq)[None, :], 0.0, -10000.0).astype(np.float32))
    h = n.op("add", [n.op("gather", [n.const(emb), n.x], {"axis": 0}), pos])
    new_caches = []
    for layer in range(layers):
        x = ln(h)
        q, k, v = (dense(x, d_model, d_model) for _ in range(3))
        split = lambda t: n.op("reshape", [t], {"shape": (batch, seq, heads, dh)})
        qh = n.op("transpose", [split(q)], {"perm": (0, 2, 1, 3)})
        if step:
            kc = n.op("dynamic_update_slice",
                      [caches[2 * layer], n.op("transpose", [split(k)], {"perm": (0, 2, 1, 3)}), pos4])
            vh = n.op("dynamic_update_slice",
                      [caches[2 * layer + 1], n.op("transpose", [split(v)], {"perm": (0, 2, 1, 3)}), pos4])
            kt = n.op("transpose", [kc], {"perm": (0, 1, 3, 2)})
            new_caches += [kc, vh]
        else:
            kt = n.op("transpose", [split(k)], {"perm": (0, 2, 3, 1)})
            vh = n.op("transpose", [split(v)], {"perm": (0, 2, 1, 3)})
        s = n.op("matmul", [qh, kt])
        s = n.op("mul", [s, n.const(np.float32(1.0 / np.sqrt(dh)))])
        s = n.op("add", [s, mask])
        o = n.op("matmul", [n.op("softmax", [s], {"axis": -1}), vh])
        o = n.op("reshape", [n.op("transpose", [o], {"perm": (0, 2, 1, 3)})], {"shape": (batch, seq, d_model)})
        h = n.op("add", [dense(o, d_model, d_model), h])
        m = n.op("gelu", [dense(ln(h), d_model, d_mlp)])
        h = n.op("add", [dense(m, d_mlp, d_model), h])
    logits = dense(ln(h), d_model, vocab, bias=False)
    n.g.outputs = [logits] + new_caches
    n.g.verify()
    return n.g


BUILDERS: dict[str, Callable] = {"mlp": mlp, "resnet18": resnet18, "mobilenet_v2": mobilenet_v2,
                                 "transformer": transformer}


def _vocab_of(graph, v, default: int = 256) -> int:
    """Rows of the embedding table that int32 input `v` indexes (by a gather), else `default`."""
    for op in graph.ops:
        if op.kind == "gather" and len(op.inputs) > 1 and op.inputs[1] is v:
            return int(op.inputs[0].type.shape[0])
    return default


def random_inputs(graph, seed: int) -> dict:
    """Seeded inputs keyed by input name: N(0, 1) for f32 (like the reference CLI's _inputs,
    cli.py:76-80), token ids uniform in [0, vocab) for i32 inputs that index an embedding."""
    rng = np.random.default_rng(seed)
    out = {}
    for v in graph.inputs:
        if v.type.dtype == "i32":
            out[v.name] = rng.integers(0, _vocab_of(graph, v), v.type.shape).astype(np.int32)
        else:
            out[v.name] = rng.standard_normal(v.type.shape).astype(np.float32)
    return out


# per-value calibration peaks of a (workload, seed, calibration batch/count/seed, builder options),
# in the order of the graph's quantizable ops: programs of one workload compiled at different batch
# sizes (or for different targets) with the same calibration share them, so their activation scales
# are identical and every per-image row of their outputs can be compared bit for bit
_PEAKS: dict = {}


def compile_w8a8(name: str, batch: int, target: str, *, seed: int = 0, n_calib: int = 4, calib_seed: int = 100,
                 calib_batch: Optional[int] = None, build_kw: Optional[dict] = None, int8_depthwise: bool = False,
                 **kw):
    """Build workload `name` at `batch` and compile it W8A8 for `target` through MIRA's compile_ir.

    Calibration feeds are `n_calib` seeded N(0, 1) batches.  With `calib_batch` (usually smaller
    than `batch`), calibration runs on the same network built at `calib_batch` - the reference's own
    _calibrate (quantize.py:73-92) over those feeds - and the resulting per-value peaks are carried
    over to the large graph op by op, so large batches do not pay hours of host-side calibration.
    Those peaks are computed once per process and calibration setting (`_PEAKS`).
    `int8_depthwise`: compile in the opt-in int8 depthwise mode (mira_b200.int8_depthwise)."""
    if int8_depthwise:
        from .depthwise import int8_depthwise as mode
        with mode():
            return _compile_w8a8(name, batch, target, seed, n_calib, calib_seed, calib_batch, build_kw, True, kw)
    return _compile_w8a8(name, batch, target, seed, n_calib, calib_seed, calib_batch, build_kw, False, kw)


def _compile_w8a8(name, batch, target, seed, n_calib, calib_seed, calib_batch, build_kw, dw_mode, kw):
    if target in ("cuda", "b200"):
        install()
    else:
        import_mira()
    from mira import compiler, passes
    from mira import quantize as Q
    build = BUILDERS[name]
    if build_kw:
        build = (lambda b, _f=build, **k: _f(b, **k, **build_kw))
    g = build(batch, seed=seed)
    if calib_batch is None:
        cal = [random_inputs(g, calib_seed + i) for i in range(n_calib)]
        return compiler.compile_ir(g, target, quantize="w8a8", calibration=cal, precision=None, **kw)
    small = build(calib_batch, seed=seed)
    passes.optimize(small, precision=None)
    passes.optimize(g, precision=None)

    def candidates(graph):
        return [op for op in graph.ops if op.kind in ("matmul", "conv2d") and Q._w8a8_weight(op) is not None]

    cs, cb = candidates(small), candidates(g)
    if len(cs) != len(cb):
        raise RuntimeError("small and large graphs differ in structure")
    key = (name, seed, calib_batch, n_calib, calib_seed, tuple(sorted((build_kw or {}).items())), dw_mode)
    if key not in _PEAKS:
        cal = [random_inputs(small, calib_seed + i) for i in range(n_calib)]
        peak_small = Q._calibrate(small, cal, {op.inputs[0] for op in cs})
        _PEAKS[key] = [peak_small[op.inputs[0]] for op in cs]
    pos_small = {v: i for i, v in enumerate(small.inputs + [r for op in small.ops for r in op.results])}
    big_values = g.inputs + [r for op in g.ops for r in op.results]
    peaks = {}
    for s_op, b_op, pk in zip(cs, cb, _PEAKS[key]):
        peaks[b_op.inputs[0]] = pk
        if pos_small.get(s_op.inputs[0]) is not None and big_values[pos_small[s_op.inputs[0]]] is not b_op.inputs[0]:
            raise RuntimeError("calibrated value does not map onto the large graph")
    original = Q._calibrate
    Q._calibrate = lambda graph, feeds, watch: {v: peaks[v] for v in watch}
    try:
        return compiler.compile_ir(g, target, optimize=False, quantize="w8a8", calibration=[{}], precision=None, **kw)
    finally:
        Q._calibrate = original
