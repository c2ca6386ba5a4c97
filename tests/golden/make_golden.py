"""Generates the golden fixtures of tests/golden/ by running the reference itself (myramay/MIRA).

    python tests/golden/make_golden.py path/to/reference      (or set $MIRA_PATH)
    python tests/golden/make_golden.py path/to/reference --only-sequence   (sequence.npz alone)
    python tests/golden/make_golden.py path/to/reference --only-weight-only   (weight_only.npz alone)
    python tests/golden/make_golden.py path/to/reference --only-depthwise   (qdwconv2d.npz alone)

The reference (a pure-Python package) is imported from the given checkout.  Every expected value comes from the
reference's own code: mira.ops.evaluate for single ops (ops.py:602-634 quantized ops, 192-199
epilogues, 265-276 convolutions, 293-296 max pooling, 318-343 means, 469-470 pads),
mira.quantize.quantize_array (quantize.py:24-31), and mira.compiler.compile_ir(..., "cpu",
quantize="w8a8") for whole programs (the cpu golden model).  Inputs are seeded.  The fixtures are
small .npz files; the tests never need the reference checkout to read them.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def _import_reference(path: str):
    sys.path.insert(0, path)
    import mira  # noqa: F401
    from mira import compiler, ir, ops, quantize
    return mira, compiler, ir, ops, quantize


def _save(name: str, **arrays) -> None:
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"wrote {name}.npz ({(HERE / f'{name}.npz').stat().st_size / 1024:.1f} KiB)")


def _epi_arrays(steps):
    """Encode an epilogue ((fn, idx, swapped), ...) as parallel arrays for the fixture."""
    fns = np.array([f for f, _, _ in steps], dtype="U16")
    idx = np.array([-1 if i is None else i for _, i, _ in steps], np.int64)
    sw = np.array([bool(s) for _, _, s in steps], np.bool_)
    return fns, idx, sw


def main(ref_path: str) -> None:
    mira, compiler, ir, O, Q = _import_reference(ref_path)
    rng = np.random.default_rng(20261201)

    # ---- quantize_activation (ops.py:602-603): ties, extremes, signed zero
    scales = np.array([0.0123, 1.0, 0.5, 3.0e-3, 1.0 / 127.0], np.float64)
    xs, qs = [], []
    for s in scales:
        x = (rng.standard_normal(4000) * 80 * s).astype(np.float32)
        x[::5] = ((rng.integers(-140, 140, x.size)[::5] + 0.5) * np.float32(s)).astype(np.float32)
        x[1::97] = np.float32(1e30)
        x[2::97] = np.float32(-1e30)
        x[3::97] = np.float32(-0.0)
        xs.append(x)
        qs.append(O.quantize_activation(x, float(s)))
    _save("quantize_activation", scales=scales, x=np.stack(xs), q=np.stack(qs).astype(np.int8))

    # ---- quantize_array (quantize.py:24-31)
    w = rng.standard_normal((96, 40)).astype(np.float32)
    w[:, 3] = 0.0
    q1, s1 = Q.quantize_array(w, 1)
    wc = rng.standard_normal((24, 8, 3, 3)).astype(np.float32)
    q0, s0 = Q.quantize_array(wc, 0)
    _save("quantize_array", w=w, q_axis1=q1, s_axis1=s1, wc=wc, q_axis0=q0, s_axis0=s0)

    # ---- qmatmul (ops.py:616-620) with epilogues (ops.py:192-199)
    cases = {}
    specs = [
        ((37, 100), 70, ()),
        ((2, 5, 64), 48, (("add", 1, False), ("relu", None, False))),
        ((16, 96), 33, (("add", 1, False), ("add", 2, True), ("relu", None, False))),
        ((8, 32), 16, (("maximum", 1, False), ("minimum", 2, False))),
        ((12, 40), 24, (("mul", 1, False), ("sub", 2, True), ("div", 3, False))),
    ]
    for i, (xshape, n, steps) in enumerate(specs):
        x = rng.standard_normal(xshape).astype(np.float32)
        k = xshape[-1]
        qw, ws = Q.quantize_array(rng.standard_normal((k, n)).astype(np.float32), 1)
        x_scale = float(np.abs(x).max() / 127.0)
        operands = []
        for fn, idx, _ in steps:
            if idx is None:
                continue
            if fn in ("maximum",):
                operands.append(np.asarray(np.float32(0.0)))
            elif fn in ("minimum",):
                operands.append(np.asarray(np.float32(6.0)))
            elif idx == 2 and fn == "add":
                operands.append(rng.standard_normal(xshape[:-1] + (n,)).astype(np.float32))
            elif fn == "div":
                operands.append(rng.uniform(0.5, 2.0, n).astype(np.float32))
            else:
                operands.append(rng.standard_normal(n).astype(np.float32))
        attrs = {"q": qw, "w_scale": ws, "x_scale": x_scale, "dtype": "f32"}
        if steps:
            attrs["epilogue"] = steps
        y = O.evaluate("qmatmul", [x] + operands, attrs)
        fns, idx, sw = _epi_arrays(steps)
        cases.update({f"c{i}_x": x, f"c{i}_q": qw, f"c{i}_w_scale": ws, f"c{i}_x_scale": np.float64(x_scale),
                      f"c{i}_fns": fns, f"c{i}_idx": idx, f"c{i}_sw": sw, f"c{i}_y": y,
                      f"c{i}_n_operands": np.int64(len(operands))})
        for j, o in enumerate(operands):
            cases[f"c{i}_op{j}"] = o
    _save("qmatmul", n_cases=np.int64(len(specs)), **cases)

    # ---- qconv2d (ops.py:630-634 through _conv2d_ref 265-276)
    cases = {}
    cspecs = [
        dict(n=2, c=3, h=17, w=15, o=8, k=7, s=2, p=3, d=1, epi="bias_relu"),
        dict(n=2, c=16, h=10, w=10, o=24, k=3, s=1, p=1, d=1, epi="bias_res_relu"),
        dict(n=1, c=32, h=9, w=11, o=16, k=1, s=2, p=0, d=1, epi="bias"),
        dict(n=2, c=8, h=12, w=12, o=8, k=3, s=1, p=2, d=2, epi="relu6"),
        dict(n=1, c=5, h=7, w=7, o=4, k=3, s=2, p=1, d=1, epi="none"),
    ]
    for i, cs in enumerate(cspecs):
        x = rng.standard_normal((cs["n"], cs["c"], cs["h"], cs["w"])).astype(np.float32)
        qw, ws = Q.quantize_array(rng.standard_normal((cs["o"], cs["c"], cs["k"], cs["k"])).astype(np.float32), 0)
        x_scale = float(np.abs(x).max() / 127.0)
        attrs = {"stride": (cs["s"], cs["s"]), "padding": (cs["p"], cs["p"]), "q": qw, "w_scale": ws,
                 "x_scale": x_scale, "dtype": "f32"}
        if cs["d"] != 1:
            attrs["dilation"] = (cs["d"], cs["d"])
        oh = (cs["h"] + 2 * cs["p"] - cs["d"] * (cs["k"] - 1) - 1) // cs["s"] + 1
        ow = (cs["w"] + 2 * cs["p"] - cs["d"] * (cs["k"] - 1) - 1) // cs["s"] + 1
        bias = rng.standard_normal((cs["o"], 1, 1)).astype(np.float32)
        res = rng.standard_normal((cs["n"], cs["o"], oh, ow)).astype(np.float32)
        if cs["epi"] == "bias_relu":
            steps, operands = (("add", 1, False), ("relu", None, False)), [bias]
        elif cs["epi"] == "bias_res_relu":
            steps, operands = (("add", 1, False), ("add", 2, True), ("relu", None, False)), [bias, res]
        elif cs["epi"] == "bias":
            steps, operands = (("add", 1, False),), [bias]
        elif cs["epi"] == "relu6":
            steps = (("add", 1, False), ("maximum", 2, False), ("minimum", 3, False))
            operands = [bias, np.asarray(np.float32(0)), np.asarray(np.float32(6))]
        else:
            steps, operands = (), []
        if steps:
            attrs["epilogue"] = steps
        y = O.evaluate("qconv2d", [x] + operands, attrs)
        fns, idx, sw = _epi_arrays(steps)
        cases.update({f"c{i}_x": x, f"c{i}_q": qw, f"c{i}_w_scale": ws, f"c{i}_x_scale": np.float64(x_scale),
                      f"c{i}_geom": np.array([cs["s"], cs["p"], cs["d"]], np.int64), f"c{i}_fns": fns,
                      f"c{i}_idx": idx, f"c{i}_sw": sw, f"c{i}_y": y, f"c{i}_n_operands": np.int64(len(operands))})
        for j, o in enumerate(operands):
            cases[f"c{i}_op{j}"] = o
    _save("qconv2d", n_cases=np.int64(len(cspecs)), **cases)

    # ---- f32 ops between the quantized ones
    x = np.maximum(rng.standard_normal((2, 8, 13, 13)), 0).astype(np.float32)
    padded = O.evaluate("pad", [x], {"pads": ((0, 0), (0, 0), (1, 1), (1, 1)), "value": -np.inf})
    pooled = O.evaluate("maxpool2d", [padded], {"size": 3, "stride": 2})
    pooled2 = O.evaluate("maxpool2d", [x], {"size": 2, "stride": 2})
    xm = (rng.standard_normal((3, 24, 7, 7)) * 4).astype(np.float32)
    xm2 = rng.standard_normal((2, 16, 14, 14)).astype(np.float32)
    mean = O.evaluate("reduce_mean", [xm], {"axes": (2, 3), "keepdims": False})
    mean2 = O.evaluate("reduce_mean", [xm2], {"axes": (2, 3), "keepdims": True})
    xd = rng.standard_normal((2, 12, 11, 11)).astype(np.float32)
    wd = rng.standard_normal((12, 1, 3, 3)).astype(np.float32)
    bd = rng.standard_normal((12, 1, 1)).astype(np.float32)
    dw1 = O.evaluate("conv2d", [xd, wd], {"stride": (1, 1), "padding": (1, 1), "groups": 12})
    dw2 = O.evaluate("conv2d", [xd, wd, bd, np.float32(0), np.float32(6)],
                     {"stride": (2, 2), "padding": (1, 1), "groups": 12,
                      "epilogue": (("add", 2, False), ("maximum", 3, False), ("minimum", 4, False))})
    _save("f32_ops", pool_x=x, pool_pad_3_2=pooled, pool_2_2=pooled2, mean_x=xm, mean=mean, mean_x2=xm2,
          mean2=mean2, dw_x=xd, dw_w=wd, dw_b=bd, dw_s1=dw1, dw_s2_relu6=dw2)

    # ---- whole W8A8 programs on the reference cpu target (the golden model)
    sys.path.insert(0, str(ROOT))
    from mira_b200 import configs
    progs = {}
    for name, batch, kw, n_cal in (("mlp", 16, {}, 8), ("resnet18", 2, {"image": 32}, 2),
                                   ("mobilenet_v2", 2, {"image": 32}, 2)):
        g = configs.BUILDERS[name](batch, **kw)
        cal = [configs.random_inputs(g, 100 + i) for i in range(n_cal)]
        prog = compiler.compile_ir(g, "cpu", quantize="w8a8", calibration=cal, precision=None)
        feeds = configs.random_inputs(g, 1)
        out = prog.run(feeds)
        scales = np.array([op.attrs["x_scale"] for op in prog.graph.ops if op.kind in ("qmatmul", "qconv2d")])
        progs.update({f"{name}_x": feeds["x"], f"{name}_out": out, f"{name}_x_scales": scales,
                      f"{name}_batch": np.int64(batch), f"{name}_n_calib": np.int64(n_cal)})
        progs[f"{name}_image"] = np.int64(kw.get("image", 0))
    _save("programs", **progs)
    sequence(ref_path)
    weight_only(ref_path)


TINY_TRANSFORMER = dict(seq=16, layers=2, d_model=64, heads=4, d_mlp=128, vocab=32, max_seq=16)


def sequence(ref_path: str) -> None:
    """sequence.npz: the f32 ops of the transformer path through mira.ops.evaluate (layernorm
    ops.py:356-360, softmax 310-313, matmul with epilogue 217-219, gather 482-487) and a small
    W8A8 transformer program on the reference cpu target."""
    mira, compiler, ir, O, Q = _import_reference(ref_path)
    rng = np.random.default_rng(20261202)
    out = {}
    for d in (768, 100, 5):
        x = (rng.standard_normal((6, d)) * rng.uniform(0.1, 5, (6, 1)) + rng.normal(0, 2, (6, 1))).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        b = (0.1 * rng.standard_normal(d)).astype(np.float32)
        out.update({f"ln{d}_x": x, f"ln{d}_g": g, f"ln{d}_b": b,
                    f"ln{d}_y": O.evaluate("layernorm", [x, g, b], {"eps": 1e-5})})
    s = (rng.standard_normal((6, 1024)) * 3).astype(np.float32)
    s[:, 700:] -= np.float32(10000)
    out.update({"sm_x": s, "sm_y": O.evaluate("softmax", [s], {"axis": -1})})
    q = rng.standard_normal((2, 3, 16, 8)).astype(np.float32)
    kt = rng.standard_normal((2, 3, 8, 16)).astype(np.float32)
    mask = np.where(np.arange(16)[:, None] >= np.arange(16)[None, :], 0.0, -10000.0).astype(np.float32)
    out.update({"mm_a": q, "mm_b": kt, "mm_mask": mask,
                "mm_y": O.evaluate("matmul", [q, kt, np.float32(0.125), mask],
                                   {"epilogue": (("mul", 2, False), ("add", 3, False))})})
    table = rng.standard_normal((32, 16)).astype(np.float32)
    idx = rng.integers(-32, 32, (2, 5)).astype(np.int32)
    out.update({"ga_table": table, "ga_idx": idx, "ga_y": O.evaluate("gather", [table, idx], {"axis": 0})})

    sys.path.insert(0, str(ROOT))
    from mira_b200 import configs
    g = configs.transformer(2, **TINY_TRANSFORMER)
    cal = [configs.random_inputs(g, 100 + i) for i in range(2)]
    prog = compiler.compile_ir(g, "cpu", quantize="w8a8", calibration=cal, precision=None)
    feeds = configs.random_inputs(g, 1)
    out.update({"tf_tok": feeds["tok"], "tf_out": prog.run(feeds),
                "tf_x_scales": np.array([op.attrs["x_scale"] for op in prog.graph.ops if op.kind == "qmatmul"])})
    _save("sequence", **out)


def weight_only(ref_path: str) -> None:
    """weight_only.npz: the `dequantize` constant (ops.py:583-587) of weights quantized by
    quantize_array (quantize.py:24-31) along either axis, and whole programs compiled with
    quantize="int8" (quantize.py:45-68) on the reference cpu target."""
    mira, compiler, ir, O, Q = _import_reference(ref_path)
    rng = np.random.default_rng(20261203)
    out = {}
    w = (rng.standard_normal((96, 40)) * rng.uniform(0.01, 3, (1, 40))).astype(np.float32)
    w[:, 7] = 0.0                                    # an all-zero column: scale 1.0
    for axis in (0, 1):
        q, s = Q.quantize_array(w, axis)
        out.update({f"q_axis{axis}": q, f"s_axis{axis}": s,
                    f"w_axis{axis}": O.evaluate("dequantize", [], {"q": q, "scale": s, "axis": axis, "dtype": "f32"})})
    sys.path.insert(0, str(ROOT))
    from mira_b200 import configs
    for name, batch, kw in (("mlp", 8, {}), ("transformer", 2, TINY_TRANSFORMER)):
        g = configs.BUILDERS[name](batch, **kw)
        prog = compiler.compile_ir(g, "cpu", quantize="int8", precision=None)
        feeds = configs.random_inputs(g, 1)
        key = next(iter(feeds))
        out.update({f"{name}_in": feeds[key], f"{name}_out": prog.run(feeds),
                    f"{name}_n_dequantize": np.int64(sum(op.kind == "dequantize" for op in prog.graph.ops))})
    _save("weight_only", **out)


def depthwise(ref_path: str) -> None:
    """qdwconv2d.npz: the reference's qconv2d (ops.py:630-634) with groups == channels, the op the
    opt-in int8 depthwise mode creates, evaluated by mira.ops.evaluate; and MobileNetV2 compiled in
    that mode (mira_b200.int8_depthwise around compile_ir) on the reference cpu target."""
    mira, compiler, ir, O, Q = _import_reference(ref_path)
    rng = np.random.default_rng(20261204)
    cases = {}
    cspecs = [
        dict(n=2, c=32, h=13, w=11, k=3, s=1, p=1, d=1, epi="bias_relu6"),
        dict(n=2, c=96, h=12, w=12, k=3, s=2, p=1, d=1, epi="bias_relu6"),
        dict(n=1, c=16, h=9, w=10, k=5, s=1, p=2, d=1, epi="bias"),
        dict(n=1, c=8, h=10, w=10, k=3, s=1, p=2, d=2, epi="none"),
        dict(n=2, c=12, h=7, w=9, k=3, s=2, p=0, d=1, epi="bias_relu6"),
    ]
    for i, cs in enumerate(cspecs):
        x = rng.standard_normal((cs["n"], cs["c"], cs["h"], cs["w"])).astype(np.float32)
        qw, ws = Q.quantize_array(rng.standard_normal((cs["c"], 1, cs["k"], cs["k"])).astype(np.float32), 0)
        x_scale = float(np.abs(x).max() / 127.0)
        attrs = {"stride": (cs["s"], cs["s"]), "padding": (cs["p"], cs["p"]), "groups": cs["c"], "q": qw,
                 "w_scale": ws, "x_scale": x_scale, "dtype": "f32"}
        if cs["d"] != 1:
            attrs["dilation"] = (cs["d"], cs["d"])
        bias = rng.standard_normal((cs["c"], 1, 1)).astype(np.float32)
        if cs["epi"] == "bias_relu6":
            steps = (("add", 1, False), ("maximum", 2, False), ("minimum", 3, False))
            operands = [bias, np.asarray(np.float32(0)), np.asarray(np.float32(6))]
        elif cs["epi"] == "bias":
            steps, operands = (("add", 1, False),), [bias]
        else:
            steps, operands = (), []
        if steps:
            attrs["epilogue"] = steps
        y = O.evaluate("qconv2d", [x] + operands, attrs)
        fns, idx, sw = _epi_arrays(steps)
        cases.update({f"c{i}_x": x, f"c{i}_q": qw, f"c{i}_w_scale": ws, f"c{i}_x_scale": np.float64(x_scale),
                      f"c{i}_geom": np.array([cs["s"], cs["p"], cs["d"]], np.int64), f"c{i}_fns": fns,
                      f"c{i}_idx": idx, f"c{i}_sw": sw, f"c{i}_y": y, f"c{i}_n_operands": np.int64(len(operands))})
        for j, o in enumerate(operands):
            cases[f"c{i}_op{j}"] = o
    sys.path.insert(0, str(ROOT))
    from mira_b200 import configs
    from mira_b200.depthwise import int8_depthwise
    g = configs.BUILDERS["mobilenet_v2"](2, image=32)
    cal = [configs.random_inputs(g, 100 + i) for i in range(2)]
    with int8_depthwise():
        prog = compiler.compile_ir(g, "cpu", quantize="w8a8", calibration=cal, precision=None)
    feeds = configs.random_inputs(g, 1)
    cases.update({"mbv2_in": feeds["x"], "mbv2_out": prog.run(feeds),
                  "mbv2_n_grouped_qconv": np.int64(sum(op.kind == "qconv2d" and op.attrs.get("groups", 1) != 1
                                                       for op in prog.graph.ops))})
    _save("qdwconv2d", n_cases=np.int64(len(cspecs)), **cases)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    path = args[0] if args else os.environ.get("MIRA_PATH")
    if not path:
        raise SystemExit("usage: make_golden.py path/to/reference [--only-sequence|--only-weight-only] (or set MIRA_PATH)")
    if "--only-sequence" in sys.argv:
        sequence(path)
    elif "--only-weight-only" in sys.argv:
        weight_only(path)
    elif "--only-depthwise" in sys.argv:
        depthwise(path)
    else:
        main(path)
