"""Opt-in int8 depthwise mode.

MIRA's W8A8 pass leaves grouped convolutions in float32: `_w8a8_weight` (mira/quantize.py:95-115)
returns None for `groups != 1` (line 105-106), so MobileNetV2's depthwise layers stay f32 and the
1x1 convolutions around them write and read f32 activations.  Inside `int8_depthwise()` the pass
also quantizes depthwise convolutions (groups == input channels == output channels, one weight per
channel and tap): their weights per output channel exactly as for ungrouped convs
(`quantize_array(w, 0)`, quantize.py:24-31), their input at a calibrated activation scale, and
`quantize_w8a8` (quantize.py:118-143) turns them into `qconv2d` ops that keep their `groups`
attribute.  Nothing else changes.

The reference itself evaluates such an op: `_qconv2d_ref` (mira/ops.py:630-634) runs the grouped
`_conv2d_ref` (265-276) on the quantized operands, so a cpu program compiled inside the same
context is the bit-exact oracle of the cuda program (the cuda target runs these ops with
`mira_cuda_qdwconv2d_nhwc`).  The results differ from the default mode's by the quantization of
the depthwise input and weights; that is the point of the opt-in.

    from mira_b200 import int8_depthwise
    with int8_depthwise():
        prog = mira.compiler.compile_ir(g, "cuda", quantize="w8a8", calibration=feeds)
"""
from __future__ import annotations

import contextlib
from typing import Optional

import numpy as np

from .hostfw import import_mira


def depthwise_weight(op, quantize_array) -> Optional[tuple[np.ndarray, np.ndarray]]:
    """(int8 weights [c, 1, kh, kw], per-channel scales) of a depthwise conv2d with constant
    weights, else None."""
    if op.kind != "conv2d":
        return None
    groups = op.attrs.get("groups", 1)
    x = op.inputs[0]
    w = op.inputs[1].producer
    if groups == 1 or x.type.rank != 4 or w is None or not w.is_constant_like:
        return None
    wshape = tuple(op.inputs[1].type.shape)
    if len(wshape) != 4 or groups != x.type.shape[1] or wshape[0] != groups or wshape[1] != 1:
        return None
    if w.kind == "dequantize" and w.attrs["axis"] == 0:
        return w.attrs["q"], w.attrs["scale"]
    value = w.attrs["value"] if w.is_const else None
    if value is None:
        return None
    return quantize_array(value, 0)


@contextlib.contextmanager
def int8_depthwise():
    """While active, MIRA's W8A8 quantization also turns depthwise convolutions into int8 qconv2d."""
    import_mira()
    from mira import quantize as Q
    original = Q._w8a8_weight

    def weight(op):
        got = original(op)
        if got is not None:
            return got
        return depthwise_weight(op, Q.quantize_array)

    Q._w8a8_weight = weight
    try:
        yield
    finally:
        Q._w8a8_weight = original
