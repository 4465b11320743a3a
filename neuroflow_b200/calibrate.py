"""Quantise an FNO2d IR with activation statistics gathered on the GPU: the counterpart
of the reference's quantise_model + quant_to_ir (neuroflow/quant/static_quant.py:855-935,
neuroflow/ir/export.py:600-642) for calibration sets too large for host hooks.

    from neuroflow_b200.calibrate import quantise_fno2d
    quantise_fno2d("fp32.nneuroir", batches, "int8.nneuroir", percentile=100.0)

The activation qparams of every Linear output (lift, locs.i, proj_q, proj_out) come
from the GPU runtime (InferenceRuntime.calibrate_*, nfx_calibrate_* in libnfx.so); the
weight qparams are computed on the host from the weights, as the reference does
(per channel along the reference's channel axis, or per tensor).
"""
from __future__ import annotations

from typing import Iterable

import numpy as np

from . import ir, quant
from .runtime import InferenceRuntime


def calibrate_fno2d(ir_path: str, batches: Iterable[np.ndarray], percentile: float = 100.0,
                    device: int = 0) -> dict:
    """{".output" key: (scale, zero_point, fp8_scale, lo, hi)} over all batches."""
    rt = InferenceRuntime(ir_path, device)
    try:
        rt.calibrate_begin(keep_values=percentile < 100.0)
        for x in batches:
            rt.calibrate_observe(x)
        return rt.calibrate_results(percentile)
    finally:
        rt.calibrate_end()
        rt.close()


def quantise_fno2d(ir_path: str, batches: Iterable[np.ndarray], out_path: str,
                   percentile: float = 100.0, per_channel_weights: bool = True,
                   fp8_activations: bool = False, device: int = 0) -> ir.Model:
    """Write `out_path`: the FP32 IR's weights with a NIRQ block of GPU-calibrated
    activation qparams (and FP8 E4M3 scales when `fp8_activations`)."""
    m = ir.read(ir_path)
    if m.op != "FNO2d":
        raise RuntimeError("quantise_fno2d: model op is " + m.op)
    acts = calibrate_fno2d(ir_path, batches, percentile, device)
    qp = quant.weight_qparams(m.weights, per_channel=per_channel_weights)
    for key, (scale, zp, f8, _, _) in acts.items():
        qp[key] = ir.PerTensor(float(scale), int(zp))
    if fp8_activations:
        # quant_to_ir (static_quant.py:1131-1139): the FP8 entry replaces the INT8 one
        for key, (_, _, f8, _, _) in acts.items():
            qp[key] = ir.FP8(float(f8))
    m.qparams = qp
    m.quant_enabled = True
    ir.write(out_path, m)
    return m
