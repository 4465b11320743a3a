"""Calibration-side quantisation rules (the producer of the NIRQ block).

These restate the reference's qparam derivations so that synthetic models built by
tests and bench.py carry the same kind of qparams a reference user would export:
  * compute_tensor_qparams      neuroflow/quant/static_quant.py:480-533
  * compute_per_channel_qparams neuroflow/quant/static_quant.py:536-589
  * _channel_axis_for_weight    neuroflow/quant/static_quant.py:837-852
  * compute_fp8_e4m3_qparams    neuroflow/quant/static_quant.py:338-352
  * calibrate(per_token=True)   neuroflow/quant/static_quant.py:658-717
The inference path never calls this module; it reads the qparams from the IR.
"""
from __future__ import annotations

import numpy as np

from .ir import FP8, PerChannel, PerTensor, PerToken

INT8_MIN, INT8_MAX = -128, 127


def tensor_qparams(t: np.ndarray) -> PerTensor:
    """Asymmetric per-tensor INT8 qparams with the zero-point clipping fix-up."""
    t = np.asarray(t, dtype=np.float32)
    t_min = float(t.min())
    t_max = float(t.max())
    if t_max == t_min or t_min != t_min or t_max != t_max:
        return PerTensor(1.0, 0)
    scale = (t_max - t_min) / (INT8_MAX - INT8_MIN)
    raw = np.round(INT8_MIN - t_min / scale)
    zp = int(np.clip(raw, INT8_MIN, INT8_MAX))
    if zp != raw:
        if zp == INT8_MIN:
            scale = (t_max - 0.0) / (INT8_MAX - INT8_MIN)
        else:
            scale = (0.0 - t_min) / (INT8_MAX - INT8_MIN)
    return PerTensor(float(np.float32(scale)), zp)


def per_channel_qparams(t: np.ndarray, channel_axis: int = 0) -> PerChannel:
    """Per-channel asymmetric INT8 qparams (one pair per slice of `channel_axis`)."""
    t = np.asarray(t, dtype=np.float32)
    moved = np.moveaxis(t, channel_axis, 0)
    flat = moved.reshape(moved.shape[0], -1)
    mins = flat.min(axis=1)
    maxs = flat.max(axis=1)
    spans = maxs - mins
    scales = np.where(spans > 0, spans / (INT8_MAX - INT8_MIN), 1.0).astype(np.float32)
    raw = np.round(INT8_MIN - mins / scales)
    zps = np.clip(raw, INT8_MIN, INT8_MAX).astype(np.int32)
    lo = zps == INT8_MIN
    hi = zps == INT8_MAX
    scales = np.where(lo & (maxs > 0), maxs / (INT8_MAX - INT8_MIN), scales).astype(np.float32)
    scales = np.where(hi & (mins < 0), -mins / (INT8_MAX - INT8_MIN), scales).astype(np.float32)
    return PerChannel(scales, zps, channel_axis)


def channel_axis_for_weight(name: str, ndim: int) -> int:
    if name.endswith(".weight") and ndim == 2:
        return 0
    if ("specs." in name or "weights_real" in name or "weights_imag" in name) and ndim == 3:
        return 1
    return 0


def fp8_qparams(t: np.ndarray) -> FP8:
    t_max = float(np.abs(np.asarray(t, np.float32)).max())
    if t_max != t_max or t_max == 0.0:
        return FP8(1.0)
    return FP8(float(t_max / 448.0))


def weight_qparams(weights: dict, per_channel: bool = True) -> dict:
    """quantise_model's weight loop (static_quant.py:900-914)."""
    out = {}
    for name, t in weights.items():
        if per_channel and t.ndim >= 1 and name.endswith((".weight", "weights_real",
                                                          "weights_imag")):
            out[name] = per_channel_qparams(t, channel_axis_for_weight(name, t.ndim))
        else:
            out[name] = tensor_qparams(t)
    return out


def quantise_rows(a: np.ndarray):
    """Per-row (per-token) INT8 codes: tensor_qparams applied to each row, then the
    runtime quantiser (round half away from zero, int8_gemm.cpp:514-518).
    Returns (codes int8 (M,K), scales f32 (M,), zero points i32 (M,))."""
    a = np.asarray(a, np.float32)
    mins = a.min(axis=1).astype(np.float64)
    maxs = a.max(axis=1).astype(np.float64)
    spans = maxs - mins
    const = spans <= 0
    scale = np.where(const, 1.0, spans / 255.0)
    raw = np.round(-128.0 - mins / np.where(const, 1.0, scale))
    zp = np.clip(raw, -128, 127)
    lo_clip = (zp != raw) & (zp == -128)
    hi_clip = (zp != raw) & (zp == 127)
    scale = np.where(lo_clip, maxs / 255.0, scale)
    scale = np.where(hi_clip, -mins / 255.0, scale)
    zp = np.where(const, 0, zp).astype(np.int32)
    scale = scale.astype(np.float32)
    # round half away from zero on the float32 quotient (std::round semantics); the
    # float64 floor(|q| + 0.5) is exact for every float32 |q| < 2**52.
    quo = (a / scale[:, None]).astype(np.float32).astype(np.float64)
    q = np.sign(quo) * np.floor(np.abs(quo) + 0.5)
    q = np.clip(q.astype(np.int64) + zp[:, None], -128, 127).astype(np.int8)
    return q, scale, zp


def quantise_weight_2d(W: np.ndarray, qp: PerChannel):
    """Per-output-row weight codes and sum_w[o] = sum_i (W_q[o,i] - zp[o]) (the rule of
    the reference's QuantiseWeight2D, cpp/src/fno.cpp:325-358)."""
    W = np.asarray(W, np.float32)
    s = np.asarray(qp.scales, np.float32)[:, None]
    zp = np.asarray(qp.zero_points, np.int32)
    quo = (W / s).astype(np.float32).astype(np.float64)
    q = np.sign(quo) * np.floor(np.abs(quo) + 0.5)
    q = (q.astype(np.float32) + zp[:, None].astype(np.float32))
    q = np.clip(q, -128, 127).astype(np.int8)
    sum_w = (q.astype(np.int32) - zp[:, None]).sum(axis=1).astype(np.int32)
    return q, sum_w


def gemm_case(seed: int, M: int, K: int, N: int):
    """Synthetic INT8 GEMM operands of the GEMM sweep: per-token (per-row) codes of
    N(0,1) activations, per-channel codes of Kaiming-uniform weights, fp32 bias."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K)).astype(np.float32)
    Aq, sA, zA = quantise_rows(a) if M > 0 else (np.zeros((0, K), np.int8),
                                                 np.zeros(0, np.float32), np.zeros(0, np.int32))
    bound = 1.0 / np.sqrt(K)
    W = rng.uniform(-bound, bound, (N, K)).astype(np.float32)
    bias = rng.uniform(-bound, bound, N).astype(np.float32)
    qp = per_channel_qparams(W, 0)
    Wq, sum_w = quantise_weight_2d(W, qp)
    return dict(Aq=Aq, sA=sA, zA=zA, Wq=Wq, sW=np.asarray(qp.scales, np.float32),
                zW=np.asarray(qp.zero_points, np.int32), sum_w=sum_w, bias=bias)


def per_token_qparams(stacked: np.ndarray) -> PerToken:
    """Per-token (per (n, w) element) INT8 qparams of a stacked (batch, n, w) Linear
    output: min/max over the batch axis, the per-channel rule per element, flattened
    row-major over (n, w)."""
    t = np.asarray(stacked, dtype=np.float32)
    _, n, w = t.shape
    mins = t.min(axis=0)
    maxs = t.max(axis=0)
    spans = maxs - mins
    scales = np.where(spans > 0, spans / (INT8_MAX - INT8_MIN), 1.0).astype(np.float32)
    raw = np.round(INT8_MIN - mins / scales)
    zps = np.clip(raw, INT8_MIN, INT8_MAX).astype(np.int32)
    lo = zps == INT8_MIN
    hi = zps == INT8_MAX
    scales = np.where(lo & (maxs > 0), maxs / (INT8_MAX - INT8_MIN), scales).astype(np.float32)
    scales = np.where(hi & (mins < 0), -mins / (INT8_MAX - INT8_MIN), scales).astype(np.float32)
    return PerToken(scales.reshape(-1), zps.reshape(-1), w)
