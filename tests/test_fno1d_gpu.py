"""FNO1d executor on the GPU vs the CPU restatement of FNO1d::Forward (oracle, itself
pinned bit-exact against the reference runtime).

* ReLU models: every operation on the path is reproduced with the reference's
  rounding (radix-2 FFT with the recurrence twiddles, contraction, Linear dot products,
  INT8 LinearForwardBatched, fake-quant), so the GPU output is BIT-IDENTICAL.
* GELU models: tanhf is CUDA's where its result is consumed as fp32 (glibc's and
  CUDA's tanhf differ by a few ulps); where GELU feeds a per-tensor snap the exact
  code table is used.  Tolerances are stated per case below.
"""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, synth
from oracle.cpu import Oracle

VARIANTS = {
    "plain": dict(quantised=False),
    "per_token": dict(per_token=True),
    "per_tensor": dict(per_token=False),
    "per_tensor_weights": dict(per_token=False, per_channel=False),
}


def _model(tmp_path, name, act="gelu", width=32, modes=8, L=3, n=128, pad_factor=0, seed=5):
    m = synth.fno1d_model(seed, width=width, modes=modes, L=L, n=n, n_calib=8,
                          pad_factor=pad_factor, **VARIANTS[name])
    m.activation = act
    p = os.path.join(str(tmp_path), f"fno1d_{name}_{act}.nneuroir")
    ir.write(p, m)
    return m, p


def _run(path, x, out_ch, int8):
    from neuroflow_b200.runtime import InferenceRuntime
    rt = InferenceRuntime(path)
    if int8:
        rt.enable_int8_gemm()
    y = np.zeros(x.shape[:-1] + (out_ch,), np.float32)
    rt.run(x, y)
    return y


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(VARIANTS))
@pytest.mark.parametrize("int8", [False, True])
def test_fno1d_relu_bit_exact(tmp_path, name, int8):
    m, p = _model(tmp_path, name, act="relu")
    x = synth.fno1d_inputs(np.random.default_rng(2), 3, 128)
    want = Oracle().fno1d_forward(m, x, int8=int8)
    got = _run(p, x, 1, int8)
    assert np.array_equal(_bits(got), _bits(want)), float(np.abs(got - want).max())


@pytest.mark.gpu
def test_fno1d_relu_bit_exact_padded_and_wide(tmp_path):
    # padding (n = 48 -> 64 is not a power of two in the reference, so use 32 -> 64),
    # width 64 with the tcgen05 INT8 GEMM, modes up to n/2 + 1
    m, p = _model(tmp_path, "per_tensor", act="relu", width=64, modes=17, L=2, n=32,
                  pad_factor=64)
    x = synth.fno1d_inputs(np.random.default_rng(3), 2, 32)
    for int8 in (False, True):
        want = Oracle().fno1d_forward(m, x, int8=int8)
        got = _run(p, x, 1, int8)
        assert np.array_equal(_bits(got), _bits(want)), (int8, float(np.abs(got - want).max()))


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(VARIANTS))
def test_fno1d_gelu_close(tmp_path, name):
    """GELU: differences come only from tanhf ulps.  Without per-element snaps the
    outputs agree to rtol 1e-5; per-token snaps can flip a code where a value sits on a
    rounding boundary, so there the bound is on the fraction of moved outputs."""
    m, p = _model(tmp_path, name, width=64, modes=16, L=4, n=1024)
    x = synth.fno1d_inputs(np.random.default_rng(4), 4, 1024)
    for int8 in (False, True):
        want = Oracle().fno1d_forward(m, x, int8=int8)
        got = _run(p, x, 1, int8)
        d = np.abs(got - want)
        tol = 1e-5 * np.abs(want) + 1e-6 * np.abs(want).max()
        frac = float(np.mean(d > tol))
        print(name, int8, float(d.max()), frac)
        assert np.all(np.isfinite(got))
        if name == "per_token":
            assert frac < 0.02, (frac, float(d.max()))
            assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-3
        else:
            assert frac == 0.0, (frac, float(d.max()))


@pytest.mark.gpu
def test_fno1d_configs0_shape_int8(tmp_path):
    """configs[0] geometry (width 64, 16 modes, 4 layers, n = 1024) with per-tensor
    activations and EnableInt8Gemm (the reference's INT8 dispatch), GELU."""
    m, p = _model(tmp_path, "per_tensor", width=64, modes=16, L=4, n=1024)
    x = synth.fno1d_inputs(np.random.default_rng(6), 8, 1024)
    want = Oracle().fno1d_forward(m, x, int8=True)
    got = _run(p, x, 1, True)
    assert np.allclose(got, want, rtol=1e-5, atol=1e-6 * np.abs(want).max())


@pytest.mark.gpu
def test_fno1d_errors_and_flags(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    _, p = _model(tmp_path, "plain", L=1, n=64)
    rt = InferenceRuntime(p)
    assert rt.op() == "FNO1d"
    assert not rt.is_int8_gemm_enabled()
    rt.enable_int8_gemm()  # the reference sets the flag whatever the IR holds
    assert rt.is_int8_gemm_enabled()
    x = np.zeros((1, 64, 2), np.float32)
    with pytest.raises(RuntimeError, match="expected 3D input"):
        rt.run(np.zeros((64, 2), np.float32), np.zeros((64, 1), np.float32))
    with pytest.raises(RuntimeError, match="input channels mismatch"):
        rt.run(np.zeros((1, 64, 3), np.float32), np.zeros((1, 64, 1), np.float32))
    with pytest.raises(RuntimeError, match="output buffer shape mismatch"):
        rt.run(x, np.zeros((1, 32, 1), np.float32))
    with pytest.raises(RuntimeError, match="power of two"):
        rt.run(np.zeros((1, 48, 2), np.float32), np.zeros((1, 48, 1), np.float32))
    y = np.ones((0, 64, 1), np.float32)
    rt.run(np.zeros((0, 64, 2), np.float32), y)  # empty batch


@pytest.mark.gpu
def test_fno1d_growing_batch_reuses_handle(tmp_path):
    m, p = _model(tmp_path, "per_tensor", act="relu", n=64)
    from neuroflow_b200.runtime import InferenceRuntime
    rt = InferenceRuntime(p)
    rt.enable_int8_gemm()
    o = Oracle()
    for B in (1, 3, 2, 5):
        x = synth.fno1d_inputs(np.random.default_rng(B), B, 64)
        y = np.zeros((B, 64, 1), np.float32)
        rt.run(x, y)
        assert np.array_equal(_bits(y), _bits(o.fno1d_forward(m, x, int8=True))), B


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["pt", "pc"])
def test_fno1d_reference_exported_models(tag):
    """Models calibrated and exported by the reference's Python package, against the
    reference C++ runtime's own outputs (tests/golden, made by make_golden.py)."""
    gold = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    d = np.load(os.path.join(gold, "fno1d.npz"))
    path = os.path.join(gold, f"fno1d_{tag}.nneuroir")
    for int8 in (False, True):
        want = d[f"y_{tag}_int8" if int8 else f"y_{tag}"]
        got = _run(path, d["x"], 1, int8)
        diff = np.abs(got - want)
        tol = 1e-5 * np.abs(want) + 1e-6 * np.abs(want).max()
        assert np.mean(diff > tol) <= (0.02 if tag == "pt" else 0.0), (int8, float(diff.max()))


@pytest.mark.gpu
@pytest.mark.parametrize("width", [16, 20, 48])
def test_fno1d_relu_bit_exact_untiled_widths(tmp_path, width):
    """INT8 local layers at widths the tcgen05 GEMM does not tile run the same integer
    arithmetic on CUDA cores; FP32 dot products with vector tails (width 20)."""
    m, p = _model(tmp_path, "per_tensor", act="relu", width=width, modes=6, L=2, n=64)
    x = synth.fno1d_inputs(np.random.default_rng(8), 2, 64)
    for int8 in (False, True):
        want = Oracle().fno1d_forward(m, x, int8=int8)
        got = _run(p, x, 1, int8)
        assert np.array_equal(_bits(got), _bits(want)), (int8, float(np.abs(got - want).max()))
