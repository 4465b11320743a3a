"""FNO2d FP32 fake-quant executor (the reference's Run without EnableInt8Gemm) on the
GPU vs the CPU restatement (oracle mode 0, pinned bit-exact against the reference).

ReLU models are bit-identical: the row/column radix-2 transforms with the reference's
twiddle recurrence, the contraction, the Linear dot products and the fake-quant are
reproduced with the reference's rounding.  GELU models differ only through CUDA's
tanhf (a few ulps), which a fake-quant boundary may turn into one quantisation step
for an element sitting on a rounding boundary; the bound is stated per test.
"""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, synth
from oracle.cpu import Oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _run(path, x, out_ch):
    from neuroflow_b200.runtime import InferenceRuntime
    rt = InferenceRuntime(path)
    y = np.zeros(x.shape[:-1] + (out_ch,), np.float32)
    rt.run(x, y)
    assert not rt.is_int8_gemm_enabled()
    return y


def _model(tmp_path, act, quant, in_ch=5, width=20, mh=5, mw=4, L=3, H=16, W=32, pad=1,
           out_ch=1):
    m = synth.fno2d_model(9, in_ch=in_ch, out_ch=out_ch, width=width, mh=mh, mw=mw, L=L, H=H,
                          W=W, n_calib=2, calib_chunk=2)
    m.activation = act
    m.quant_enabled = quant
    m.config["pad_factor"] = pad
    p = os.path.join(str(tmp_path), f"f2_{act}_{quant}_{pad}.nneuroir")
    ir.write(p, m)
    return m, p


@pytest.mark.gpu
@pytest.mark.parametrize("quant", [True, False])
@pytest.mark.parametrize("geom", [(16, 32, 1), (32, 16, 1), (16, 8, 32), (128, 128, 1), (128, 64, 1)])
def test_fno2d_fp32_relu_bit_exact(tmp_path, quant, geom):
    H, W, pad = geom
    m, p = _model(tmp_path, "relu", quant, H=H, W=W, pad=pad)
    x = synth.fno2d_inputs(np.random.default_rng(5), 2, H, W, in_ch=5)
    want = Oracle().fno2d_forward(m, x, mode=0)
    got = _run(p, x, 1)
    assert np.array_equal(_bits(got), _bits(want)), float(np.abs(got - want).max())


@pytest.mark.gpu
def test_fno2d_fp32_relu_wide_multi_output(tmp_path):
    m, p = _model(tmp_path, "relu", True, in_ch=3, width=64, mh=12, mw=12, L=2, H=64, W=64,
                  out_ch=3)
    x = synth.fno2d_inputs(np.random.default_rng(6), 2, 64, 64)
    want = Oracle().fno2d_forward(m, x, mode=0)
    got = _run(p, x, 3)
    assert np.array_equal(_bits(got), _bits(want)), float(np.abs(got - want).max())


@pytest.mark.gpu
def test_fno2d_fp32_gelu_configs2_geometry(tmp_path):
    """configs[2] geometry (128x128, width 64, 12x12 modes, 4 layers), GELU: outputs are
    fake-quantised with proj_out.output, so agreement is counted in output steps."""
    m, p = _model(tmp_path, "gelu", True, in_ch=3, width=64, mh=12, mw=12, L=4, H=128, W=128)
    x = synth.fno2d_inputs(np.random.default_rng(7), 2, 128, 128)
    want = Oracle().fno2d_forward(m, x, mode=0)
    got = _run(p, x, 1)
    step = m.qparams["proj_out.output"].scale
    d = np.abs(got - want) / step
    print("max steps", float(d.max()), "frac moved", float(np.mean(d > 0)))
    assert np.mean(d > 0) < 0.01 and d.max() <= 4


@pytest.mark.gpu
@pytest.mark.parametrize("name,key", [("fno2d_q", "y_q"), ("fno2d_plain", "y_plain")])
def test_fno2d_fp32_reference_exported_models(name, key):
    """Models exported by the reference's Python package, against the reference C++
    runtime's own outputs (GELU)."""
    d = np.load(os.path.join(GOLD, "fno2d_q.npz"))
    got = _run(os.path.join(GOLD, name + ".nneuroir"), d["x"], 1)
    want = d[key]
    diff = np.abs(got - want)
    if key == "y_q":
        m = ir.read(os.path.join(GOLD, name + ".nneuroir"))
        step = m.qparams["proj_out.output"].scale
        assert np.mean(diff > 0) < 0.01 and diff.max() <= 4 * step
    else:
        assert np.allclose(got, want, rtol=1e-5, atol=1e-6 * np.abs(want).max())
