"""FNO2d INT8 composition (EnableInt8Gemm) on geometries outside the width-64 12x12
executor: other widths and mode counts, grids wider than 128, channel counts, and IRs
where only some layers qualify for the INT8 GEMM.  These run on the FP32 executor's
transform kernels with the int8 Linear and the input snaps of the composition; every
output must equal the CPU restatement's (oracle mode 1, which follows the reference
FNO1d INT8 convention of cpp/src/fno.cpp:475-549 on FNO2d::Forward, fno.cpp:777-995)."""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, quant, synth
from oracle.cpu import Oracle


def _run(tmp_path, m, x, name="m.nneuroir"):
    from neuroflow_b200.runtime import InferenceRuntime
    path = os.path.join(str(tmp_path), name)
    ir.write(path, m)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    assert rt.is_int8_gemm_enabled()
    got = np.zeros(x.shape[:3] + (m.config["out_channels"],), np.float32)
    rt.run(x, got)
    return got


def _check(got, want, m):
    assert len(np.unique(want)) > 8   # not a saturated network
    step = m.qparams["proj_out.output"].scale if "proj_out.output" in m.qparams else 1.0
    d = np.abs(got - want)
    assert np.all(np.isfinite(got))
    assert np.array_equal(got, want), dict(frac=float(np.mean(d > 0)), max_steps=float(d.max() / step))


@pytest.mark.gpu
@pytest.mark.parametrize("act", ["relu", "gelu"])
@pytest.mark.parametrize("seed,width,mh,mw,H,W,L,B", [
    (8, 32, 8, 8, 64, 64, 3, 3),
    (8, 48, 6, 10, 32, 128, 2, 2),
    (6, 64, 12, 12, 32, 256, 2, 1),     # the width-64 model on a grid wider than 128
    (8, 128, 5, 7, 16, 32, 2, 2),
])
def test_fno2d_int8_other_geometries_match_oracle(tmp_path, act, seed, width, mh, mw, H, W, L, B):
    m = synth.fno2d_model(seed, width=width, mh=mh, mw=mw, L=L, H=H, W=W, n_calib=2, calib_chunk=2)
    m.activation = act
    x = synth.fno2d_inputs(np.random.default_rng(17), B, H, W)
    want = Oracle().fno2d_forward(m, x, mode=1)
    _check(_run(tmp_path, m, x), want, m)


@pytest.mark.gpu
def test_fno2d_int8_mixed_layers_and_channel_counts(tmp_path):
    """in_ch 5 and out_ch 7; locs.1 with per-tensor weight qparams (FP32 Linear on its
    snapped input), locs.0.output FP8 (so layer 1's input is not snapped and layer 1's
    Linear stays FP32 as well), the rest INT8."""
    m = synth.fno2d_model(9, in_ch=5, out_ch=7, width=16, mh=4, mw=3, L=3, H=16, W=32,
                          n_calib=2, calib_chunk=2)
    w = m.weights["locs.1.weight"]
    m.qparams["locs.1.weight"] = quant.tensor_qparams(np.array([w.min(), w.max()], np.float32))
    m.qparams["locs.0.output"] = ir.FP8(float(np.float32(0.02)))
    x = synth.fno2d_inputs(np.random.default_rng(3), 3, 16, 32, 5)
    want = Oracle().fno2d_forward(m, x, mode=1)
    got = _run(tmp_path, m, x)
    _check(got, want, m)
    # the composition differs from the FP32 network on this model
    assert not np.array_equal(want, Oracle().fno2d_forward(m, x, mode=0))


@pytest.mark.gpu
def test_fno2d_int8_width64_grid_outside_the_executor_range_reuses_handle(tmp_path):
    """One handle: a 32x64 grid on the width-64 executor, then 16x256 and 16x512 (beyond
    its W range) on the composition kernels, then back; all equal the oracle."""
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.fno2d_model(6, L=2, H=32, W=64, n_calib=2, calib_chunk=2)
    path = os.path.join(str(tmp_path), "w64.nneuroir")
    ir.write(path, m)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    o = Oracle()
    for (H, W, B) in ((32, 64, 2), (16, 256, 2), (16, 512, 1), (32, 64, 3)):
        x = synth.fno2d_inputs(np.random.default_rng(H + W + B), B, H, W)
        got = np.zeros((B, H, W, 1), np.float32)
        rt.run(x, got)
        _check(got, o.fno2d_forward(m, x, mode=1), m)
