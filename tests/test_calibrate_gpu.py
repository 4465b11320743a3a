"""Activation calibration on the GPU (nfx_calibrate_*).

Two checks:
* against the CPU restatement of the runtime (oracle taps of every Linear output, with
  the reference's qparam rules restated in neuroflow_b200.quant and numpy's percentile):
  a ReLU model, where the GPU FP32 executor is bit-identical to the restatement, gives
  identical results; a GELU model agrees to rtol 1e-6 (CUDA's tanhf);
* against the reference's own calibration of the same model (tests/golden: the FNO2d
  built by the reference's PyTorch model and calibrated by its quantise_model on the
  batch saved in calib.npz).  The reference observes its PyTorch model, whose GELU is
  the erf form (neuroflow/nn/fno2d.py:137-138) while its C++ runtime -- and so the GPU
  executor -- uses the tanh form (cpp/src/fno.cpp:36-48): tensors computed before the
  first activation (lift, locs.0) agree to rtol 1e-5 with equal zero points, the later
  ones to the GELU forms' difference (rtol 2e-3, zero points within one).
"""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _check(got, keys, scales, zps, what):
    for k, s_ref, z_ref in zip(keys, scales, zps):
        s, z = got[str(k)][0], got[str(k)][1]
        before_act = str(k) in ("lift.output", "locs.0.output")
        assert np.isclose(s, s_ref, rtol=1e-5 if before_act else 2e-3, atol=0), (what, k, s, s_ref)
        assert abs(z - z_ref) <= (0 if before_act else 1), (what, k, z, z_ref)


def _oracle_stats(m, batches, pct):
    """The reference's rules over the restatement's Linear outputs of all batches."""
    from neuroflow_b200 import quant
    from oracle.cpu import Oracle
    L = m.config["n_layers"]
    obs = {}
    for x in batches:
        y, taps = Oracle().fno2d_forward(m, x, mode=0, taps=True)
        cur = {"lift.output": taps["lift_out"], "proj_q.output": taps["q_out"],
               "proj_out.output": y}
        for i in range(L):
            cur[f"locs.{i}.output"] = taps[f"x2.{i}"]
        for k, v in cur.items():
            obs.setdefault(k, []).append(v.ravel())
    out = {}
    for k, vs in obs.items():
        a = np.concatenate(vs)
        f8 = float(np.float32(quant.fp8_qparams(a).scale))   # NIRQ stores float32
        if pct >= 100:
            q = quant.tensor_qparams(a)
            out[k] = (q.scale, q.zero_point, f8)
        else:
            lo_p = (100.0 - pct) / 2.0
            mins, maxs = (float(v) for v in np.percentile(a, [lo_p, 100.0 - lo_p]))
            spans = maxs - mins
            scale = spans / 255 if spans > 0 else 1.0
            zp = int(np.clip(np.round(-128 - mins / scale), -128, 127))
            if zp == -128 and maxs > 0:
                scale = maxs / 255
            elif zp == 127 and mins < 0:
                scale = -mins / 255
            out[k] = (float(np.float32(scale)), zp, f8)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("act", ["relu", "gelu"])
def test_calibration_matches_the_restatement(tmp_path, act):
    from neuroflow_b200 import synth
    from neuroflow_b200.calibrate import calibrate_fno2d
    m = synth.fno2d_model(12, width=32, mh=6, mw=5, L=3, H=32, W=32, n_calib=2, calib_chunk=2)
    m.activation = act
    m.quant_enabled = False
    p = str(tmp_path / "m.nneuroir")
    ir.write(p, m)
    rng = np.random.default_rng(3)
    batches = [synth.fno2d_inputs(rng, 3, 32, 32), synth.fno2d_inputs(rng, 2, 32, 32)]
    for pct in (100.0, 99.0, 99.9):
        got = calibrate_fno2d(p, batches, percentile=pct)
        want = _oracle_stats(m, batches, pct)
        assert sorted(got) == sorted(want)
        for k in want:
            g, w = got[k][:3], want[k]
            if act == "relu":
                assert g == w, (pct, k, g, w)
            else:
                assert np.allclose(g[0], w[0], rtol=1e-6) and g[1] == w[1], (pct, k, g, w)
                assert np.isclose(g[2], w[2], rtol=1e-6), (pct, k, g, w)


@pytest.mark.gpu
def test_minmax_percentile_and_fp8_calibration_match_the_reference():
    from neuroflow_b200.calibrate import calibrate_fno2d
    d = np.load(os.path.join(GOLD, "calib.npz"))
    g = np.load(os.path.join(GOLD, "fno2d_q.npz"))
    path = os.path.join(GOLD, "fno2d_plain.nneuroir")
    got = calibrate_fno2d(path, [d["calib"]])
    assert sorted(got) == sorted(str(k) for k in g["act_keys"])
    _check(got, g["act_keys"], g["act_scale"], g["act_zp"], "min/max")
    for k, f8 in zip(d["keys"], d["fp8_scale"]):
        tol = 1e-5 if str(k) in ("lift.output", "locs.0.output") else 2e-3
        assert np.isclose(got[str(k)][2], f8, rtol=tol), (k, got[str(k)][2], f8)
    got99 = calibrate_fno2d(path, [d["calib"]], percentile=99.0)
    _check(got99, d["keys"], d["p99_scale"], d["p99_zp"], "p99")
    # two batches observe the union: the same as one batch holding both halves
    half = d["calib"].shape[0] // 2
    got_split = calibrate_fno2d(path, [d["calib"][:half], d["calib"][half:]], percentile=99.0)
    for k in got99:
        assert got_split[k][:3] == got99[k][:3], k


@pytest.mark.gpu
def test_quantise_fno2d_writes_a_runnable_int8_model(tmp_path):
    """The calibrated IR loads, enables the FNO2d INT8 path of the reference's layout and
    keeps the reference's activation qparams."""
    from neuroflow_b200.calibrate import quantise_fno2d
    from neuroflow_b200.runtime import InferenceRuntime
    d = np.load(os.path.join(GOLD, "calib.npz"))
    out = str(tmp_path / "q.nneuroir")
    m = quantise_fno2d(os.path.join(GOLD, "fno2d_plain.nneuroir"), [d["calib"]], out)
    m2 = ir.read(out)
    assert m2.quant_enabled and sorted(m2.qparams) == sorted(m.qparams)
    ref = ir.read(os.path.join(GOLD, "fno2d_q.nneuroir"))
    for k in ("lift.output", "locs.0.output"):     # computed before the first GELU
        assert np.isclose(m2.qparams[k].scale, ref.qparams[k].scale, rtol=1e-5)
        assert m2.qparams[k].zero_point == ref.qparams[k].zero_point
    rt = InferenceRuntime(out)
    x = np.load(os.path.join(GOLD, "fno2d_q.npz"))["x"]
    y = np.zeros(x.shape[:-1] + (1,), np.float32)
    rt.run(x, y)   # the FP32 fake-quant network of the calibrated IR
    assert np.all(np.isfinite(y))


@pytest.mark.gpu
def test_calibration_errors(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    path = os.path.join(GOLD, "fno2d_plain.nneuroir")
    rt = InferenceRuntime(path)
    with pytest.raises(RuntimeError, match="nfx_calibrate_begin first"):
        rt.calibrate_observe(np.zeros((1, 16, 16, 3), np.float32))
    rt.calibrate_begin(keep_values=False)
    with pytest.raises(RuntimeError, match="no calibration batch"):
        rt.calibrate_results()
    rt.calibrate_observe(np.zeros((1, 16, 16, 3), np.float32) + 0.5)
    with pytest.raises(RuntimeError, match="percentiles need the values"):
        rt.calibrate_results(99.0)
    res = rt.calibrate_results()
    assert len(res) == 5
    rt.calibrate_end()
    rt1 = InferenceRuntime(os.path.join(GOLD, "fno1d_pc.nneuroir"))
    with pytest.raises(RuntimeError, match="supports FNO2d"):
        rt1.calibrate_begin()
