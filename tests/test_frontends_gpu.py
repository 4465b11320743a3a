"""The reference's front-ends on the GPU runtime: the `neuroflow_cpp` module functions
(`infer`, `infer_arrays`) and the `nflow_infer` command line (same flags)."""
import os
import subprocess

import numpy as np
import pytest

from neuroflow_b200 import ir, synth

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "neuroflow_b200")


@pytest.mark.gpu
def test_infer_arrays_and_cli_agree_with_the_runtime(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime, infer, infer_arrays
    m = synth.fno2d_model(2, width=16, mh=4, mw=4, L=2, H=16, W=16, n_calib=2, calib_chunk=2)
    p = str(tmp_path / "m.nneuroir")
    ir.write(p, m)
    x = synth.fno2d_inputs(np.random.default_rng(0), 2, 16, 16)
    rt = InferenceRuntime(p)
    want = np.zeros((2, 16, 16, 1), np.float32)
    rt.run(x, want)
    assert np.array_equal(infer_arrays(p, x), want)
    xin, yout = str(tmp_path / "x.npy"), str(tmp_path / "y.npy")
    np.save(xin, x)
    assert infer(p, xin, yout) == "ok"
    assert np.array_equal(np.load(yout), want)
    cli = os.path.join(PKG, "nflow_infer")
    r = subprocess.run([cli, "--model", p, "--input", xin, "--output", yout], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    assert "op=FNO2d shape=(2,16,16,1)" in r.stdout
    assert np.array_equal(np.load(yout), want)
    # rank errors as the reference reports them
    np.save(xin, x[0])
    r = subprocess.run([cli, "--model", p, "--input", xin, "--output", yout], capture_output=True,
                       text=True)
    assert r.returncode == 1 and "expected 4D input for FNO2d" in r.stderr
    with pytest.raises(RuntimeError, match="input rank mismatch"):
        infer_arrays(p, x[0])


@pytest.mark.gpu
def test_cli_runs_tokenmixer2d(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.tm2d_model(1, latent=16, n_heads=2, h=8, w=8, n_patches=16, n_layers=1)
    p = str(tmp_path / "t.nneuroir")
    ir.write(p, m)
    x = np.random.default_rng(1).standard_normal((1, 8, 8, 3)).astype(np.float32)
    want = np.zeros((1, 8, 8, 1), np.float32)
    InferenceRuntime(p).run_tokenmixer2d(x, want)
    xin, yout = str(tmp_path / "x.npy"), str(tmp_path / "y.npy")
    np.save(xin, x)
    r = subprocess.run([os.path.join(PKG, "nflow_infer"), "--model", p, "--input", xin, "--output", yout],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert np.array_equal(np.load(yout), want)
