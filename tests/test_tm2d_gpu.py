"""TokenMixer2D executor on the GPU vs the CPU restatement (oracle, pinned bit-exact
against the reference runtime's RunTokenMixer2D).

The FP32 path reproduces the reference's loop order and rounding except CUDA's expf
(softmax) and tanhf (GELU), a few ulps each; the bound below is on the relative L2
error and on the largest element error.  The INT8 variant (no reference counterpart)
quantises each Linear input row on the fly, so an upstream ulp can move a code by one
step, and the network output (not quantised) then moves continuously: nearly every
output differs from the oracle's by a few ulps, the moved codes add up to about 1e-3
of the largest output, 1e-4 to 8e-4 relative L2 on the models below.  Its bound is
2e-3 relative L2.
"""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, synth
from oracle.cpu import Oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _model(tmp_path, act="gelu", **kw):
    m = synth.tm2d_model(3, activation=act, **kw)
    p = os.path.join(str(tmp_path), "tm2d.nneuroir")
    ir.write(p, m)
    return m, p


def _run(path, x, out_d, int8=False):
    from neuroflow_b200.runtime import InferenceRuntime
    rt = InferenceRuntime(path)
    if int8:
        rt.enable_int8_gemm()
        assert rt.is_int8_gemm_enabled()
    y = np.zeros(x.shape[:-1] + (out_d,), np.float32)
    rt.run_tokenmixer2d(x, y)
    return y


def _rel(a, b):
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


SMALL = [dict(latent=16, n_heads=2, h=6, w=8, n_patches=12, n_layers=2),
         dict(latent=24, n_heads=3, h=5, w=4, n_patches=20, n_layers=1, in_dim=5, out_dim=2),
         dict(latent=32, n_heads=4, h=8, w=16, n_patches=128, n_layers=2),
         dict(latent=128, n_heads=2, h=16, w=16, n_patches=64, n_layers=1)]


@pytest.mark.gpu
@pytest.mark.parametrize("kw", SMALL)
@pytest.mark.parametrize("act", ["gelu", "relu"])
def test_tm2d_fp32_matches_reference_arithmetic(tmp_path, kw, act):
    m, p = _model(tmp_path, act, **kw)
    x = np.random.default_rng(1).standard_normal(
        (3, kw["h"], kw["w"], kw.get("in_dim", 3))).astype(np.float32)
    want = Oracle().tm2d_forward(m, x)
    got = _run(p, x, kw.get("out_dim", 1))
    assert _rel(got, want) < 1e-5, _rel(got, want)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max() + 1e-6


@pytest.mark.gpu
def test_tm2d_reference_exported_model():
    d = np.load(os.path.join(GOLD, "tm2d.npz"))
    got = _run(os.path.join(GOLD, "tm2d.nneuroir"), d["x"], 1)
    assert _rel(got, d["y"]) < 1e-5


@pytest.mark.gpu
def test_tm2d_configs4_blocks_fp32_and_int8(tmp_path):
    """configs[4] block geometry (latent 128, 4 heads, head_dim 32) on a 32x32 grid of
    1024 tokens, 2 blocks; FP32 and the INT8 per-token variant."""
    m, p = _model(tmp_path, latent=128, n_heads=4, h=32, w=32, n_patches=1024, n_layers=2)
    x = synth.tm2d_inputs(np.random.default_rng(2), 2, 32, 32)
    o = Oracle()
    want = o.tm2d_forward(m, x)
    got = _run(p, x, 1)
    assert _rel(got, want) < 1e-5, _rel(got, want)
    want8 = o.tm2d_forward(m, x, int8=True)
    got8 = _run(p, x, 1, int8=True)
    r8 = _rel(got8, want8)
    print("int8 rel", r8, "int8 vs fp32", _rel(want8, want))
    assert r8 < 2e-3, r8
    # the INT8 variant stays close to the FP32 network
    assert _rel(want8, want) < 0.1


@pytest.mark.gpu
def test_tm2d_errors(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    _, p = _model(tmp_path, latent=16, n_heads=2, h=8, w=8, n_patches=16, n_layers=1)
    rt = InferenceRuntime(p)
    assert rt.op() == "TokenMixer2D"
    x = np.zeros((1, 8, 8, 3), np.float32)
    with pytest.raises(RuntimeError, match="runtime does not support op: TokenMixer2D"):
        rt.run(x, np.zeros((1, 8, 8, 1), np.float32))
    with pytest.raises(RuntimeError, match="expected 4D"):
        rt.run_tokenmixer2d(np.zeros((8, 8, 3), np.float32), np.zeros((8, 8, 1), np.float32))
    with pytest.raises(RuntimeError, match="input feature dim mismatch"):
        rt.run_tokenmixer2d(np.zeros((1, 8, 8, 2), np.float32), np.zeros((1, 8, 8, 1), np.float32))
    with pytest.raises(RuntimeError, match="h / w mismatch"):
        rt.run_tokenmixer2d(np.zeros((1, 8, 4, 3), np.float32), np.zeros((1, 8, 4, 1), np.float32))
    with pytest.raises(RuntimeError, match="output buffer shape mismatch"):
        rt.run_tokenmixer2d(x, np.zeros((1, 8, 8, 2), np.float32))
    y = np.ones((0, 8, 8, 1), np.float32)
    rt.run_tokenmixer2d(np.zeros((0, 8, 8, 3), np.float32), y)


@pytest.mark.gpu
def test_run_tokenmixer2d_on_an_fno_runtime(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.fno1d_model(1, width=16, modes=4, L=1, n=32, quantised=False)
    p = os.path.join(str(tmp_path), "f.nneuroir")
    ir.write(p, m)
    rt = InferenceRuntime(p)
    with pytest.raises(RuntimeError, match="TokenMixer2D not initialized"):
        rt.run_tokenmixer2d(np.zeros((1, 8, 8, 3), np.float32), np.zeros((1, 8, 8, 1), np.float32))
