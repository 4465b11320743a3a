"""FNO3d executor on the GPU vs the CPU restatement (oracle, pinned bit-exact against
the reference runtime's FNO3d::Forward).

FP32 path: the reference's transforms, contraction, Linear rounding; ReLU models are
bit-identical, GELU models differ only through CUDA's tanhf.  FP8 E4M3 variant (no
reference counterpart): the reference's own E4M3 encoder on the GPU, exact products
of E4M3 codes.  At widths 8 and 16 the local layer sums them in k order on CUDA cores
(ReLU models bit-identical); at widths 32 and 64 it runs on tensor cores
(tcgen05.mma.kind::f8f6f4), whose summation order differs from the oracle's k order in
the last bits, so those models are held to the north-star FP8 tolerance of 1e-3
relative L2 (as are all GELU models).
"""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, synth
from oracle.cpu import Oracle


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _rel(a, b):
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


def _model(tmp_path, act="gelu", pad=1, **kw):
    m = synth.fno3d_model(4, n_calib=2, **kw)
    m.activation = act
    m.config["pad_factor"] = pad
    p = os.path.join(str(tmp_path), f"f3_{act}_{pad}.nneuroir")
    ir.write(p, m)
    return m, p


def _run(path, x, out_ch, fp8=False):
    from neuroflow_b200.runtime import InferenceRuntime
    rt = InferenceRuntime(path)
    if fp8:
        rt.enable_fp8()
        assert rt.is_fp8_enabled()
    y = np.zeros(x.shape[:-1] + (out_ch,), np.float32)
    rt.run(x, y)
    return y


GEOMS = [dict(width=8, modes=(3, 3, 2), L=2, S=8),
         dict(width=8, modes=(2, 2, 2), L=1, S=8, in_ch=9),   # lift with > 8 input features
         dict(width=16, modes=(2, 4, 3), L=1, S=16, in_ch=5),
         dict(width=32, modes=(4, 4, 4), L=2, S=16)]


@pytest.mark.gpu
@pytest.mark.parametrize("kw", GEOMS)
@pytest.mark.parametrize("fp8", [False, True])
def test_fno3d_relu_bit_exact(tmp_path, kw, fp8):
    m, p = _model(tmp_path, "relu", **kw)
    x = synth.fno3d_inputs(np.random.default_rng(1), 2, kw["S"], kw.get("in_ch", 4))
    want = Oracle().fno3d_forward(m, x, fp8=fp8)
    got = _run(p, x, 1, fp8)
    if fp8 and kw["width"] >= 32:   # tensor-core local layer
        print("fp8 tc rel", _rel(got, want), "moved", int(np.sum(got != want)), "of", got.size)
        assert _rel(got, want) < 1e-3
    else:
        assert np.array_equal(_bits(got), _bits(want)), float(np.abs(got - want).max())


@pytest.mark.gpu
@pytest.mark.parametrize("width,fp8,shape", [(8, False, (2, 8, 16, 64)), (8, True, (2, 8, 16, 64)),
                                              (32, False, (2, 8, 16, 64)), (8, False, (1, 64, 64, 16)),
                                              (8, False, (1, 16, 64, 64))])
def test_fno3d_relu_bit_exact_d64(tmp_path, width, fp8, shape):
    """64-point lines, which the forward and inverse passes transform in registers (D,
    W and H axes; the W pass only where D >= 64), on non-cubic grids with ReLU:
    bit-identical to the oracle."""
    m, p = _model(tmp_path, "relu", width=width, modes=(3, 4, 6), L=2, S=16)
    x = np.random.default_rng(7).standard_normal(shape + (4,)).astype(np.float32)
    want = Oracle().fno3d_forward(m, x, fp8=fp8)
    got = _run(p, x, 1, fp8)
    assert np.array_equal(_bits(got), _bits(want)), float(np.abs(got - want).max())


@pytest.mark.gpu
def test_fno3d_relu_bit_exact_padded(tmp_path):
    m, p = _model(tmp_path, "relu", pad=16, width=8, modes=(3, 3, 3), L=1, S=8)
    x = synth.fno3d_inputs(np.random.default_rng(2), 1, 8)
    for fp8 in (False, True):
        want = Oracle().fno3d_forward(m, x, fp8=fp8)
        got = _run(p, x, 1, fp8)
        assert np.array_equal(_bits(got), _bits(want)), (fp8, float(np.abs(got - want).max()))


@pytest.mark.gpu
def test_fno3d_configs3_blocks_gelu(tmp_path):
    """configs[3] block geometry (width 32, 8x8x8 modes, 4 layers) on a 32^3 grid."""
    m, p = _model(tmp_path, width=32, modes=(8, 8, 8), L=4, S=32)
    x = synth.fno3d_inputs(np.random.default_rng(3), 2, 32)
    o = Oracle()
    want = o.fno3d_forward(m, x)
    got = _run(p, x, 1)
    assert _rel(got, want) < 1e-5, _rel(got, want)
    want8 = o.fno3d_forward(m, x, fp8=True)
    got8 = _run(p, x, 1, fp8=True)
    print("fp8 rel", _rel(got8, want8), "fp8 vs fp32", _rel(want8, want))
    assert _rel(got8, want8) < 1e-3


@pytest.mark.gpu
def test_fno3d_fp8_configs3_grid():
    """configs[3] itself: the benchmarked FP8 model (64^3 grid, width 32, 8x8x8 modes, 4
    layers, scales from a 4-sample calibration batch), one of the benchmark's samples,
    within 1e-3 relative L2 of the oracle."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    path = bench.aux_model("fno3d_fp8")
    m = ir.read(path)
    x = synth.fno3d_inputs(np.random.default_rng(100), 1, 64)
    want = Oracle().fno3d_forward(m, x, fp8=True)
    got = _run(path, x, 1, fp8=True)
    print("configs[3] fp8 rel", _rel(got, want), "moved", int(np.sum(got != want)), "of", got.size)
    assert np.all(np.isfinite(got))
    assert _rel(got, want) < 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("shape,modes,width", [
    ((2, 8, 16, 16), (3, 5, 9), 32),     # kept D Nyquist mode
    ((1, 8, 16, 32), (4, 3, 6), 32),
    ((1, 8, 16, 64), (4, 3, 6), 32),     # D pass on tensor cores, fused inverse + local
    ((1, 8, 8, 64), (3, 4, 16), 32),     # ... N = 32 forward; inverse not fused (16 kd modes)
    ((1, 4, 128, 128), (2, 3, 5), 32),   # ... Wp = Dp = 128 (one row per tile)
    ((1, 4, 16, 64), (3, 8, 8), 64),     # width 64, fused
    ((3, 16, 8, 16), (5, 8, 2), 32)])
def test_fno3d_fp8_direct_dft_geometries(tmp_path, shape, modes, width):
    """FP8 at widths 32 and 64 runs the D and W passes as direct truncated DFTs (the
    forward D pass as an f16 MMA and the inverse fused into the tensor-core local layer
    when Dp is 64 or 128): non-cubic grids, odd mode counts (padded table columns), the
    D-axis Nyquist mode kept (Dp / 2 + 1 modes), and plane counts that leave the last
    CTA pass partly empty."""
    S = 16 if max(modes) <= 9 else 32     # the calibration grid holds the modes
    m, p = _model(tmp_path, "gelu", width=width, modes=modes, L=2, S=S)
    x = np.random.default_rng(5).standard_normal(shape + (4,)).astype(np.float32)
    want = Oracle().fno3d_forward(m, x, fp8=True)
    got = _run(p, x, 1, fp8=True)
    print("direct dft rel", _rel(got, want))
    assert _rel(got, want) < 1e-3


@pytest.mark.gpu
def test_fno3d_errors(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    _, p = _model(tmp_path, width=8, modes=(2, 2, 2), L=1, S=8)
    rt = InferenceRuntime(p)
    assert rt.op() == "FNO3d" and not rt.is_fp8_enabled()
    with pytest.raises(RuntimeError, match="expected 5D input"):
        rt.run(np.zeros((1, 8, 8, 4), np.float32), np.zeros((1, 8, 8, 1), np.float32))
    with pytest.raises(RuntimeError, match="input channels mismatch"):
        rt.run(np.zeros((1, 8, 8, 8, 3), np.float32), np.zeros((1, 8, 8, 8, 1), np.float32))
    with pytest.raises(RuntimeError, match="output buffer shape mismatch"):
        rt.run(np.zeros((1, 8, 8, 8, 4), np.float32), np.zeros((1, 8, 8, 4, 1), np.float32))
    with pytest.raises(RuntimeError, match="power of two"):
        rt.run(np.zeros((1, 8, 6, 8, 4), np.float32), np.zeros((1, 8, 6, 8, 1), np.float32))


@pytest.mark.gpu
@pytest.mark.parametrize("S,modes", [(64, (8, 8, 8)), (32, (8, 8, 8))])
def test_fno3d_fp8_layer_codes_match_oracle(tmp_path, S, modes):
    """The FP8 variant layer by layer: the E4M3 codes of every layer input (taps) against
    the oracle's.  The network output is fake-quantised to E4M3 and barely moves under
    small perturbations (a 0.1 % change of a layer's spectral weights moves none of
    65,536 outputs), so the layer codes are the sensitive check of the direct DFTs, the
    f16 forward D pass, the fused tf32 inverse and the tensor-core local layer.  A moved
    code is one E4M3 step from the oracle's, and few codes move."""
    import torch
    from neuroflow_b200.runtime import InferenceRuntime
    m, p = _model(tmp_path, "gelu", width=32, modes=modes, L=4, S=min(S, 32))
    x = synth.fno3d_inputs(np.random.default_rng(11), 1, S)
    o = Oracle()
    _, taps = o.fno3d_forward(m, x, fp8=True, taps=True)
    rt = InferenceRuntime(p)
    rt.enable_fp8()
    buf = torch.zeros(taps.size, dtype=torch.uint8, device="cuda")
    rt.set_code_taps(buf)
    dy = torch.empty(x.shape[:-1] + (1,), dtype=torch.float32, device="cuda")
    rt.run_device(torch.from_numpy(x).cuda(), dy)
    torch.cuda.synchronize()
    rt.set_code_taps(None)
    got = buf.cpu().numpy().reshape(taps.shape)
    dec = np.array([o.lib.nfo_e4m3_to_fp32(i) for i in range(256)], np.float32)
    vals = dec[got]
    for i in range(taps.shape[0]):
        moved = vals[i] != taps[i]
        frac = float(moved.mean())
        print(f"S={S} layer input {i}: moved {int(moved.sum())} of {moved.size} ({frac:.2e})")
        assert frac < 1e-5, (i, frac)
        if moved.any():
            # one E4M3 step: adjacent codes of one sign, or the two codes next to zero
            gc = got[i][moved].astype(np.int32)
            wc = o.fp32_to_e4m3(np.ascontiguousarray(taps[i][moved])).astype(np.int32)
            ok = (np.abs(gc - wc) <= 1) | (((gc & 0x7F) <= 1) & ((wc & 0x7F) <= 1))
            assert np.all(ok), (i, gc[~ok][:8], wc[~ok][:8])
