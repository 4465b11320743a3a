"""FNO2d INT8 executor on the GPU vs the CPU restatement (oracle mode 1), end to end.

The GPU evaluates the truncated transforms exactly (forward: integer DFT digits on
tensor cores; inverse: 3xTF32) while the restatement follows the reference's radix-2
FFT rounding, so an int8 code can in principle flip where z lies within rounding
distance of a table breakpoint (tests/test_fno2d_parity_gpu.py checks the codes layer
by layer).  On every model and input here no network output moves, and the tests
require exactly that: every output equal to the oracle's."""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, synth
from oracle.cpu import Oracle


def _model(tmp_path, seed=3, L=4, H=32, W=32, in_ch=3, out_ch=1):
    m = synth.fno2d_model(seed, in_ch=in_ch, out_ch=out_ch, width=64, mh=12, mw=12, L=L, H=H,
                          W=W, n_calib=4, calib_chunk=4)
    p = os.path.join(str(tmp_path), "fno2d.nneuroir")
    ir.write(p, m)
    return m, p


def _stats(got, want, step):
    d = np.abs(got - want)
    return dict(max_abs=float(d.max()), frac_diff=float(np.mean(d > 0)),
                max_steps=float(d.max() / step), rel_l2=float(np.linalg.norm(got - want) /
                                                             (np.linalg.norm(want) + 1e-30)))


@pytest.mark.gpu
@pytest.mark.parametrize("H,W", [(32, 32), (64, 128)])
def test_fno2d_int8_end_to_end(tmp_path, H, W):
    from neuroflow_b200.runtime import InferenceRuntime
    m, path = _model(tmp_path, H=H, W=W)
    x = synth.fno2d_inputs(np.random.default_rng(11), 3, H, W)
    want = Oracle().fno2d_forward(m, x, mode=1)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    assert rt.is_int8_gemm_enabled()
    got = np.zeros_like(want)
    rt.run(x, got)
    step = m.qparams["proj_out.output"].scale
    st = _stats(got, want, step)
    print(H, W, st)
    assert np.all(np.isfinite(got))
    assert st["frac_diff"] == 0, st


@pytest.mark.gpu
def test_fno2d_shape_errors(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    m, path = _model(tmp_path, L=1)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    x = np.zeros((1, 32, 32, 3), np.float32)
    with pytest.raises(RuntimeError, match="input channels mismatch"):
        rt.run(np.zeros((1, 32, 32, 2), np.float32), np.zeros((1, 32, 32, 1), np.float32))
    with pytest.raises(RuntimeError, match="output buffer shape mismatch"):
        rt.run(x, np.zeros((1, 32, 16, 1), np.float32))
    with pytest.raises(RuntimeError, match="power of two"):
        rt.run(np.zeros((1, 24, 32, 3), np.float32), np.zeros((1, 24, 32, 1), np.float32))
    with pytest.raises(RuntimeError, match="expected 4D"):
        rt.run(np.zeros((32, 32, 3), np.float32), np.zeros((32, 32, 1), np.float32))


@pytest.mark.gpu
def test_fno2d_without_nirq_is_not_int8(tmp_path):
    """Without NIRQ, EnableInt8Gemm leaves the flag off (the reference's flag is
    FNO1d-only) and Run executes the FP32 network."""
    from neuroflow_b200.runtime import InferenceRuntime
    m, _ = _model(tmp_path, L=1)
    m.quant_enabled = False
    p = os.path.join(str(tmp_path), "plain.nneuroir")
    ir.write(p, m)
    rt = InferenceRuntime(p)
    rt.enable_int8_gemm()
    assert not rt.is_int8_gemm_enabled()
    x = synth.fno2d_inputs(np.random.default_rng(1), 1, 32, 32)
    y = np.zeros((1, 32, 32, 1), np.float32)
    rt.run(x, y)
    want = Oracle().fno2d_forward(m, x, mode=0)
    assert np.allclose(y, want, rtol=1e-4, atol=1e-5 * np.abs(want).max())


@pytest.mark.gpu
def test_fno2d_growing_batch_reuses_handle(tmp_path):
    """Host-buffer Run with a growing batch re-allocates only the staging buffers; the
    transform tables built for the grid stay valid."""
    from neuroflow_b200.runtime import InferenceRuntime
    m, path = _model(tmp_path, L=2, H=32, W=128)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    o = Oracle()
    step = m.qparams["proj_out.output"].scale
    for B in (1, 3, 2, 4):
        x = synth.fno2d_inputs(np.random.default_rng(20 + B), B, 32, 128)
        got = np.zeros((B, 32, 128, 1), np.float32)
        rt.run(x, got)
        st = _stats(got, o.fno2d_forward(m, x, mode=1), step)
        assert st["frac_diff"] == 0, (B, st)


@pytest.mark.gpu
@pytest.mark.parametrize("W", [32, 128])
@pytest.mark.parametrize("scale,zp", [(0.0014373305020853877, 1), (0.0005, 0)])
def test_fno2d_int8_two_segment_code_table(tmp_path, scale, zp, W):
    """A layer output scale this small needs more uniform table cells than fit in
    shared memory; the executor then splits the z -> code table at a gap between
    breakpoints into a coarse (GELU's negative branch) and a fine segment.  The W = 128
    kernel has room for more cells: at the first scale it takes a one-segment table of
    about 5.2k cells, at the second the split table."""
    from neuroflow_b200.ir import PerTensor
    from neuroflow_b200.runtime import InferenceRuntime
    m, _ = _model(tmp_path, L=3, W=W)
    m.qparams["locs.1.output"] = PerTensor(scale, zp)
    path = os.path.join(str(tmp_path), "small_scale.nneuroir")
    ir.write(path, m)
    x = synth.fno2d_inputs(np.random.default_rng(5), 2, 32, W)
    want = Oracle().fno2d_forward(m, x, mode=1)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    got = np.zeros_like(want)
    rt.run(x, got)
    st = _stats(got, want, m.qparams["proj_out.output"].scale)
    print(scale, zp, st)
    assert st["frac_diff"] == 0, st


@pytest.mark.gpu
@pytest.mark.parametrize("pinned", [False, True])
@pytest.mark.parametrize("B", [5, 40, 130, 160, 300])
def test_fno2d_host_run_chunked_matches_device_run(tmp_path, B, pinned):
    """The host-buffer Run of a large batch overlaps copies and compute over batch
    chunks (2 halves below 4 q samples, q = SMs / gcd(SMs, 4); above, q / 2, 2q, ..., q:
    4 chunks at 160 and 5 at 300 on 148 SMs), reading pinned caller buffers directly and
    staging pageable ones through the runtime's pinned buffers; the result is
    bit-identical to one device-buffer run of the whole batch."""
    import torch
    from neuroflow_b200.runtime import InferenceRuntime
    m, path = _model(tmp_path, L=2)
    x = synth.fno2d_inputs(np.random.default_rng(31), B, 32, 32)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    if pinned:
        x = torch.from_numpy(x).pin_memory().numpy()
        got = torch.zeros((B, 32, 32, 1), dtype=torch.float32).pin_memory().numpy()
    else:
        got = np.zeros((B, 32, 32, 1), np.float32)
    rt.run(x, got)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((B, 32, 32, 1), dtype=torch.float32, device="cuda")
    rt.run_device(dx, dy, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert np.array_equal(got, dy.cpu().numpy())


@pytest.mark.gpu
@pytest.mark.parametrize("in_ch,out_ch", [(2, 2), (4, 4)])
def test_fno2d_int8_channel_counts(tmp_path, in_ch, out_ch):
    """Other lift widths and proj_out widths (out_ch up to 4) through the same kernels."""
    from neuroflow_b200.runtime import InferenceRuntime
    m, path = _model(tmp_path, L=2, H=32, W=128, in_ch=in_ch, out_ch=out_ch)
    x = synth.fno2d_inputs(np.random.default_rng(13), 2, 32, 128, in_ch)
    want = Oracle().fno2d_forward(m, x, mode=1)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    assert rt.is_int8_gemm_enabled()
    got = np.zeros_like(want)
    rt.run(x, got)
    st = _stats(got, want, m.qparams["proj_out.output"].scale)
    assert st["frac_diff"] == 0, st


@pytest.mark.gpu
def test_fno2d_int8_integers_beyond_two_pow_22(tmp_path):
    """Weight codes far from their zero points (all 127 against zp_w = -128) and an
    input zero point of -50: the projection's integers sum_k (a_k - zp_in)(w_k - 2 zp_w)
    reach the millions (up to 64 * 177 * 383), against a few thousand in the calibrated
    models, where an error in the zero-point terms the MMA folds in would show.  Every
    output equals the oracle's."""
    from neuroflow_b200.ir import PerTensor
    from neuroflow_b200.runtime import InferenceRuntime
    m, _ = _model(tmp_path, L=2, W=128)
    m.weights["proj_q.weight"] = np.abs(m.weights["proj_q.weight"])
    qp = m.qparams["proj_q.weight"]
    qp.scales = np.full_like(qp.scales, 1e-7)
    qp.zero_points = np.full_like(qp.zero_points, -128)
    m.qparams["locs.1.output"] = PerTensor(m.qparams["locs.1.output"].scale, -50)
    path = os.path.join(str(tmp_path), "wide_integers.nneuroir")
    ir.write(path, m)
    x = synth.fno2d_inputs(np.random.default_rng(21), 2, 32, 128)
    want = Oracle().fno2d_forward(m, x, mode=1)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    got = np.zeros_like(want)
    rt.run(x, got)
    st = _stats(got, want, m.qparams["proj_out.output"].scale)
    print(st)
    assert st["frac_diff"] == 0, st
