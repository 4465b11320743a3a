"""FNO2d INT8 executor against the CPU restatement (oracle mode 1) layer by layer, at
the benchmarked geometry and at batch sizes that fill and split the 128-sample tiles.

The executor's code taps (nfx_runtime_set_code_taps) give the int8 codes of every
layer input; the oracle's taps give the same codes and the fp32 values they were
snapped from.  The lift's codes must match bit for bit (the lift reproduces the
reference's Linear rounding exactly).  A Fourier layer's output codes come from
x1 + x2, where x1 is the spectral branch: the reference evaluates it with its radix-2
FFT in fp32, the GPU with an exact integer forward DFT and 3xTF32 inverse transforms,
so the two x1 differ by fp32 rounding (about 1e-6 relative).  A code can therefore
differ only where the oracle's pre-snap value lies within that rounding of a code
boundary (or where an earlier layer's code at the same point already differed); such a
code differs by exactly one.  The tests assert exactly that, count the differing codes
(printed), and require every network output to be identical to the oracle's.
"""
import os
import sys

import numpy as np
import pytest

from neuroflow_b200 import ir, synth
from oracle.cpu import Oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# A code may differ only where the oracle's h / scale lies within this many code steps
# of a rounding boundary (half-integer).  The spectral branch's fp32 differences are
# about 1e-6 of |x1| (|x1| is a few units, a code step about 1e-2), i.e. a few 1e-4
# code steps; the bound leaves an order of magnitude on top.
BOUNDARY_MARGIN = 5e-3


def _device_run_with_taps(rt, x, L, width):
    import torch
    B, H, W, _ = x.shape
    dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    dy = torch.full((B, H, W, 1), float("nan"), dtype=torch.float32, device="cuda")
    taps = torch.zeros((L + 1, B, H, W, width), dtype=torch.int8, device="cuda")
    rt.set_code_taps(taps)
    try:
        rt.run_device(dx, dy)
        torch.cuda.synchronize()
        rt.check()
    finally:
        rt.set_code_taps(None)
    return dy.cpu().numpy(), taps.cpu().numpy()


def _check_layers(m, got_taps, want_taps, L):
    """Returns the number of differing codes per layer input; asserts the rule above."""
    lift = want_taps["codes_in.0"]
    assert np.array_equal(got_taps[0], lift), \
        f"lift codes differ at {int(np.sum(got_taps[0] != lift))} places"
    counts = [0]
    seen = np.zeros(lift.shape[:-1], bool)          # points with an earlier difference
    for i in range(L):
        got = got_taps[i + 1]
        want = want_taps[f"codes_in.{i + 1}"]
        diff = got != want
        counts.append(int(diff.sum()))
        if not diff.any():
            continue
        d = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert d.max() == 1, f"layer {i}: codes differ by {d.max()}"
        qp = m.qparams[f"locs.{i}.output"]
        r = want_taps[f"h.{i}"].astype(np.float64) / np.float64(np.float32(qp.scale))
        margin = 0.5 - np.abs(r - np.rint(r))          # code steps to the nearest boundary
        explained = (margin < BOUNDARY_MARGIN) | seen[..., None]
        bad = diff & ~explained
        assert not bad.any(), (
            f"layer {i}: {int(bad.sum())} codes differ away from a rounding boundary "
            f"(smallest margin {float(margin[bad].min()):.3g} code steps)")
        seen |= diff.any(axis=-1)
    return counts


def _compare(m, path, x, label):
    from neuroflow_b200.runtime import InferenceRuntime
    L, width = m.config["n_layers"], m.config["width"]
    want, want_taps = Oracle().fno2d_forward(m, x, mode=1, taps=True)
    rt = InferenceRuntime(path)
    rt.enable_int8_gemm()
    assert rt.is_int8_gemm_enabled()
    got, got_taps = _device_run_with_taps(rt, x, L, width)
    counts = _check_layers(m, got_taps, want_taps, L)
    n_codes = got_taps[0].size
    moved = int(np.sum(got != want))
    print(f"{label}: differing codes per layer input {counts} of {n_codes} each; "
          f"outputs moved {moved} of {got.size}")
    assert np.all(np.isfinite(got))
    assert moved == 0, f"{moved} outputs differ (max {np.abs(got - want).max()})"
    return counts


@pytest.mark.gpu
def test_fno2d_int8_headline_model_layer_by_layer():
    """The benchmarked model itself (configs[2]: 128x128, width 64, 12x12 modes, 4
    layers, calibration on 32 samples), two of the benchmark's samples: row blocks of
    32 rows, paired rows q / q + 64, the tensor-core forward transform."""
    sys.path.insert(0, ROOT)
    import bench
    path = bench.model_path(0)
    m = ir.read(path)
    x = bench.inputs(100, 2)
    _compare(m, path, x, "configs[2] B=2")


@pytest.mark.gpu
@pytest.mark.parametrize("B", [129, 257])
def test_fno2d_int8_full_and_partial_mix_tiles(tmp_path, B):
    """Batches above 128 samples: full and partial 128-sample tiles of the tensor-core
    mix, and persistent layer / transform grids that wrap the SMs several times."""
    m = synth.fno2d_model(17, width=64, mh=12, mw=12, L=4, H=32, W=32, n_calib=4,
                          calib_chunk=4)
    p = os.path.join(str(tmp_path), "m.nneuroir")
    ir.write(p, m)
    x = synth.fno2d_inputs(np.random.default_rng(B), B, 32, 32)
    _compare(m, p, x, f"32x32 B={B}")


@pytest.mark.gpu
@pytest.mark.parametrize("H,W,B", [(128, 128, 3), (64, 64, 4), (256, 128, 1)])
def test_fno2d_int8_geometries_layer_by_layer(tmp_path, H, W, B):
    """Other grids through the same kernels: the W = 128 transform with 32- and 64-row
    blocks, and the general (W != 128) path."""
    m = synth.fno2d_model(23, width=64, mh=12, mw=12, L=4, H=H, W=W, n_calib=2,
                          calib_chunk=2)
    p = os.path.join(str(tmp_path), "m.nneuroir")
    ir.write(p, m)
    x = synth.fno2d_inputs(np.random.default_rng(H + W + B), B, H, W)
    _compare(m, p, x, f"{H}x{W} B={B}")


@pytest.mark.gpu
def test_code_taps_reject_a_small_buffer(tmp_path):
    import torch
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.fno2d_model(2, width=64, mh=12, mw=12, L=2, H=32, W=32, n_calib=2, calib_chunk=2)
    p = os.path.join(str(tmp_path), "m.nneuroir")
    ir.write(p, m)
    rt = InferenceRuntime(p)
    rt.enable_int8_gemm()
    x = torch.zeros((2, 32, 32, 3), device="cuda")
    y = torch.zeros((2, 32, 32, 1), device="cuda")
    small = torch.zeros(3 * 2 * 32 * 32 * 64 - 1, dtype=torch.int8, device="cuda")
    rt.set_code_taps(small)
    with pytest.raises(RuntimeError, match="code-tap buffer too small"):
        rt.run_device(x, y)
    rt.set_code_taps(None)
    rt.run_device(x, y)
    torch.cuda.synchronize()
    rt.check()
