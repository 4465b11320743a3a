"""The allocation-free FNO2d entry point (nfx_runtime_run_device_noalloc) against the
ordinary device entry point (nfx_runtime_run_device), through the C-ABI.

It serves callers that cannot allocate device memory while they run inference (their
device memory belongs to another allocator, or their rules forbid allocating after
start-up).  This file checks that it gives bit-identical outputs to the allocating
entry point on two calls in a row (the second call reuses the fixed scratch the first
one left behind), on a 32 x 32 grid and on the benchmarked 128 x 128 grid, where both
run the tensor-core forward transform; that the outputs equal the CPU restatement's;
that the second call allocates no device memory; and that the capacity limit sits
where the documentation puts it (13 samples of 128 x 128 at width 64 accepted, 14
refused).  The file name keeps it last in collection order.
"""
import ctypes as C
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, synth


def _setup(tmp_path, B=3, H=32, W=32):
    import torch
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.fno2d_model(21, width=64, mh=12, mw=12, L=2, H=H, W=W, n_calib=2, calib_chunk=2)
    p = os.path.join(str(tmp_path), "noalloc.nneuroir")
    ir.write(p, m)
    rt = InferenceRuntime(p, 0)
    rt.enable_int8_gemm()
    assert rt.is_int8_gemm_enabled()
    xh = synth.fno2d_inputs(np.random.default_rng(4), B, H, W)
    return m, rt, xh, torch.from_numpy(xh).cuda()


def _call_noalloc(rt, x, y):
    import torch
    from neuroflow_b200 import _nfx
    fn = _nfx.lib.nfx_runtime_run_device_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_int64), C.c_int, C.c_void_p,
                   C.POINTER(C.c_int64), C.c_int, C.c_void_p]
    xs = (C.c_int64 * 4)(*x.shape)
    ys = (C.c_int64 * 4)(*y.shape)
    stream = torch.cuda.current_stream().cuda_stream
    return fn(rt._h, C.c_void_p(x.data_ptr()), xs, 4, C.c_void_p(y.data_ptr()), ys, 4,
              C.c_void_p(stream))


@pytest.mark.gpu
@pytest.mark.parametrize("H,W,B", [(32, 32, 3), (128, 128, 2)])
def test_noalloc_matches_allocating_entry_point(tmp_path, H, W, B):
    import torch
    from oracle.cpu import Oracle
    m, rt, xh, x = _setup(tmp_path, B, H, W)
    y_ref = torch.empty(x.shape[:-1] + (1,), dtype=torch.float32, device="cuda")
    rt.run_device(x, y_ref)
    torch.cuda.synchronize()
    rt.check()
    want = y_ref.cpu().numpy()
    # the allocating entry point itself equals the CPU restatement on this input
    assert np.array_equal(want, Oracle().fno2d_forward(m, xh, mode=1))
    free_before = None
    for call in range(2):
        y = torch.full_like(y_ref, float("nan"))
        torch.cuda.synchronize()
        if call == 1:
            free_before = torch.cuda.mem_get_info()[0]
        rc = _call_noalloc(rt, x, y)
        assert rc == 0, rt._err()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before
        got = y.cpu().numpy()
        # same kernels, same inputs: bit-identical to the allocating entry point
        assert np.array_equal(got, want), (call, float(np.nanmax(np.abs(got - want))))


@pytest.mark.gpu
def test_noalloc_capacity_limit(tmp_path):
    """2,465,792 B per 128x128 sample at width 64 plus 66,048 B of header and tables:
    13 samples fit in the 32 MiB, 14 do not."""
    import torch
    m, rt, _, _ = _setup(tmp_path, 1, 128, 128)
    for B, ok in ((13, True), (14, False)):
        x = torch.zeros((B, 128, 128, 3), dtype=torch.float32, device="cuda")
        y = torch.full((B, 128, 128, 1), float("nan"), dtype=torch.float32, device="cuda")
        rc = _call_noalloc(rt, x, y)
        if ok:
            assert rc == 0, rt._err()
            assert bool(torch.isfinite(y).all())
        else:
            assert rc == 1
            assert "32 MiB" in rt._err() and "13" in rt._err()
