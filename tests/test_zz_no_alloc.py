"""The allocation-free FNO2d entry point (nfx_runtime_run_device_noalloc) against the
ordinary device entry point (nfx_runtime_run_device), through the C-ABI.

It is meant for callers that cannot allocate device memory while they run inference;
this file checks that it gives the same outputs as the allocating entry point on two
calls in a row (the second call reuses the fixed scratch the first one left behind),
that it allocates no device memory, and that a batch too large for its fixed scratch
is refused with a clear error.  The file name keeps it last in collection order.
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
    x = torch.from_numpy(synth.fno2d_inputs(np.random.default_rng(4), B, H, W)).cuda()
    return m, rt, x


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
def test_noalloc_matches_allocating_entry_point(tmp_path):
    import torch
    m, rt, x = _setup(tmp_path)
    y_ref = torch.empty(x.shape[:-1] + (1,), dtype=torch.float32, device="cuda")
    rt.run_device(x, y_ref)
    torch.cuda.synchronize()
    rt.check()
    want = y_ref.cpu().numpy()
    step = m.qparams["proj_out.output"].scale
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
        d = np.abs(got - want)
        assert np.all(np.isfinite(got))
        # the tolerance of the FNO2d end-to-end tests (units of the output step)
        assert np.mean(d > 0) < 1e-3 and d.max() <= 2 * step, (call, d.max(), np.mean(d > 0))


@pytest.mark.gpu
def test_noalloc_rejects_batches_beyond_its_scratch(tmp_path):
    import torch
    m, rt, _ = _setup(tmp_path)
    x = torch.zeros((16, 128, 128, 3), dtype=torch.float32, device="cuda")
    y = torch.zeros((16, 128, 128, 1), dtype=torch.float32, device="cuda")
    rc = _call_noalloc(rt, x, y)
    assert rc == 1
    assert "32 MiB" in rt._err()
