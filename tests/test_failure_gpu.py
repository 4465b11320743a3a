"""The failure path of the bounded device waits, without a GPU fault.

Every wait inside the kernels is bounded; when one runs out the kernel raises its
abort flag, records the timeout in the device error word, waits for its own loads and
MMAs in flight, releases its tensor memory and returns, and the host reports the error
as NFX_INTERNAL.  These tests shrink the INT8 GEMM kernel's wait budget to 1 ns
(nfx_debug_set_wait_budget_ns), far below the latency of its first TMA load: such a
budget is spent at the first retry of any wait that does not succeed at once, so the
pipeline waits give up; then they restore the default and check that the same
context computes the right result again.  Nothing is made to fault, trap or hang: the
drains before teardown keep their normal (bounded) budget."""
import ctypes as C
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, quant, synth


def _set_budget(ns):
    from neuroflow_b200 import _nfx
    f = _nfx.lib.nfx_debug_set_wait_budget_ns
    f.restype = None
    f.argtypes = [C.c_ulonglong]
    f(int(ns))


@pytest.fixture
def tiny_budget():
    yield _set_budget
    _set_budget(0)


@pytest.mark.gpu
def test_gemm_wait_timeout_is_reported_and_the_context_recovers(tiny_budget):
    import torch
    from neuroflow_b200 import _nfx
    from oracle.cpu import Oracle
    c = quant.gemm_case(3, 1 << 20, 64, 64)
    want, _ = Oracle().int8_gemm_rows(c["Aq"], c["sA"], c["zA"], c["Wq"], c["sW"], c["zW"],
                                      c["sum_w"], c["bias"], gelu=False)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in c.items()}

    def gemm():
        return _nfx.int8_gemm(t["Aq"], t["Wq"], t["sW"], t["zW"], t["sum_w"], bias=t["bias"],
                              scale_a=t["sA"], zp_a=t["zA"])

    assert _nfx.device_errors() == 0
    tiny_budget(1)
    gemm()
    flags = _nfx.device_errors()          # synchronises; the launch itself succeeded
    assert flags != 0, "no wait ran out with a 1 ns budget"
    assert flags & ~0x1F == 0, hex(flags)  # only the wait-timeout bits
    tiny_budget(0)
    for _ in range(2):
        got = gemm().cpu().numpy()
        assert _nfx.device_errors() == 0
        assert np.array_equal(got, want)


@pytest.mark.gpu
def test_runtime_check_reports_internal_after_a_timeout(tmp_path, tiny_budget):
    """FNO1d with per-tensor activation qparams runs its local layers through the GEMM
    kernel; a timed-out wait surfaces as the reference's Internal status."""
    import torch
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.fno1d_model(5, width=64, modes=8, L=2, n=1024, n_calib=8, per_token=False)
    p = os.path.join(str(tmp_path), "fno1d.nneuroir")
    ir.write(p, m)
    rt = InferenceRuntime(p)
    rt.enable_int8_gemm()
    x = torch.from_numpy(synth.fno1d_inputs(np.random.default_rng(1), 256, 1024)).cuda()
    y = torch.empty((256, 1024, 1), device="cuda")
    rt.run_device(x, y)
    rt.check()
    want = y.cpu().numpy()
    tiny_budget(1)
    rt.run_device(x, y)
    with pytest.raises(RuntimeError, match="gave up waiting"):
        rt.check()
    tiny_budget(0)
    y.fill_(float("nan"))
    rt.run_device(x, y)
    rt.check()
    assert np.array_equal(y.cpu().numpy(), want)
