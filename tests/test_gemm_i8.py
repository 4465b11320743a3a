"""INT8 GEMM (tcgen05 kind::i8) vs the CPU restatement of the reference epilogue.

Bit-exact: the int32 accumulators (checked through unit scales) and the fp32 outputs
without activation.  With GELU the outputs agree within rtol 1e-5 plus an absolute
term of 2^-22 * max|y|: the kernel evaluates GELU as z * sigmoid(2u) with the hardware
exp2 approximation (a few ulp from the exact GELU), while the reference's
0.5 z (1 + tanh u) with glibc tanhf loses relative accuracy to cancellation on tiny
outputs (u << 0)."""
import numpy as np
import pytest

from neuroflow_b200 import quant
from oracle.cpu import Oracle

SIZES = [32, 64, 128, 256]


def _run_gpu(case, act, unit=False):
    import torch
    from neuroflow_b200 import _nfx
    dev = torch.device("cuda:0")
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in case.items()}
    return _nfx.int8_gemm(t["Aq"], t["Wq"], t["sW"], t["zW"], t["sum_w"], bias=t["bias"],
                          scale_a=t["sA"], zp_a=t["zA"], act=act).cpu().numpy()


def _unit(case):
    c = dict(case)
    c["sA"] = np.ones_like(case["sA"])
    c["sW"] = np.ones_like(case["sW"])
    c["zA"] = np.zeros_like(case["zA"])
    c["bias"] = np.zeros_like(case["bias"])
    return c


@pytest.mark.gpu
@pytest.mark.parametrize("K", SIZES)
@pytest.mark.parametrize("N", SIZES)
def test_gemm_exact_no_act(K, N):
    o = Oracle()
    for M in (1, 127, 128, 129, 1000):
        case = quant.gemm_case(1000 * K + N + M, M, K, N)
        want, acc = o.int8_gemm_rows(case["Aq"], case["sA"], case["zA"], case["Wq"], case["sW"],
                                     case["zW"], case["sum_w"], case["bias"], gelu=False)
        got = _run_gpu(case, act=0)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (M, K, N)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N", [(32, 32), (64, 64), (128, 128), (256, 256), (64, 256)])
def test_gemm_int32_accumulators_exact(K, N):
    # unit scales, zp_a = 0, zero bias: y = float(acc - zp_w * sum_a), |.| < 2^24,
    # so the float output is the reference's integer exactly.
    o = Oracle()
    case = _unit(quant.gemm_case(7 + K + N, 777, K, N))
    want, acc = o.int8_gemm_rows(case["Aq"], case["sA"], case["zA"], case["Wq"], case["sW"],
                                 case["zW"], case["sum_w"], None, gelu=False)
    got = _run_gpu(case, act=0)
    sum_a = case["Aq"].astype(np.int64).sum(axis=1)
    v = acc.astype(np.int64) - case["zW"][None, :].astype(np.int64) * sum_a[:, None]
    assert np.abs(v).max() < 2 ** 24
    assert np.array_equal(got.astype(np.int64), v)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N", [(32, 32), (64, 64), (128, 128), (256, 256)])
def test_gemm_gelu_tolerance(K, N):
    o = Oracle()
    case = quant.gemm_case(11 + K, 4096 + 17, K, N)
    want, _ = o.int8_gemm_rows(case["Aq"], case["sA"], case["zA"], case["Wq"], case["sW"],
                               case["zW"], case["sum_w"], case["bias"], gelu=True)
    got = _run_gpu(case, act=1)
    tol = 1e-5 * np.abs(want) + 2.0 ** -22 * np.abs(want).max()
    assert np.all(np.abs(got - want) <= tol)
    # away from the cancellation region the two agree to a few ulp
    big = np.abs(want) > 1e-3 * np.abs(want).max()
    ulp = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
    assert np.percentile(ulp[big], 99) <= 8 and np.median(ulp[big]) <= 2


@pytest.mark.gpu
def test_gemm_zero_rows_and_bad_shapes():
    import torch
    from neuroflow_b200 import _nfx
    dev = torch.device("cuda:0")
    W = torch.zeros((64, 64), dtype=torch.int8, device=dev)
    s = torch.ones(64, device=dev)
    z = torch.zeros(64, dtype=torch.int32, device=dev)
    A = torch.zeros((0, 64), dtype=torch.int8, device=dev)
    out = _nfx.int8_gemm(A, W, s, z, z)
    assert out.shape == (0, 64)
    with pytest.raises(_nfx.NfxError) as ei:
        _nfx.int8_gemm(torch.zeros((4, 48), dtype=torch.int8, device=dev),
                       torch.zeros((64, 48), dtype=torch.int8, device=dev), s, z, z)
    assert ei.value.code == 1
    assert _nfx.device_errors() == 0
