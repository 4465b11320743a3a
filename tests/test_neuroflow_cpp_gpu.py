"""The `neuroflow_cpp` module on the GPU runtime, called as the reference's own tests call
the reference module (tests/test_int8_gemm_inline.py:120-223, tests/test_fp8_e4m3.py,
the module functions of cpp/bindings/pybind_module.cpp:58-238), on models that the
reference's exporter wrote (tests/golden, made by make_golden.py) and against outputs of
the reference C++ runtime."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.gpu
def test_fno1d_int8_gemm_dispatch_flag():
    """test_int8_gemm_inline.py:120-141: the flag is False until enable_int8_gemm() on
    a per-channel calibrated FNO1d IR, True after."""
    import neuroflow_cpp
    rt = neuroflow_cpp.InferenceRuntime(os.path.join(GOLD, "fno1d_pc.nneuroir"))
    assert rt.op() == "FNO1d"
    assert not rt.is_int8_gemm_enabled()
    rt.enable_int8_gemm()
    assert rt.is_int8_gemm_enabled()


@pytest.mark.gpu
def test_fno1d_int8_gemm_matches_fp32_within_int8_budget():
    """test_int8_gemm_inline.py:144-223: the INT8-dispatched forward stays within the
    INT8 budget of the FP32 path; here both also equal the reference runtime's outputs."""
    import neuroflow_cpp
    d = np.load(os.path.join(GOLD, "fno1d.npz"))
    path = os.path.join(GOLD, "fno1d_pc.nneuroir")
    rt_fp32 = neuroflow_cpp.InferenceRuntime(path)
    y_fp32 = np.zeros(d["y_pc"].shape, dtype=np.float32)
    rt_fp32.run(d["x"], y_fp32)
    rt_int8 = neuroflow_cpp.InferenceRuntime(path)
    rt_int8.enable_int8_gemm()
    assert rt_int8.is_int8_gemm_enabled()
    y_int8 = np.zeros(d["y_pc_int8"].shape, dtype=np.float32)
    rt_int8.run(d["x"], y_int8)
    assert float(np.abs(y_fp32 - y_int8).max()) < 1.0
    for got, want in ((y_fp32, d["y_pc"]), (y_int8, d["y_pc_int8"])):
        assert np.allclose(got, want, rtol=1e-5, atol=1e-6 * np.abs(want).max())


@pytest.mark.gpu
def test_infer_and_infer_arrays_on_a_reference_exported_fno2d(tmp_path):
    """pybind_module.cpp:61-158 on the reference-exported FNO2d (GELU, fp32: rtol 1e-5
    of the reference runtime's output)."""
    import neuroflow_cpp
    d = np.load(os.path.join(GOLD, "fno2d_q.npz"))
    path = os.path.join(GOLD, "fno2d_plain.nneuroir")
    want = d["y_plain"]
    tol = dict(rtol=1e-5, atol=1e-6 * float(np.abs(want).max()))
    y = neuroflow_cpp.infer_arrays(path, d["x"])
    assert y.shape == want.shape and y.dtype == np.float32
    assert np.allclose(y, want, **tol)
    xin, yout = str(tmp_path / "x.npy"), str(tmp_path / "y.npy")
    np.save(xin, d["x"])
    assert neuroflow_cpp.infer(path, xin, yout) == "ok"
    assert np.array_equal(np.load(yout), y)


@pytest.mark.gpu
def test_errors_raise_runtime_error_with_the_reference_messages(tmp_path):
    import neuroflow_cpp
    with pytest.raises(RuntimeError, match="^load IR failed"):
        neuroflow_cpp.infer_arrays(str(tmp_path / "missing.nneuroir"), np.zeros((1, 4, 1), np.float32))
    with pytest.raises(RuntimeError, match="^create runtime failed"):
        neuroflow_cpp.InferenceRuntime(str(tmp_path / "missing.nneuroir"))
    path = os.path.join(GOLD, "fno1d_pc.nneuroir")
    with pytest.raises(RuntimeError, match="input rank mismatch for op FNO1d"):
        neuroflow_cpp.infer_arrays(path, np.zeros((4, 2), np.float32))
    rt = neuroflow_cpp.InferenceRuntime(path)
    with pytest.raises(RuntimeError, match="^Run failed"):
        rt.run(np.zeros((1, 64, 3), np.float32), np.zeros((1, 64, 1), np.float32))
    with pytest.raises(RuntimeError, match="not DeepONet"):
        neuroflow_cpp.infer_deeponet_arrays(path, np.zeros((1, 4, 1), np.float32),
                                            np.zeros((1, 4, 1), np.float32))


@pytest.mark.gpu
def test_fp8_helpers_known_answers_and_oracle_sweep():
    """The reference's FP8 known answers (cpp/tests/test_fp8_e4m3.cpp:50-140, the values
    of tests/test_oracle_pin.py) through fp8_e4m3_to_bits / from_bits on the GPU, and a
    sweep of float patterns bit-exact against the CPU restatement of fp8_e4m3.h."""
    import neuroflow_cpp
    from oracle.cpu import Oracle
    kat = [(0.0, 0x00), (-0.0, 0x80), (1.0, 0x38), (-1.0, 0xB8), (448.0, 0x7E),
           (-448.0, 0xFE), (1.0625, 0x38), (1.1875, 0x3A), (1.10, 0x39), (1000.0, 0x7E),
           (-1000.0, 0xFE), (float("inf"), 0x7E), (float("-inf"), 0xFE),
           (float("nan"), 0x7F), (7.6 / 512, 0x07), (7.99 / 512, 0x07), (1.0 / 64, 0x08),
           (3.0 / 512, 0x03)]
    v = np.array([a for a, _ in kat], np.float32)
    assert neuroflow_cpp.fp8_e4m3_to_bits(v).tolist() == [b for _, b in kat]
    dec = neuroflow_cpp.fp8_e4m3_from_bits(np.arange(256, dtype=np.uint8))
    assert dec[0x38] == 1.0 and dec[0x7E] == 448.0 and dec[0x08] == 1.0 / 64
    assert np.isnan(dec[0x7F]) and np.isnan(dec[0xFF])
    o = Oracle()
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    f = bits.view(np.float32)
    assert np.array_equal(neuroflow_cpp.fp8_e4m3_to_bits(f), o.fp32_to_e4m3(f))
    want_dec = np.array([o.lib.nfo_e4m3_to_fp32(i) for i in range(256)], np.float32)
    assert np.array_equal(dec.view(np.uint32), want_dec.view(np.uint32))
    # fake-quant = decode(encode(clamp(x / scale))) * scale, scale 0 dividing by 1
    x = (rng.standard_normal(4096) * 3).astype(np.float32)
    for scale in (np.float32(0.05), np.float32(0.0)):
        inv = np.float32(1.0) if scale == 0 else np.float32(1.0) / scale
        xs = np.clip(x * inv, -448.0, 448.0).astype(np.float32)
        want = (want_dec[o.fp32_to_e4m3(xs)] * scale).astype(np.float32)
        assert np.array_equal(neuroflow_cpp.fp8_e4m3_fake_quant(x, float(scale)), want)


@pytest.mark.gpu
def test_fp8_hardware_conversions_match_the_reference_encoder():
    """The FP8 executors encode and decode with the hardware E4M3 conversions, patched to
    the reference's subnormal rule ([7.5, 8) * 2^-9 stays at code 7) and NaN codes, with
    the conversion's own saturation standing in for the clamp to +-448: every fp32 bit
    pattern (the reference encoder's input clamped) and every code agree bit for bit with
    the reference's encoder and decoder (fp8_e4m3.h:106-284)."""
    import ctypes
    from neuroflow_b200 import _nfx
    n = ctypes.c_ulonglong(12345)
    assert _nfx.lib.nfx_fp8_e4m3_selfcheck(ctypes.byref(n)) == 0
    assert n.value == 0
