"""neuroflow_cpp -- the reference's Python module (cpp/bindings/pybind_module.cpp:58-238)
on the B200 runtime: the same names, arguments, results and RuntimeError messages,
served by libnfx.so (every call runs on the GPU; there is no CPU path).

    import neuroflow_cpp
    neuroflow_cpp.infer(model_path, input_npy, output_npy)        # -> "ok"
    y = neuroflow_cpp.infer_arrays(model_path, x)
    rt = neuroflow_cpp.InferenceRuntime(model_path)
    rt.op(); rt.enable_int8_gemm(); rt.is_int8_gemm_enabled(); rt.run(x, y)
    neuroflow_cpp.fp8_e4m3_fake_quant(a, scale)                   # fp8_e4m3_pybind.h:24-66
    neuroflow_cpp.fp8_e4m3_to_bits(a); neuroflow_cpp.fp8_e4m3_from_bits(b)

Runtimes are created on CUDA device 0, or on $NFX_DEVICE.  Every op of the reference
runtime runs on the GPU: FNO1d/2d/3d through `run`, TokenMixer, GraphOp, TokenMixer2D
and GraphOp2D through their own Run calls (as `infer` dispatches them), DeepONet through
`infer_deeponet_arrays`.
"""
from __future__ import annotations

import ctypes as _C
import os as _os

import numpy as _np

from neuroflow_b200 import _nfx
from neuroflow_b200.runtime import InferenceRuntime as _Runtime

__all__ = ["infer", "infer_arrays", "infer_deeponet_arrays", "InferenceRuntime",
           "fp8_e4m3_fake_quant", "fp8_e4m3_to_bits", "fp8_e4m3_from_bits"]

_lib = _nfx.lib
_lib.nfx_fp8_e4m3_to_bits_host.restype = _C.c_int
_lib.nfx_fp8_e4m3_to_bits_host.argtypes = [_C.c_void_p, _C.c_void_p, _C.c_int64]
_lib.nfx_fp8_e4m3_from_bits_host.restype = _C.c_int
_lib.nfx_fp8_e4m3_from_bits_host.argtypes = [_C.c_void_p, _C.c_void_p, _C.c_int64]
_lib.nfx_fp8_e4m3_fake_quant_host.restype = _C.c_int
_lib.nfx_fp8_e4m3_fake_quant_host.argtypes = [_C.c_void_p, _C.c_float, _C.c_void_p, _C.c_int64]

# input rank and output-channel slot of the IR config per op (pybind_module.cpp:74-89)
_RANK = {"FNO1d": 3, "FNO2d": 4, "FNO3d": 5, "TokenMixer": 3, "GraphOp": 3,
         "TokenMixer2D": 4, "GraphOp2D": 4}
_RUN = {"TokenMixer": "run_tokenmixer", "GraphOp": "run_graphop", "TokenMixer2D": "run_tokenmixer2d",
        "GraphOp2D": "run_graphop2d"}


def _device() -> int:
    return int(_os.environ.get("NFX_DEVICE", "0"))


def _load(model_path: str):
    try:
        op, cfg, _, _ = _nfx.load_neuroir(model_path)
    except _nfx.NfxError as e:
        raise RuntimeError("load IR failed: " + str(e).split("] ", 1)[-1]) from None
    return op, cfg


def _run_loaded(model_path: str, op: str, cfg, x: _np.ndarray) -> _np.ndarray:
    if op not in _RANK or x.ndim != _RANK[op]:
        raise RuntimeError("input rank mismatch for op " + op)
    try:
        rt = _Runtime(model_path, _device())
    except RuntimeError as e:
        raise RuntimeError("create runtime failed: " + str(e).split(": ", 1)[-1]) from None
    y = _np.zeros(tuple(x.shape[:-1]) + (cfg[1],), _np.float32)
    try:
        getattr(rt, _RUN.get(op, "run"))(x, y)
    except RuntimeError as e:
        raise RuntimeError("infer failed: " + str(e).split(": ", 1)[-1]) from None
    finally:
        rt.close()
    return y


def infer(model_path: str, input_path: str, output_path: str) -> str:
    """Load .nneuroir, read .npy, run, write .npy (pybind_module.cpp:61-111)."""
    op, cfg = _load(model_path)
    try:
        x = _np.load(input_path)
    except Exception as e:  # the reference reports its npy reader's message
        raise RuntimeError("read input failed: " + str(e)) from None
    x = _np.ascontiguousarray(x, dtype=_np.float32)
    y = _run_loaded(model_path, op, cfg, x)
    try:
        _np.save(output_path, y)
    except Exception as e:
        raise RuntimeError("write output failed: " + str(e)) from None
    return "ok"


def infer_arrays(model_path: str, x) -> _np.ndarray:
    """In-memory inference (pybind_module.cpp:113-158): returns y."""
    op, cfg = _load(model_path)
    return _run_loaded(model_path, op, cfg, _np.ascontiguousarray(x, dtype=_np.float32))


def infer_deeponet_arrays(model_path: str, u, y) -> _np.ndarray:
    """DeepONet in memory (pybind_module.cpp:200-233): out (batch, n_query, out_channels)
    with batch and n_query taken from y."""
    op, cfg = _load(model_path)
    if op != "DeepONet":
        raise RuntimeError("infer_deeponet_arrays: model op is " + op + ", not DeepONet")
    u = _np.ascontiguousarray(u, dtype=_np.float32)
    y = _np.ascontiguousarray(y, dtype=_np.float32)
    if u.ndim != 3:
        raise RuntimeError("DeepONet u must be 3D (batch, n_sensor, in_branch)")
    if y.ndim != 3:
        raise RuntimeError("DeepONet y must be 3D (batch, n_query, in_trunk)")
    try:
        rt = _Runtime(model_path, _device())
    except RuntimeError as e:
        raise RuntimeError("create runtime failed: " + str(e).split(": ", 1)[-1]) from None
    out = _np.zeros((y.shape[0], y.shape[1], cfg[3]), _np.float32)
    try:
        rt.run_deeponet(u, y, out)
    except RuntimeError as e:
        raise RuntimeError("infer failed: " + str(e).split(": ", 1)[-1]) from None
    finally:
        rt.close()
    return out


class InferenceRuntime:
    """Persistent runtime (load once, run many) -- pybind_module.cpp:160-197."""

    def __init__(self, ir_path: str):
        try:
            self._rt = _Runtime(ir_path, _device())
        except RuntimeError as e:
            raise RuntimeError("create runtime failed: " + str(e).split(": ", 1)[-1]) from None

    def op(self) -> str:
        return self._rt.op()

    def enable_int8_gemm(self) -> None:
        self._rt.enable_int8_gemm()

    def is_int8_gemm_enabled(self) -> bool:
        return self._rt.is_int8_gemm_enabled()

    def run(self, x, y) -> None:
        """FNO1d/2d/3d inference into the pre-allocated float32 array y."""
        self._rt.run(x, y)

    # calls of the reference's C++ runtime that its Python class does not expose
    def run_tokenmixer2d(self, x, y) -> None:
        self._rt.run_tokenmixer2d(x, y)

    def run_tokenmixer(self, x, y) -> None:
        self._rt.run_tokenmixer(x, y)

    def run_graphop(self, x, y) -> None:
        self._rt.run_graphop(x, y)

    def run_graphop2d(self, x, y) -> None:
        self._rt.run_graphop2d(x, y)

    def run_deeponet(self, u, y, out) -> None:
        self._rt.run_deeponet(u, y, out)

    def enable_fp8(self) -> None:
        self._rt.enable_fp8()

    def is_fp8_enabled(self) -> bool:
        return self._rt.is_fp8_enabled()


def _vec(a, dtype):
    a = _np.ascontiguousarray(a, dtype=dtype)
    if a.ndim != 1:
        raise RuntimeError("array has incorrect number of dimensions: %d; expected 1" % a.ndim)
    return a


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(_lib.nfx_last_error().decode())


def fp8_e4m3_fake_quant(in_, scale: float) -> _np.ndarray:
    """Per-tensor FP8 E4M3 fake-quant (fp8_e4m3.h:312-334), on the GPU."""
    a = _vec(in_, _np.float32)
    out = _np.empty_like(a)
    _check(_lib.nfx_fp8_e4m3_fake_quant_host(a.ctypes.data, float(scale), out.ctypes.data, a.size))
    return out


def fp8_e4m3_to_bits(in_) -> _np.ndarray:
    """FP32 -> FP8 E4M3 byte (fp8_e4m3.h:106-221, 286), on the GPU."""
    a = _vec(in_, _np.float32)
    out = _np.empty(a.shape, _np.uint8)
    _check(_lib.nfx_fp8_e4m3_to_bits_host(a.ctypes.data, out.ctypes.data, a.size))
    return out


def fp8_e4m3_from_bits(in_) -> _np.ndarray:
    """FP8 E4M3 byte -> FP32 (fp8_e4m3.h:223-284, 295), on the GPU."""
    a = _vec(in_, _np.uint8)
    out = _np.empty(a.shape, _np.float32)
    _check(_lib.nfx_fp8_e4m3_from_bits_host(a.ctypes.data, out.ctypes.data, a.size))
    return out
