"""Python front-end of the GPU runtime, mirroring the reference `neuroflow_cpp` module
(cpp/bindings/pybind_module.cpp:61-197): `InferenceRuntime(path)` with `op()`,
`enable_int8_gemm()`, `is_int8_gemm_enabled()` and `run(x, y)`, plus `infer_arrays`.
Errors raise RuntimeError like the reference binding.  Every call goes through the
C-ABI of libnfx.so; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _nfx

_lib = _nfx.lib


def _shape(a):
    return (C.c_int64 * a.ndim)(*a.shape)


class InferenceRuntime:
    """Persistent runtime (load once, run many), bound to one CUDA device."""

    def __init__(self, ir_path: str, device: int = 0):
        h = C.c_void_p()
        rc = _lib.nfx_runtime_create(str(ir_path).encode(), int(device), C.byref(h))
        if rc != 0:
            raise RuntimeError("create runtime failed: " + _lib.nfx_last_error().decode())
        self._h = h
        self.device = int(device)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _lib.nfx_runtime_destroy(h)
            self._h = None

    def close(self):
        self.__del__()

    def op(self) -> str:
        return _lib.nfx_runtime_op(self._h).decode()

    def enable_int8_gemm(self) -> None:
        _lib.nfx_runtime_enable_int8_gemm(self._h)

    def is_int8_gemm_enabled(self) -> bool:
        return bool(_lib.nfx_runtime_is_int8_gemm_enabled(self._h))

    def enable_fp8(self) -> None:
        """FNO3d: switch to the FP8 E4M3 executor (needs NIRQ FP8 scales)."""
        _lib.nfx_runtime_enable_fp8(self._h)

    def is_fp8_enabled(self) -> bool:
        return bool(_lib.nfx_runtime_is_fp8_enabled(self._h))

    def _err(self) -> str:
        return _lib.nfx_runtime_last_error(self._h).decode()

    def run(self, x: np.ndarray, y: np.ndarray) -> None:
        """x, y: float32 C-contiguous host arrays (y is written in place)."""
        if not (isinstance(y, np.ndarray) and y.dtype == np.float32 and y.flags.c_contiguous):
            raise RuntimeError("Run failed: y must be a C-contiguous float32 array")
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = _lib.nfx_runtime_run(self._h, x.ctypes.data_as(C.c_void_p), _shape(x), x.ndim,
                                  y.ctypes.data_as(C.c_void_p), _shape(y), y.ndim)
        if rc != 0:
            raise RuntimeError("Run failed: " + self._err())

    def run_tokenmixer2d(self, x: np.ndarray, y: np.ndarray) -> None:
        """The reference's `run_tokenmixer2d` (x (B, h, w, in_dim) -> y in place)."""
        if not (isinstance(y, np.ndarray) and y.dtype == np.float32 and y.flags.c_contiguous):
            raise RuntimeError("RunTokenMixer2D failed: y must be a C-contiguous float32 array")
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = _lib.nfx_runtime_run_tokenmixer2d(self._h, x.ctypes.data_as(C.c_void_p), _shape(x),
                                               x.ndim, y.ctypes.data_as(C.c_void_p), _shape(y),
                                               y.ndim)
        if rc != 0:
            raise RuntimeError("RunTokenMixer2D failed: " + self._err())

    @staticmethod
    def _stream(x, stream):
        import torch
        if stream is None:
            return torch.cuda.current_stream(x.device).cuda_stream
        return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream

    def run_device(self, x, y, stream=None) -> None:
        """x, y: CUDA float32 tensors on this runtime's device; asynchronous on `stream`
        (a torch.cuda.Stream or raw handle; default: the current torch stream)."""
        stream = self._stream(x, stream)
        xs = (C.c_int64 * x.dim())(*x.shape)
        ys = (C.c_int64 * y.dim())(*y.shape)
        rc = _lib.nfx_runtime_run_device(self._h, C.c_void_p(x.data_ptr()), xs, x.dim(),
                                         C.c_void_p(y.data_ptr()), ys, y.dim(), C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError("Run failed: " + self._err())

    def run_tokenmixer2d_device(self, x, y, stream=None) -> None:
        stream = self._stream(x, stream)
        xs = (C.c_int64 * x.dim())(*x.shape)
        ys = (C.c_int64 * y.dim())(*y.shape)
        rc = _lib.nfx_runtime_run_tokenmixer2d_device(self._h, C.c_void_p(x.data_ptr()), xs,
                                                      x.dim(), C.c_void_p(y.data_ptr()), ys,
                                                      y.dim(), C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError("RunTokenMixer2D failed: " + self._err())

    def profile(self, enable: bool = True) -> None:
        """Enable (and reset) or disable per-kernel CUDA-event timing."""
        rc = _lib.nfx_runtime_profile_enable(self._h, int(bool(enable)))
        if rc != 0:
            raise RuntimeError(self._err())

    def profile_read(self) -> dict:
        """{kernel name: (launches, total device ms)} since profiling was enabled."""
        out = {}
        for i in range(_lib.nfx_runtime_profile_count(self._h)):
            name = C.c_char_p()
            n = C.c_int()
            ms = C.c_double()
            rc = _lib.nfx_runtime_profile_entry(self._h, i, C.byref(name), C.byref(n), C.byref(ms))
            if rc != 0:
                raise RuntimeError(self._err())
            out[name.value.decode()] = (n.value, ms.value)
        return out

    def check(self) -> None:
        rc = _lib.nfx_runtime_check(self._h)
        if rc != 0:
            raise RuntimeError("device error: " + self._err())


def infer_arrays(model_path: str, x: np.ndarray, out_channels: int, enable_int8: bool = True,
                 device: int = 0) -> np.ndarray:
    """Load, run once, return y (the reference's `infer_arrays`, with the output channel
    count given explicitly)."""
    rt = InferenceRuntime(model_path, device)
    if enable_int8:
        rt.enable_int8_gemm()
    y = np.zeros(tuple(x.shape[:-1]) + (out_channels,), np.float32)
    rt.run(x, y)
    return y
