"""Python front-end of the GPU runtime, mirroring the reference `neuroflow_cpp` module
(cpp/bindings/pybind_module.cpp:61-197): `InferenceRuntime(path)` with `op()`,
`enable_int8_gemm()`, `is_int8_gemm_enabled()`, `run(x, y)`, and the reference runtime's
other Run calls (`run_tokenmixer2d`, `run_tokenmixer`, `run_graphop`, `run_graphop2d`,
`run_deeponet`), plus the module functions `infer`, `infer_arrays` and
`infer_deeponet_arrays`.
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

    def _run_other(self, name: str, label: str, x: np.ndarray, y: np.ndarray) -> None:
        if not (isinstance(y, np.ndarray) and y.dtype == np.float32 and y.flags.c_contiguous):
            raise RuntimeError(label + " failed: y must be a C-contiguous float32 array")
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = getattr(_lib, "nfx_runtime_run_" + name)(self._h, x.ctypes.data_as(C.c_void_p), _shape(x),
                                                     x.ndim, y.ctypes.data_as(C.c_void_p), _shape(y),
                                                     y.ndim)
        if rc != 0:
            raise RuntimeError(label + " failed: " + self._err())

    def run_tokenmixer(self, x: np.ndarray, y: np.ndarray) -> None:
        """RunTokenMixer (runtime.cpp:115-123): x (B, n_points, in_dim) -> y in place."""
        self._run_other("tokenmixer", "RunTokenMixer", x, y)

    def run_graphop(self, x: np.ndarray, y: np.ndarray) -> None:
        """RunGraphOp (runtime.cpp:125-133): x (B, n_nodes, in_dim) -> y in place."""
        self._run_other("graphop", "RunGraphOp", x, y)

    def run_graphop2d(self, x: np.ndarray, y: np.ndarray) -> None:
        """RunGraphOp2D (runtime.cpp:145-153): x (B, h, w, in_dim) -> y in place."""
        self._run_other("graphop2d", "RunGraphOp2D", x, y)

    def run_deeponet(self, u: np.ndarray, y: np.ndarray, out: np.ndarray) -> None:
        """RunDeepONet (runtime.cpp:103-113): u (B, n_sensor, in_branch), y (B, n_query,
        in_trunk) -> out (B, n_query, out_channels) in place."""
        if not (isinstance(out, np.ndarray) and out.dtype == np.float32 and out.flags.c_contiguous):
            raise RuntimeError("RunDeepONet failed: out must be a C-contiguous float32 array")
        u = np.ascontiguousarray(u, dtype=np.float32)
        y = np.ascontiguousarray(y, dtype=np.float32)
        rc = _lib.nfx_runtime_run_deeponet(self._h, u.ctypes.data_as(C.c_void_p), _shape(u), u.ndim,
                                           y.ctypes.data_as(C.c_void_p), _shape(y), y.ndim,
                                           out.ctypes.data_as(C.c_void_p), _shape(out), out.ndim)
        if rc != 0:
            raise RuntimeError("RunDeepONet failed: " + self._err())

    def run_deeponet_device(self, u, y, out, stream=None) -> None:
        stream = self._stream(out, stream)
        sh = lambda t: (C.c_int64 * t.dim())(*t.shape)
        rc = _lib.nfx_runtime_run_deeponet_device(self._h, C.c_void_p(u.data_ptr()), sh(u), u.dim(),
                                                  C.c_void_p(y.data_ptr()), sh(y), y.dim(),
                                                  C.c_void_p(out.data_ptr()), sh(out), out.dim(),
                                                  C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError("RunDeepONet failed: " + self._err())

    def run_other_device(self, name: str, x, y, stream=None) -> None:
        """Device-buffer RunTokenMixer / RunGraphOp / RunGraphOp2D (`name` "tokenmixer",
        "graphop" or "graphop2d") on `stream`."""
        stream = self._stream(x, stream)
        xs = (C.c_int64 * x.dim())(*x.shape)
        ys = (C.c_int64 * y.dim())(*y.shape)
        rc = getattr(_lib, "nfx_runtime_run_" + name + "_device")(
            self._h, C.c_void_p(x.data_ptr()), xs, x.dim(), C.c_void_p(y.data_ptr()), ys, y.dim(),
            C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError("Run failed: " + self._err())

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

    def set_code_taps(self, buf=None) -> None:
        """Parity taps: `buf` a byte CUDA tensor of at least (n_layers + 1) * batch *
        points * width bytes receives the codes of every layer input on each later
        device run (FNO2d INT8: int8, channel-last; FNO3d FP8: E4M3, channel-first on
        the padded grid); None turns the taps off."""
        if buf is None:
            rc = _lib.nfx_runtime_set_code_taps(self._h, None, 0)
        else:
            rc = _lib.nfx_runtime_set_code_taps(self._h, C.c_void_p(buf.data_ptr()),
                                                int(buf.numel() * buf.element_size()))
        if rc != 0:
            raise RuntimeError(self._err())

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


    # -- calibration on the GPU (nfx_calibrate_*) --------------------------------------
    def calibrate_begin(self, keep_values: bool = False) -> None:
        rc = _lib.nfx_calibrate_begin(self._h, int(bool(keep_values)))
        if rc != 0:
            raise RuntimeError("calibration failed: " + self._err())

    def calibrate_observe(self, x: np.ndarray) -> None:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = _lib.nfx_calibrate_observe(self._h, x.ctypes.data_as(C.c_void_p), _shape(x), x.ndim)
        if rc != 0:
            raise RuntimeError("calibration failed: " + self._err())

    def calibrate_results(self, percentile: float = 100.0) -> dict:
        """{".output" key: (scale, zero_point, fp8_scale, lo, hi)} of every observed
        Linear output."""
        out = {}
        for i in range(_lib.nfx_calibrate_count(self._h)):
            name = C.create_string_buffer(64)
            sc, zp, f8 = C.c_float(), C.c_int32(), C.c_float()
            lo, hi = C.c_double(), C.c_double()
            rc = _lib.nfx_calibrate_result(self._h, i, float(percentile), name, 64, C.byref(sc),
                                           C.byref(zp), C.byref(f8), C.byref(lo), C.byref(hi))
            if rc != 0:
                raise RuntimeError("calibration failed: " + self._err())
            out[name.value.decode()] = (sc.value, zp.value, f8.value, lo.value, hi.value)
        return out

    def calibrate_end(self) -> None:
        _lib.nfx_calibrate_end(self._h)

    def run_sharded(self, comm: "Comm", x, y, root: int = -1, stream=None) -> None:
        """Batch partitioned over the ranks of `comm` (one process per GPU): x, y are the
        WHOLE batch as CUDA tensors on this runtime's device; this rank computes its
        slice and NCCL gathers the outputs into every rank's y (root < 0) or into the
        root's y.  Every rank makes the same call.  Asynchronous on `stream`."""
        stream = self._stream(x, stream)
        xs = (C.c_int64 * x.dim())(*x.shape)
        ys = (C.c_int64 * y.dim())(*y.shape)
        rc = _lib.nfx_runtime_run_sharded(self._h, comm._h, C.c_void_p(x.data_ptr()), xs, x.dim(),
                                          C.c_void_p(y.data_ptr()), ys, y.dim(), int(root),
                                          C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError("Run failed: " + self._err())

    def run_sharded_host(self, comm: "Comm", x: np.ndarray, y: np.ndarray, root: int = -1) -> None:
        """The same with host arrays (synchronous): each rank copies only its own input
        slice; y is written on every rank (root < 0) or on the root only."""
        if not (isinstance(y, np.ndarray) and y.dtype == np.float32 and y.flags.c_contiguous):
            raise RuntimeError("Run failed: y must be a C-contiguous float32 array")
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = _lib.nfx_runtime_run_sharded_host(self._h, comm._h, x.ctypes.data_as(C.c_void_p),
                                               _shape(x), x.ndim, y.ctypes.data_as(C.c_void_p),
                                               _shape(y), y.ndim, int(root))
        if rc != 0:
            raise RuntimeError("Run failed: " + self._err())


def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for Comm(); made on one rank, shared by all."""
    buf = C.create_string_buffer(128)
    rc = _lib.nfx_comm_unique_id(buf, 128)
    if rc != 0:
        raise RuntimeError("nfx_comm_unique_id failed: " + _lib.nfx_last_error().decode())
    return buf.raw


class Comm:
    """NCCL communicator of one rank (one process per GPU) for InferenceRuntime.run_sharded."""

    def __init__(self, unique_id: bytes, world: int, rank: int, device: int):
        h = C.c_void_p()
        rc = _lib.nfx_comm_create(bytes(unique_id), len(unique_id), int(world), int(rank),
                                  int(device), C.byref(h))
        if rc != 0:
            raise RuntimeError("nfx_comm_create failed: " + _lib.nfx_last_error().decode())
        self._h = h
        self.world, self.rank, self.device = int(world), int(rank), int(device)

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            _lib.nfx_comm_destroy(h)
            self._h = None

    def __del__(self):
        self.close()


class RuntimeGroup:
    """One process driving several GPUs: InferenceRuntime's calls over a device list; a
    batch runs as contiguous slices, one per device, with the weights on every device."""

    def __init__(self, ir_path: str, devices):
        devices = [int(d) for d in devices]
        arr = (C.c_int * len(devices))(*devices)
        h = C.c_void_p()
        rc = _lib.nfx_group_create(str(ir_path).encode(), arr, len(devices), C.byref(h))
        if rc != 0:
            raise RuntimeError("create runtime group failed: " + _lib.nfx_last_error().decode())
        self._h = h
        self.devices = devices

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            _lib.nfx_group_destroy(h)
            self._h = None

    def __del__(self):
        self.close()

    def _err(self) -> str:
        return _lib.nfx_group_last_error(self._h).decode()

    def enable_int8_gemm(self) -> None:
        _lib.nfx_group_enable_int8_gemm(self._h)

    def is_int8_gemm_enabled(self) -> bool:
        return bool(_lib.nfx_group_is_int8_gemm_enabled(self._h))

    def enable_fp8(self) -> None:
        _lib.nfx_group_enable_fp8(self._h)

    def run(self, x: np.ndarray, y: np.ndarray) -> None:
        """Host arrays: every device copies its own slice in and out."""
        if not (isinstance(y, np.ndarray) and y.dtype == np.float32 and y.flags.c_contiguous):
            raise RuntimeError("Run failed: y must be a C-contiguous float32 array")
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = _lib.nfx_group_run(self._h, x.ctypes.data_as(C.c_void_p), _shape(x), x.ndim,
                                y.ctypes.data_as(C.c_void_p), _shape(y), y.ndim)
        if rc != 0:
            raise RuntimeError("Run failed: " + self._err())

    def run_device(self, x, y, stream=None) -> None:
        """CUDA tensors on the first device; NCCL scatters the inputs and gathers the
        outputs.  Asynchronous on `stream` (a stream of the first device)."""
        stream = InferenceRuntime._stream(x, stream)
        xs = (C.c_int64 * x.dim())(*x.shape)
        ys = (C.c_int64 * y.dim())(*y.shape)
        rc = _lib.nfx_group_run_device(self._h, C.c_void_p(x.data_ptr()), xs, x.dim(),
                                       C.c_void_p(y.data_ptr()), ys, y.dim(), C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError("Run failed: " + self._err())

    def check(self) -> None:
        rc = _lib.nfx_group_check(self._h)
        if rc != 0:
            raise RuntimeError("device error: " + self._err())


_RANK = {"FNO1d": 3, "FNO2d": 4, "FNO3d": 5, "TokenMixer": 3, "GraphOp": 3, "TokenMixer2D": 4,
         "GraphOp2D": 4}
# the Run* call of each op (pybind_module.cpp:95-105)
_RUN = {"TokenMixer": "run_tokenmixer", "GraphOp": "run_graphop", "TokenMixer2D": "run_tokenmixer2d",
        "GraphOp2D": "run_graphop2d"}


def _run_once(model_path: str, x: np.ndarray, enable_int8: bool, enable_fp8: bool,
              device: int) -> np.ndarray:
    op, cfg, _, _ = _nfx.load_neuroir(model_path)
    if op not in _RANK or x.ndim != _RANK[op]:
        raise RuntimeError("input rank mismatch for op " + op)
    rt = InferenceRuntime(model_path, device)
    if enable_int8:
        rt.enable_int8_gemm()
    if enable_fp8:
        rt.enable_fp8()
    y = np.zeros(tuple(x.shape[:-1]) + (cfg[1],), np.float32)
    getattr(rt, _RUN.get(op, "run"))(x, y)
    return y


def infer_deeponet_arrays(model_path: str, u: np.ndarray, y: np.ndarray, device: int = 0) -> np.ndarray:
    """The reference's `infer_deeponet_arrays` (pybind_module.cpp:200-233): out (B,
    n_query, out_channels) with B and n_query from y."""
    op, cfg, _, _ = _nfx.load_neuroir(model_path)
    if op != "DeepONet":
        raise RuntimeError("infer_deeponet_arrays: model op is " + op + ", not DeepONet")
    u = np.ascontiguousarray(u, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    if u.ndim != 3:
        raise RuntimeError("DeepONet u must be 3D (batch, n_sensor, in_branch)")
    if y.ndim != 3:
        raise RuntimeError("DeepONet y must be 3D (batch, n_query, in_trunk)")
    rt = InferenceRuntime(model_path, device)
    out = np.zeros((y.shape[0], y.shape[1], cfg[3]), np.float32)
    rt.run_deeponet(u, y, out)
    return out


def infer_arrays(model_path: str, x: np.ndarray, enable_int8: bool = False,
                 enable_fp8: bool = False, device: int = 0) -> np.ndarray:
    """The reference's `infer_arrays` (pybind_module.cpp:113-158): load, run once,
    return y; the output channel count comes from the IR.  `enable_int8` / `enable_fp8`
    switch to the quantised executors (the reference function has no such switch)."""
    return _run_once(model_path, np.ascontiguousarray(x, dtype=np.float32), enable_int8,
                     enable_fp8, device)


def infer(model_path: str, input_path: str, output_path: str, enable_int8: bool = False,
          enable_fp8: bool = False, device: int = 0) -> str:
    """The reference's `infer` (pybind_module.cpp:61-111): .npy in, .npy out."""
    x = np.load(input_path)
    if x.dtype != np.float32:
        x = x.astype(np.float32)
    y = _run_once(model_path, np.ascontiguousarray(x), enable_int8, enable_fp8, device)
    np.save(output_path, y)
    return "ok"
