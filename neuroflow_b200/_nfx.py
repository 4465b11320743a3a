"""ctypes binding of libnfx.so (the C-ABI in include/nfx.h).

The product path: every call goes to the CUDA library; there is no CPU fallback.
Importing this module fails loudly when the library has not been built.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnfx.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build the CUDA library first "
        "(python -m neuroflow_b200.build, or __graft_entry__.build())")

lib = C.CDLL(LIB_PATH)

_vp = C.c_void_p
_i64p = C.POINTER(C.c_int64)

lib.nfx_last_error.restype = C.c_char_p
lib.nfx_int8_gemm.restype = C.c_int
lib.nfx_int8_gemm.argtypes = [_vp, _vp, _vp, C.c_float, C.c_int32, C.c_int, C.c_int, _vp, _vp,
                              _vp, _vp, _vp, C.c_int, C.c_int, _vp, _vp]
lib.nfx_load_neuroir.restype = C.c_int
lib.nfx_load_neuroir.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.POINTER(C.c_int32),
                                 C.POINTER(C.c_int), C.POINTER(C.c_int)]
lib.nfx_device_errors.restype = C.c_int
lib.nfx_device_errors.argtypes = [C.POINTER(C.c_uint)]

if hasattr(lib, "nfx_runtime_create"):
    lib.nfx_runtime_create.restype = C.c_int
    lib.nfx_runtime_create.argtypes = [C.c_char_p, C.c_int, C.POINTER(_vp)]
    lib.nfx_runtime_destroy.restype = None
    lib.nfx_runtime_destroy.argtypes = [_vp]
    lib.nfx_runtime_op.restype = C.c_char_p
    lib.nfx_runtime_op.argtypes = [_vp]
    lib.nfx_runtime_enable_int8_gemm.restype = None
    lib.nfx_runtime_enable_int8_gemm.argtypes = [_vp]
    lib.nfx_runtime_is_int8_gemm_enabled.restype = C.c_int
    lib.nfx_runtime_is_int8_gemm_enabled.argtypes = [_vp]
    lib.nfx_runtime_run.restype = C.c_int
    lib.nfx_runtime_run.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int]
    lib.nfx_runtime_run_device.restype = C.c_int
    lib.nfx_runtime_run_device.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int, _vp]
    lib.nfx_runtime_enable_fp8.restype = None
    lib.nfx_runtime_enable_fp8.argtypes = [_vp]
    lib.nfx_runtime_is_fp8_enabled.restype = C.c_int
    lib.nfx_runtime_is_fp8_enabled.argtypes = [_vp]
    for name in ("tokenmixer", "graphop", "graphop2d"):
        f = getattr(lib, "nfx_runtime_run_" + name)
        f.restype = C.c_int
        f.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int]
        f = getattr(lib, "nfx_runtime_run_" + name + "_device")
        f.restype = C.c_int
        f.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int, _vp]
    lib.nfx_runtime_run_deeponet.restype = C.c_int
    lib.nfx_runtime_run_deeponet.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int, _vp,
                                             _i64p, C.c_int]
    lib.nfx_runtime_run_deeponet_device.restype = C.c_int
    lib.nfx_runtime_run_deeponet_device.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int,
                                                    _vp, _i64p, C.c_int, _vp]
    lib.nfx_runtime_run_tokenmixer2d.restype = C.c_int
    lib.nfx_runtime_run_tokenmixer2d.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int]
    lib.nfx_runtime_run_tokenmixer2d_device.restype = C.c_int
    lib.nfx_runtime_run_tokenmixer2d_device.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p,
                                                        C.c_int, _vp]
    lib.nfx_runtime_set_code_taps.restype = C.c_int
    lib.nfx_runtime_set_code_taps.argtypes = [_vp, _vp, C.c_int64]
    lib.nfx_runtime_check.restype = C.c_int
    lib.nfx_runtime_check.argtypes = [_vp]
    lib.nfx_runtime_last_error.restype = C.c_char_p
    lib.nfx_runtime_last_error.argtypes = [_vp]
    lib.nfx_runtime_profile_enable.restype = C.c_int
    lib.nfx_runtime_profile_enable.argtypes = [_vp, C.c_int]
    lib.nfx_runtime_profile_count.restype = C.c_int
    lib.nfx_runtime_profile_count.argtypes = [_vp]
    lib.nfx_runtime_profile_entry.restype = C.c_int
    lib.nfx_runtime_profile_entry.argtypes = [_vp, C.c_int, C.POINTER(C.c_char_p),
                                              C.POINTER(C.c_int), C.POINTER(C.c_double)]

    lib.nfx_batch_slice.restype = None
    lib.nfx_batch_slice.argtypes = [C.c_int64, C.c_int, C.c_int, _i64p, _i64p]
    lib.nfx_group_create.restype = C.c_int
    lib.nfx_group_create.argtypes = [C.c_char_p, C.POINTER(C.c_int), C.c_int, C.POINTER(_vp)]
    lib.nfx_group_destroy.restype = None
    lib.nfx_group_destroy.argtypes = [_vp]
    lib.nfx_group_size.restype = C.c_int
    lib.nfx_group_size.argtypes = [_vp]
    lib.nfx_group_member.restype = _vp
    lib.nfx_group_member.argtypes = [_vp, C.c_int]
    lib.nfx_group_last_error.restype = C.c_char_p
    lib.nfx_group_last_error.argtypes = [_vp]
    lib.nfx_group_enable_int8_gemm.restype = None
    lib.nfx_group_enable_int8_gemm.argtypes = [_vp]
    lib.nfx_group_is_int8_gemm_enabled.restype = C.c_int
    lib.nfx_group_is_int8_gemm_enabled.argtypes = [_vp]
    lib.nfx_group_enable_fp8.restype = None
    lib.nfx_group_enable_fp8.argtypes = [_vp]
    lib.nfx_group_run.restype = C.c_int
    lib.nfx_group_run.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int]
    lib.nfx_group_run_device.restype = C.c_int
    lib.nfx_group_run_device.argtypes = [_vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int, _vp]
    lib.nfx_group_check.restype = C.c_int
    lib.nfx_group_check.argtypes = [_vp]
    lib.nfx_comm_unique_id.restype = C.c_int
    lib.nfx_comm_unique_id.argtypes = [C.c_char_p, C.c_int]
    lib.nfx_comm_create.restype = C.c_int
    lib.nfx_comm_create.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    lib.nfx_comm_destroy.restype = None
    lib.nfx_comm_destroy.argtypes = [_vp]
    lib.nfx_runtime_run_sharded.restype = C.c_int
    lib.nfx_runtime_run_sharded.argtypes = [_vp, _vp, _vp, _i64p, C.c_int, _vp, _i64p, C.c_int,
                                            C.c_int, _vp]
    lib.nfx_runtime_run_sharded_host.restype = C.c_int
    lib.nfx_runtime_run_sharded_host.argtypes = [_vp, _vp, _vp, _i64p, C.c_int, _vp, _i64p,
                                                 C.c_int, C.c_int]
    lib.nfx_calibrate_begin.restype = C.c_int
    lib.nfx_calibrate_begin.argtypes = [_vp, C.c_int]
    lib.nfx_calibrate_observe.restype = C.c_int
    lib.nfx_calibrate_observe.argtypes = [_vp, _vp, _i64p, C.c_int]
    lib.nfx_calibrate_count.restype = C.c_int
    lib.nfx_calibrate_count.argtypes = [_vp]
    lib.nfx_calibrate_result.restype = C.c_int
    lib.nfx_calibrate_result.argtypes = [_vp, C.c_int, C.c_double, C.c_char_p, C.c_int,
                                         C.POINTER(C.c_float), C.POINTER(C.c_int32),
                                         C.POINTER(C.c_float), C.POINTER(C.c_double),
                                         C.POINTER(C.c_double)]
    lib.nfx_calibrate_end.restype = C.c_int
    lib.nfx_calibrate_end.argtypes = [_vp]


def batch_slice(batch: int, world: int, rank: int):
    """(first, count): the samples rank `rank` of `world` computes (nfx_batch_slice)."""
    a, b = C.c_int64(), C.c_int64()
    lib.nfx_batch_slice(int(batch), int(world), int(rank), C.byref(a), C.byref(b))
    return a.value, b.value


class NfxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[status {code}] {msg}")
        self.code = code


def check(rc: int, handle=None) -> None:
    if rc != 0:
        if handle is not None:
            msg = lib.nfx_runtime_last_error(handle)
        else:
            msg = lib.nfx_last_error()
        raise NfxError(rc, (msg or b"").decode())


def device_errors() -> int:
    v = C.c_uint(0)
    check(lib.nfx_device_errors(C.byref(v)))
    return int(v.value)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def int8_gemm(A, W, scale_w, zp_w, sum_w, bias=None, scale_a=None, zp_a=None, scale_a_t=1.0,
              zp_a_t=0, act=0, out=None, stream=None):
    """torch-tensor front-end of nfx_int8_gemm (device tensors, current device)."""
    import torch
    M, K = A.shape
    N = W.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    s = stream if stream is not None else torch.cuda.current_stream(A.device).cuda_stream
    check(lib.nfx_int8_gemm(_ptr(A), _ptr(scale_a), _ptr(zp_a), float(scale_a_t), int(zp_a_t),
                            M, K, _ptr(W), _ptr(scale_w), _ptr(zp_w), _ptr(sum_w), _ptr(bias), N,
                            int(act), _ptr(out), C.c_void_p(s)))
    return out


def load_neuroir(path: str):
    """LoadNeuroIr on the host: (op, config ints, n_weights, quant_enabled); raises
    NfxError with the reference StatusCode on failure."""
    op = C.create_string_buffer(32)
    cfg = (C.c_int32 * 8)()
    nw = C.c_int()
    q = C.c_int()
    check(lib.nfx_load_neuroir(str(path).encode(), op, 32, cfg, C.byref(nw), C.byref(q)))
    return op.value.decode(), list(cfg), nw.value, bool(q.value)
