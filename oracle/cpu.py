"""ctypes front-end for the CPU parity checkers.

TEST INFRASTRUCTURE ONLY.  `Oracle` wraps oracle/liboracle.so (the C restatement in
nfo_oracle.c); `Reference` wraps oracle/_ref/libnflow_ref.so (the reference sources
compiled by oracle/Makefile).  Only tests/, __graft_entry__.smoke() and bench.py's
CPU legs use this module, as the checker or the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libnflow_ref.so")
MAX_LAYERS = 8

_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_i8p = C.POINTER(C.c_int8)
_i64p = C.POINTER(C.c_int64)


def _p(a, t=_f32p):
    return None if a is None else a.ctypes.data_as(t)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


class _WQ(C.Structure):
    _fields_ = [("pc_scales", _f32p), ("pc_zps", _i32p), ("pc_n", C.c_int64),
                ("pc_axis", C.c_int32), ("has_pc", C.c_int32), ("pt_scale", C.c_float),
                ("pt_zp", C.c_int32), ("has_pt", C.c_int32)]


class _AQ(C.Structure):
    _fields_ = [("scale", C.c_float), ("zp", C.c_int32), ("has", C.c_int32),
                ("fp8_scale", C.c_float), ("has_fp8", C.c_int32)]


class _FNO2d(C.Structure):
    _fields_ = ([(n, C.c_int32) for n in ("in_ch", "out_ch", "width", "modes_h", "modes_w",
                                          "n_layers", "pad_factor", "relu", "quant_enabled")]
                + [(n, _f32p) for n in ("lift_w", "lift_b", "proj_q_w", "proj_q_b",
                                        "proj_out_w", "proj_out_b")]
                + [(n, _f32p * MAX_LAYERS) for n in ("spec_wr", "spec_wi", "loc_w", "loc_b")]
                + [(n, _WQ) for n in ("q_lift_w", "q_lift_b", "q_proj_q_w", "q_proj_q_b",
                                      "q_proj_out_w", "q_proj_out_b")]
                + [(n, _WQ * MAX_LAYERS) for n in ("q_spec_wr", "q_spec_wi", "q_loc_w",
                                                   "q_loc_b")]
                + [(n, _AQ) for n in ("a_lift", "a_proj_q", "a_proj_out")]
                + [("a_locs", _AQ * MAX_LAYERS)])


class _AQ1(C.Structure):
    _fields_ = [("scale", C.c_float), ("zp", C.c_int32), ("has", C.c_int32),
                ("fp8_scale", C.c_float), ("has_fp8", C.c_int32), ("pt_scales", _f32p),
                ("pt_zps", _i32p), ("pt_n", C.c_int64), ("pt_width", C.c_int32),
                ("has_pt", C.c_int32)]


class _FNO1d(C.Structure):
    _fields_ = ([(n, C.c_int32) for n in ("in_ch", "out_ch", "width", "modes", "n_layers",
                                          "pad_factor", "relu", "quant_enabled", "int8_enabled")]
                + [(n, _f32p) for n in ("lift_w", "lift_b", "proj_q_w", "proj_q_b",
                                        "proj_out_w", "proj_out_b")]
                + [(n, _f32p * MAX_LAYERS) for n in ("spec_wr", "spec_wi", "loc_w", "loc_b")]
                + [(n, _WQ) for n in ("q_lift_w", "q_lift_b", "q_proj_q_w", "q_proj_q_b",
                                      "q_proj_out_w", "q_proj_out_b")]
                + [(n, _WQ * MAX_LAYERS) for n in ("q_spec_wr", "q_spec_wi", "q_loc_w",
                                                   "q_loc_b")]
                + [("a_lift", _AQ1), ("a_locs", _AQ1 * MAX_LAYERS)])


class _TM2D(C.Structure):
    _fields_ = ([(n, C.c_int32) for n in ("in_dim", "out_dim", "latent", "h", "w", "n_patches",
                                          "n_heads", "n_layers", "relu")]
                + [(n, _f32p) for n in ("se_w", "se_b", "un_w", "un_b", "head_w", "head_b")]
                + [("blk_w", (_f32p * 8) * MAX_LAYERS), ("blk_b", (_f32p * 8) * MAX_LAYERS),
                   ("pc_s", (_f32p * 8) * MAX_LAYERS), ("pc_zp", (_i32p * 8) * MAX_LAYERS)])


class _FNO3d(C.Structure):
    _fields_ = ([(n, C.c_int32) for n in ("in_ch", "out_ch", "width", "modes_h", "modes_w",
                                          "modes_d", "n_layers", "pad_factor", "relu")]
                + [(n, _f32p) for n in ("lift_w", "lift_b", "proj_q_w", "proj_q_b",
                                        "proj_out_w", "proj_out_b")]
                + [(n, _f32p * MAX_LAYERS) for n in ("spec_wr", "spec_wi", "loc_w", "loc_b")]
                + [(n, C.c_float) for n in ("s_lift_w", "s_proj_q_w", "s_proj_out_w")]
                + [("s_loc_w", C.c_float * MAX_LAYERS)]
                + [(n, C.c_float) for n in ("s_lift", "s_proj_q", "s_proj_out")]
                + [("s_locs", C.c_float * MAX_LAYERS)])


MAX_MLP = 8


class _DeepONet(C.Structure):
    _fields_ = ([(n, C.c_int32) for n in ("in_branch", "in_trunk", "latent", "out_ch", "n_branch",
                                          "n_trunk", "hidden_branch", "hidden_trunk", "relu")]
                + [("bw", _f32p * MAX_MLP), ("bb", _f32p * MAX_MLP), ("tw", _f32p * MAX_MLP),
                   ("tb", _f32p * MAX_MLP), ("bias", _f32p)])


class _GraphOp(C.Structure):
    _fields_ = ([(n, C.c_int32) for n in ("in_dim", "out_dim", "n_nodes", "hidden", "n_layers",
                                          "relu")]
                + [("lift_w", _f32p), ("lift_b", _f32p), ("self_w", _f32p * MAX_LAYERS),
                   ("self_b", _f32p * MAX_LAYERS), ("neigh_w", _f32p * MAX_LAYERS),
                   ("neigh_b", _f32p * MAX_LAYERS), ("head_w", _f32p), ("head_b", _f32p),
                   ("adj_off", _i32p), ("adj_idx", _i32p), ("deg_inv", _f32p)])


class _Taps(C.Structure):
    _fields_ = [("codes_in", _i8p * (MAX_LAYERS + 1)), ("x1_out", _f32p * MAX_LAYERS),
                ("h_out", _f32p * MAX_LAYERS), ("lift_out", _f32p), ("x2_out", _f32p * MAX_LAYERS),
                ("q_out", _f32p)]


class Oracle:
    """The C restatement (nfo_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        self.lib = C.CDLL(path)
        L = self.lib
        L.nfo_fno2d_forward.restype = C.c_int
        L.nfo_fno2d_forward.argtypes = [C.POINTER(_FNO2d), C.c_int, _f32p, C.c_int, C.c_int,
                                        C.c_int, _f32p, C.POINTER(_Taps)]
        L.nfo_fno3d_forward_taps.restype = C.c_int
        L.nfo_fno3d_forward_taps.argtypes = [C.POINTER(_FNO3d), C.c_int, _f32p, C.c_int, C.c_int,
                                             C.c_int, C.c_int, _f32p, _f32p]
        L.nfo_fno3d_forward.restype = C.c_int
        L.nfo_fno3d_forward.argtypes = [C.POINTER(_FNO3d), C.c_int, _f32p, C.c_int, C.c_int,
                                        C.c_int, C.c_int, _f32p]
        L.nfo_fp32_to_e4m3.restype = C.c_uint8
        L.nfo_fp32_to_e4m3.argtypes = [C.c_float]
        L.nfo_e4m3_to_fp32.restype = C.c_float
        L.nfo_e4m3_to_fp32.argtypes = [C.c_uint8]
        L.nfo_tm2d_forward.restype = C.c_int
        L.nfo_tm2d_forward.argtypes = [C.POINTER(_TM2D), C.c_int, _f32p, C.c_int, _f32p]
        L.nfo_fno1d_forward.restype = C.c_int
        L.nfo_fno1d_forward.argtypes = [C.POINTER(_FNO1d), _f32p, C.c_int, C.c_int, _f32p]

    # -- primitives ---------------------------------------------------------
    def quantise_activation(self, A, scale, zp):
        A = _c(A, np.float32)
        out = np.empty(A.shape, np.int8)
        self.lib.nfo_quantise_activation(_p(A), _p(out, _i8p), C.c_int64(A.size),
                                         C.c_float(scale), C.c_int32(zp))
        return out

    def fake_quant(self, x, scale, zp):
        x = _c(x, np.float32).copy()
        self.lib.nfo_fake_quant(_p(x), C.c_int64(x.size), C.c_float(scale), C.c_int32(zp))
        return x

    def quantise_weight_2d(self, W, scales, zps):
        W = _c(W, np.float32)
        n, k = W.shape
        q = np.empty((n, k), np.int8)
        s = np.empty(n, np.int32)
        self.lib.nfo_quantise_weight_2d(_p(W), n, k, _p(_c(scales, np.float32)),
                                        _p(_c(zps, np.int32), _i32p), _p(q, _i8p), _p(s, _i32p))
        return q, s

    def linear_forward_batched(self, Wq, sW, zpW, sumW, bias, sA, zpA, A):
        A = _c(A, np.float32)
        M, K = A.shape
        N = Wq.shape[0]
        out = np.empty((M, N), np.float32)
        acc = np.empty((M, N), np.int32)
        codes = np.empty((M, K), np.int8)
        bias_c = None if bias is None else _c(bias, np.float32)
        self.lib.nfo_linear_forward_batched(
            _p(_c(Wq, np.int8), _i8p), _p(_c(sW, np.float32)), _p(_c(zpW, np.int32), _i32p),
            _p(_c(sumW, np.int32), _i32p), _p(bias_c), K, N, C.c_float(sA), C.c_int32(zpA),
            M, _p(A), _p(out), _p(acc, _i32p), _p(codes, _i8p))
        return out, acc, codes

    def int8_gemm_rows(self, Aq, sA, zpA, Wq, sW, zpW, sumW, bias, gelu):
        Aq = _c(Aq, np.int8)
        M, K = Aq.shape
        N = Wq.shape[0]
        out = np.empty((M, N), np.float32)
        acc = np.empty((M, N), np.int32)
        bias_c = None if bias is None else _c(bias, np.float32)
        self.lib.nfo_int8_gemm_rows(
            _p(Aq, _i8p), _p(_c(sA, np.float32)), _p(_c(zpA, np.int32), _i32p), M, K,
            _p(_c(Wq, np.int8), _i8p), _p(_c(sW, np.float32)), _p(_c(zpW, np.int32), _i32p),
            _p(_c(sumW, np.int32), _i32p), N, _p(bias_c), int(bool(gelu)), _p(out),
            _p(acc, _i32p))
        return out, acc

    def linear(self, x, W, b):
        x = _c(x, np.float32)
        M, K = x.shape
        N = W.shape[0]
        y = np.empty((M, N), np.float32)
        self.lib.nfo_linear(_p(x), _p(_c(W, np.float32)),
                            None if b is None else _p(_c(b, np.float32)), M, K, N, _p(y))
        return y

    def activation(self, x, relu=False):
        x = _c(x, np.float32).copy()
        self.lib.nfo_apply_activation(_p(x), C.c_int64(x.size), int(relu))
        return x

    def rfft2(self, x):
        x = _c(x, np.float32)
        H, W = x.shape
        out = np.empty((H, W // 2 + 1, 2), np.float32)
        self.lib.nfo_rfft2(_p(x), H, W, _p(out))
        return out

    def irfft2(self, xc, H, W):
        xc = _c(xc, np.float32)
        out = np.empty((H, W), np.float32)
        self.lib.nfo_irfft2(_p(xc), H, W, _p(out))
        return out

    def rfft(self, x):
        x = _c(x, np.float32)
        out = np.empty((x.size // 2 + 1, 2), np.float32)
        self.lib.nfo_rfft(_p(x), x.size, _p(out))
        return out

    def irfft(self, xc, n):
        out = np.empty(n, np.float32)
        self.lib.nfo_irfft(_p(_c(xc, np.float32)), n, _p(out))
        return out

    def spectral_conv2d(self, h, wr, wi):
        h = _c(h, np.float32)
        b, w, H, W = h.shape
        mh, mw = wr.shape[2], wr.shape[3]
        out = np.empty_like(h)
        self.lib.nfo_spectral_conv2d(_p(h), b, w, H, W, mh, mw, _p(_c(wr, np.float32)),
                                     _p(_c(wi, np.float32)), _p(out))
        return out

    # -- FNO2d -----------------------------------------------------------------
    def fno2d_forward(self, model, x, mode: int, taps: bool = False):
        """mode 0: reference fake-quant FNO2d; mode 1: INT8 composition.
        Returns y, or (y, taps_dict) when taps=True."""
        x = _c(x, np.float32)
        B, H, W, _ = x.shape
        st, keep = build_fno2d_struct(model)
        cfg = model.config
        y = np.empty((B, H, W, cfg["out_channels"]), np.float32)
        tp = None
        tap_arrays = {}
        if taps:
            tp = _Taps()
            L, w = cfg["n_layers"], cfg["width"]
            for i in range(L + 1):
                a = np.zeros((B, H, W, w), np.int8)
                tap_arrays[f"codes_in.{i}"] = a
                tp.codes_in[i] = _p(a, _i8p)
            pf = cfg.get("pad_factor", 0)
            Hp = H + ((pf - H % pf) % pf if pf > 1 else 0)
            Wp = W + ((pf - W % pf) % pf if pf > 1 else 0)
            for i in range(L):
                a = np.zeros((B, w, Hp, Wp), np.float32)
                tap_arrays[f"x1.{i}"] = a
                tp.x1_out[i] = _p(a)
                a = np.zeros((B, Hp, Wp, w), np.float32)
                tap_arrays[f"h.{i}"] = a
                tp.h_out[i] = _p(a)
                a = np.zeros((B, Hp, Wp, w), np.float32)
                tap_arrays[f"x2.{i}"] = a
                tp.x2_out[i] = _p(a)
            for key in ("lift_out", "q_out"):
                a = np.zeros((B, H, W, w), np.float32)
                tap_arrays[key] = a
                setattr(tp, key, _p(a))
        rc = self.lib.nfo_fno2d_forward(C.byref(st), int(mode), _p(x), B, H, W, _p(y),
                                        C.byref(tp) if tp is not None else None)
        if rc != 0:
            raise RuntimeError(f"nfo_fno2d_forward failed: {rc}")
        del keep
        return (y, tap_arrays) if taps else y


    # -- FNO1d -----------------------------------------------------------------
    def fno1d_forward(self, model, x, int8: bool = False):
        """The reference FNO1d::Forward after Create (and EnableInt8Gemm if `int8`)."""
        x = _c(x, np.float32)
        B, n, _ = x.shape
        st, keep = build_fno1d_struct(model, int8)
        y = np.empty((B, n, model.config["out_channels"]), np.float32)
        rc = self.lib.nfo_fno1d_forward(C.byref(st), _p(x), B, n, _p(y))
        if rc != 0:
            raise RuntimeError(f"nfo_fno1d_forward failed: {rc}")
        del keep
        return y


    # -- TokenMixer2D ---------------------------------------------------------------
    def tm2d_forward(self, model, x, int8: bool = False):
        """mode 0 (int8=False): the reference TokenMixer2D::Forward; int8=True: the INT8
        variant (per-token activations, per-channel weight codes on q/k/v/o/ffn)."""
        x = _c(x, np.float32)
        st, keep = build_tm2d_struct(model)
        cfg = model.config
        y = np.empty(x.shape[:-1] + (cfg["out_dim"],), np.float32)
        rc = self.lib.nfo_tm2d_forward(C.byref(st), 1 if int8 else 0, _p(x), x.shape[0], _p(y))
        if rc != 0:
            raise RuntimeError(f"nfo_tm2d_forward failed: {rc}")
        del keep
        return y


    def tokenmixer_forward(self, model, x, int8: bool = False):
        """The reference TokenMixer::Forward (fno.cpp:1460-1644): the TokenMixer2D
        network on a (1, n_points) grid (the same loops, with x (b, n_points, in_dim))."""
        cfg = model.config
        m2 = type(model)(op="TokenMixer2D", config=dict(
            in_dim=cfg["in_dim"], out_dim=cfg["out_dim"], latent_dim=cfg["latent_dim"], h=1,
            w=cfg["n_points"], n_patches=cfg["n_patches"], n_heads=cfg["n_heads"],
            n_layers=cfg["n_layers"]), activation=model.activation, weights=model.weights,
            qparams=model.qparams, quant_enabled=model.quant_enabled)
        x = _c(x, np.float32)
        return self.tm2d_forward(m2, x[:, None], int8=int8)[:, 0]

    def deeponet_forward(self, model, u, y):
        """DeepONet::Forward (fno.cpp:1289-1406): u (b, n_sensor, in_branch), y (b, n_query,
        in_trunk) -> (b, n_query, out_channels)."""
        u, y = _c(u, np.float32), _c(y, np.float32)
        st, keep = build_deeponet_struct(model)
        out = np.empty((y.shape[0], y.shape[1], model.config["out_channels"]), np.float32)
        rc = self.lib.nfo_deeponet_forward(C.byref(st), _p(u), u.shape[0], u.shape[1], _p(y),
                                           y.shape[1], _p(out))
        if rc != 0:
            raise RuntimeError(f"nfo_deeponet_forward failed: {rc}")
        del keep
        return out

    def graphop_forward(self, model, x):
        """GraphOp::Forward / GraphOp2D::Forward (fno.cpp:1653-1741, :1969-2060): x (b,
        n_nodes, in_dim) or (b, h, w, in_dim) -> the same with out_dim."""
        x = _c(x, np.float32)
        st, keep = build_graphop_struct(model)
        y = np.empty(x.shape[:-1] + (model.config["out_dim"],), np.float32)
        rc = self.lib.nfo_graphop_forward(C.byref(st), _p(x), x.shape[0], _p(y))
        if rc != 0:
            raise RuntimeError(f"nfo_graphop_forward failed: {rc}")
        del keep
        return y

    # -- FP8 E4M3 / FNO3d ------------------------------------------------------------
    def fp32_to_e4m3(self, x):
        x = _c(x, np.float32).ravel()
        out = np.empty(x.size, np.uint8)
        self.lib.nfo_fp32_to_e4m3_array(_p(x), out.ctypes.data_as(C.c_void_p), C.c_int64(x.size))
        return out

    def fno3d_forward(self, model, x, fp8: bool = False, taps: bool = False):
        """mode 0 (fp8=False): the reference FNO3d::Forward; fp8=True: the E4M3 variant.
        With taps (fp8 only), returns (y, t): t[i] the E4M3 values of layer i's input
        (the lift's output, then each layer's output), channel-first on the padded grid
        (L + 1, B, C, Hp, Wp, Dp)."""
        x = _c(x, np.float32)
        st, keep = build_fno3d_struct(model)
        y = np.empty(x.shape[:-1] + (model.config["out_channels"],), np.float32)
        B, H, W, D, _ = x.shape
        if not taps:
            rc = self.lib.nfo_fno3d_forward(C.byref(st), 1 if fp8 else 0, _p(x), B, H, W, D, _p(y))
            if rc != 0:
                raise RuntimeError(f"nfo_fno3d_forward failed: {rc}")
            del keep
            return y
        if not fp8:
            raise ValueError("FNO3d taps exist for the FP8 variant only")
        pf = int(model.config.get("pad_factor", 0))
        pd = [d + ((pf - d % pf) % pf if pf > 1 else 0) for d in (H, W, D)]
        t = np.empty((model.config["n_layers"] + 1, B, model.config["width"]) + tuple(pd), np.float32)
        rc = self.lib.nfo_fno3d_forward_taps(C.byref(st), 1, _p(x), B, H, W, D, _p(y), _p(t))
        if rc != 0:
            raise RuntimeError(f"nfo_fno3d_forward_taps failed: {rc}")
        del keep
        return y, t


def build_fno3d_struct(model):
    from neuroflow_b200 import ir
    cfg, w = model.config, model.weights
    keep = []
    st = _FNO3d()
    for f, k in (("in_ch", "in_channels"), ("out_ch", "out_channels"), ("width", "width"),
                 ("modes_h", "modes_h"), ("modes_w", "modes_w"), ("modes_d", "modes_d"),
                 ("n_layers", "n_layers"), ("pad_factor", "pad_factor")):
        setattr(st, f, cfg[k])
    st.relu = 1 if model.activation == "relu" else 0

    def arr(name):
        a = _c(w[name], np.float32)
        keep.append(a)
        return _p(a)

    def fs(name):
        qp = model.qparams.get(name)
        return float(qp.scale) if isinstance(qp, ir.FP8) else 1.0

    for fld, nm in (("lift_w", "lift.weight"), ("lift_b", "lift.bias"),
                    ("proj_q_w", "proj_q.weight"), ("proj_q_b", "proj_q.bias"),
                    ("proj_out_w", "proj_out.weight"), ("proj_out_b", "proj_out.bias")):
        setattr(st, fld, arr(nm))
    st.s_lift_w, st.s_proj_q_w, st.s_proj_out_w = fs("lift.weight"), fs("proj_q.weight"), fs("proj_out.weight")
    st.s_lift, st.s_proj_q, st.s_proj_out = fs("lift.output"), fs("proj_q.output"), fs("proj_out.output")
    for i in range(cfg["n_layers"]):
        for fld, nm in (("spec_wr", f"specs.{i}.weights_real"), ("spec_wi", f"specs.{i}.weights_imag"),
                        ("loc_w", f"locs.{i}.weight"), ("loc_b", f"locs.{i}.bias")):
            getattr(st, fld)[i] = arr(nm)
        st.s_loc_w[i] = fs(f"locs.{i}.weight")
        st.s_locs[i] = fs(f"locs.{i}.output")
    return st, keep


def build_deeponet_struct(model):
    cfg, w = model.config, model.weights
    keep = []
    st = _DeepONet()
    nb, nt = cfg["n_layers_branch"], cfg["n_layers_trunk"]
    st.in_branch, st.in_trunk = cfg["in_branch"], cfg["in_trunk"]
    st.latent, st.out_ch, st.n_branch, st.n_trunk = cfg["latent_dim"], cfg["out_channels"], nb, nt
    st.hidden_branch = w[f"branch.layers.{nb - 2}.weight"].shape[0] if nb >= 2 else 0
    st.hidden_trunk = w[f"trunk.layers.{nt - 2}.weight"].shape[0] if nt >= 2 else 0
    st.relu = 1 if model.activation == "relu" else 0

    def arr(a):
        a = _c(a, np.float32)
        keep.append(a)
        return _p(a)

    for i in range(nb):
        st.bw[i], st.bb[i] = arr(w[f"branch.layers.{i}.weight"]), arr(w[f"branch.layers.{i}.bias"])
    for i in range(nt):
        st.tw[i], st.tb[i] = arr(w[f"trunk.layers.{i}.weight"]), arr(w[f"trunk.layers.{i}.bias"])
    st.bias = arr(w["bias.weight"])
    return st, keep


def build_graphop_struct(model):
    cfg, w = model.config, model.weights
    keep = []
    st = _GraphOp()
    st.in_dim, st.out_dim = cfg["in_dim"], cfg["out_dim"]
    st.n_nodes = cfg["h"] * cfg["w"] if model.op == "GraphOp2D" else cfg["n_nodes"]
    st.hidden, st.n_layers = cfg["hidden_dim"], cfg["n_layers"]
    st.relu = 1 if model.activation == "relu" else 0

    def arr(a, dt=np.float32, t=_f32p):
        a = _c(a, dt)
        keep.append(a)
        return _p(a, t)

    st.lift_w, st.lift_b = arr(w["lift.weight"]), arr(w["lift.bias"])
    for i in range(cfg["n_layers"]):
        p = f"blocks.{i}."
        st.self_w[i], st.self_b[i] = arr(w[p + "lin_self.weight"]), arr(w[p + "lin_self.bias"])
        st.neigh_w[i], st.neigh_b[i] = arr(w[p + "lin_neigh.weight"]), arr(w[p + "lin_neigh.bias"])
    st.head_w, st.head_b = arr(w["head.weight"]), arr(w["head.bias"])
    # the loader's float -> int32 conversion of the CSR arrays (ir_loader.h:421-429)
    st.adj_off = arr(w["graph.adj_offsets"].astype(np.int32), np.int32, _i32p)
    st.adj_idx = arr(w["graph.adj_indices"].astype(np.int32), np.int32, _i32p)
    st.deg_inv = arr(w["graph.deg_inv"])
    return st, keep


def build_tm2d_struct(model):
    from neuroflow_b200.synth import TM2D_PARTS
    cfg, w = model.config, model.weights
    keep = []
    st = _TM2D()
    for f, k in (("in_dim", "in_dim"), ("out_dim", "out_dim"), ("latent", "latent_dim"), ("h", "h"),
                 ("w", "w"), ("n_patches", "n_patches"), ("n_heads", "n_heads"),
                 ("n_layers", "n_layers")):
        setattr(st, f, cfg[k])
    st.relu = 1 if model.activation == "relu" else 0

    def arr(a, dt=np.float32, t=_f32p):
        a = _c(a, dt)
        keep.append(a)
        return _p(a, t)

    st.se_w, st.se_b = arr(w["slice_embed.proj.weight"]), arr(w["slice_embed.proj.bias"])
    st.un_w, st.un_b = arr(w["unslice.proj.weight"]), arr(w["unslice.proj.bias"])
    st.head_w, st.head_b = arr(w["head.weight"]), arr(w["head.bias"])
    for i in range(cfg["n_layers"]):
        for j, part in enumerate(TM2D_PARTS):
            st.blk_w[i][j] = arr(w[f"blocks.{i}.{part}.weight"])
            st.blk_b[i][j] = arr(w[f"blocks.{i}.{part}.bias"])
            qp = model.qparams.get(f"blocks.{i}.{part}.weight")
            if qp is not None and hasattr(qp, "scales"):
                st.pc_s[i][j] = arr(qp.scales)
                st.pc_zp[i][j] = arr(qp.zero_points, np.int32, _i32p)
    return st, keep


def _aq1(model, key, keep):
    from neuroflow_b200 import ir
    a = _AQ1()
    qp = model.qparams.get(key) if model.quant_enabled else None
    if isinstance(qp, ir.PerTensor):
        a.scale, a.zp, a.has = float(qp.scale), int(qp.zero_point), 1
    elif isinstance(qp, ir.FP8):
        a.fp8_scale, a.has_fp8 = float(qp.scale), 1
    elif isinstance(qp, ir.PerToken):
        sc = _c(qp.scales, np.float32)
        zp = _c(qp.zero_points, np.int32)
        keep += [sc, zp]
        a.pt_scales, a.pt_zps, a.pt_n = _p(sc), _p(zp, _i32p), sc.size
        a.pt_width, a.has_pt = int(qp.width), 1
    return a


def build_fno1d_struct(model, int8: bool):
    cfg, w = model.config, model.weights
    keep = []
    st = _FNO1d()
    st.in_ch, st.out_ch, st.width = cfg["in_channels"], cfg["out_channels"], cfg["width"]
    st.modes, st.n_layers, st.pad_factor = cfg["modes"], cfg["n_layers"], cfg.get("pad_factor", 0)
    st.relu = 1 if model.activation == "relu" else 0
    st.quant_enabled = 1 if model.quant_enabled else 0
    st.int8_enabled = 1 if int8 else 0

    def arr(name):
        a = _c(w[name], np.float32)
        keep.append(a)
        return _p(a)

    for fld, nm in (("lift_w", "lift.weight"), ("lift_b", "lift.bias"),
                    ("proj_q_w", "proj_q.weight"), ("proj_q_b", "proj_q.bias"),
                    ("proj_out_w", "proj_out.weight"), ("proj_out_b", "proj_out.bias")):
        setattr(st, fld, arr(nm))
        setattr(st, "q_" + fld, _wq(model.qparams.get(nm), keep))
    for i in range(cfg["n_layers"]):
        for fld, nm in (("spec_wr", f"specs.{i}.weights_real"), ("spec_wi", f"specs.{i}.weights_imag"),
                        ("loc_w", f"locs.{i}.weight"), ("loc_b", f"locs.{i}.bias")):
            getattr(st, fld)[i] = arr(nm)
            getattr(st, "q_" + fld)[i] = _wq(model.qparams.get(nm), keep)
        st.a_locs[i] = _aq1(model, f"locs.{i}.output", keep)
    st.a_lift = _aq1(model, "lift.output", keep)
    return st, keep


def _wq(qp, keep):
    from neuroflow_b200 import ir
    s = _WQ()
    if isinstance(qp, ir.PerChannel):
        sc = _c(qp.scales, np.float32)
        zp = _c(qp.zero_points, np.int32)
        keep += [sc, zp]
        s.pc_scales, s.pc_zps, s.pc_n = _p(sc), _p(zp, _i32p), sc.size
        s.pc_axis, s.has_pc = int(qp.channel_axis), 1
    elif isinstance(qp, ir.PerTensor):
        s.pt_scale, s.pt_zp, s.has_pt = float(qp.scale), int(qp.zero_point), 1
    return s


def _aq(model, key):
    from neuroflow_b200 import ir
    a = _AQ()
    qp = model.qparams.get(key)
    if isinstance(qp, ir.PerTensor):
        a.scale, a.zp, a.has = float(qp.scale), int(qp.zero_point), 1
    elif isinstance(qp, ir.FP8):
        a.fp8_scale, a.has_fp8 = float(qp.scale), 1
    return a


def build_fno2d_struct(model):
    """Fill the C model struct from an ir.Model (FNO2d)."""
    cfg, w = model.config, model.weights
    keep = []
    st = _FNO2d()
    st.in_ch, st.out_ch, st.width = cfg["in_channels"], cfg["out_channels"], cfg["width"]
    st.modes_h, st.modes_w, st.n_layers = cfg["modes_h"], cfg["modes_w"], cfg["n_layers"]
    st.pad_factor = cfg.get("pad_factor", 1)
    st.relu = 1 if model.activation == "relu" else 0
    st.quant_enabled = 1 if model.quant_enabled else 0

    def arr(name):
        a = _c(w[name], np.float32)
        keep.append(a)
        return _p(a)

    for fld, nm in (("lift_w", "lift.weight"), ("lift_b", "lift.bias"),
                    ("proj_q_w", "proj_q.weight"), ("proj_q_b", "proj_q.bias"),
                    ("proj_out_w", "proj_out.weight"), ("proj_out_b", "proj_out.bias")):
        setattr(st, fld, arr(nm))
        setattr(st, "q_" + fld, _wq(model.qparams.get(nm), keep))
    for i in range(cfg["n_layers"]):
        for fld, nm in (("spec_wr", f"specs.{i}.weights_real"), ("spec_wi", f"specs.{i}.weights_imag"),
                        ("loc_w", f"locs.{i}.weight"), ("loc_b", f"locs.{i}.bias")):
            getattr(st, fld)[i] = arr(nm)
            getattr(st, "q_" + fld)[i] = _wq(model.qparams.get(nm), keep)
        st.a_locs[i] = _aq(model, f"locs.{i}.output")
    st.a_lift = _aq(model, "lift.output")
    st.a_proj_q = _aq(model, "proj_q.output")
    st.a_proj_out = _aq(model, "proj_out.output")
    return st, keep


class Reference:
    """The reference runtime compiled from its sources (oracle/_ref)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        self.lib = C.CDLL(path)
        self.lib.ref_last_error.restype = C.c_char_p
        self.lib.ref_bench_run.restype = C.c_double

    def run(self, path, x, out_ch, enable_int8=False, tokenmixer2d=False):
        x = _c(x, np.float32)
        h = C.c_void_p()
        rc = self.lib.ref_runtime_create(path.encode(), C.byref(h))
        if rc != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        try:
            if enable_int8:
                self.lib.ref_runtime_enable_int8(h)
            ys = list(x.shape[:-1]) + [out_ch]
            y = np.zeros(ys, np.float32)
            xs = (C.c_int64 * x.ndim)(*x.shape)
            yv = (C.c_int64 * y.ndim)(*y.shape)
            fn = self.lib.ref_runtime_run_tokenmixer2d if tokenmixer2d else self.lib.ref_runtime_run
            rc = fn(h, _p(x), xs, x.ndim, _p(y), yv, y.ndim)
            if rc != 0:
                raise RuntimeError(self.lib.ref_last_error().decode())
            return y
        finally:
            self.lib.ref_runtime_destroy(h)

    def run_deeponet(self, path, u, y, out_ch):
        """InferenceRuntime::RunDeepONet (runtime.cpp:103-113)."""
        u, y = _c(u, np.float32), _c(y, np.float32)
        h = C.c_void_p()
        if self.lib.ref_runtime_create(path.encode(), C.byref(h)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        try:
            out = np.zeros((y.shape[0], y.shape[1], out_ch), np.float32)
            shp = lambda a: (C.c_int64 * a.ndim)(*a.shape)
            rc = self.lib.ref_runtime_run_deeponet(h, _p(u), shp(u), u.ndim, _p(y), shp(y), y.ndim,
                                                   _p(out), shp(out), out.ndim)
            if rc != 0:
                raise RuntimeError(self.lib.ref_last_error().decode())
            return out
        finally:
            self.lib.ref_runtime_destroy(h)

    def run_other(self, path, op, x, out_ch):
        """RunTokenMixer / RunGraphOp / RunGraphOp2D (runtime.cpp:115-153) by op name."""
        kind = {"TokenMixer": 0, "GraphOp": 1, "GraphOp2D": 2}[op]
        x = _c(x, np.float32)
        h = C.c_void_p()
        if self.lib.ref_runtime_create(path.encode(), C.byref(h)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        try:
            y = np.zeros(x.shape[:-1] + (out_ch,), np.float32)
            xs = (C.c_int64 * x.ndim)(*x.shape)
            ys = (C.c_int64 * y.ndim)(*y.shape)
            rc = self.lib.ref_runtime_run_other(h, kind, _p(x), xs, x.ndim, _p(y), ys, y.ndim)
            if rc != 0:
                raise RuntimeError(self.lib.ref_last_error().decode())
            return y
        finally:
            self.lib.ref_runtime_destroy(h)

    def bench(self, path, x, out_ch, nthreads, reps=1, enable_int8=False, tokenmixer2d=False):
        """Wall seconds for `reps` passes over x split across `nthreads` runtimes."""
        x = _c(x, np.float32)
        xs = (C.c_int64 * x.ndim)(*x.shape)
        ys = (C.c_int64 * x.ndim)(*(list(x.shape[:-1]) + [out_ch]))
        t = self.lib.ref_bench_run(path.encode(), int(tokenmixer2d), int(enable_int8), _p(x),
                                   xs, x.ndim, ys, int(nthreads), int(reps))
        if t < 0:
            raise RuntimeError(f"ref_bench_run failed ({t})")
        return t

    def linear(self, x, W, b):
        x = _c(x, np.float32)
        M, K = x.shape
        N = W.shape[0]
        y = np.empty((M, N), np.float32)
        self.lib.ref_linear(_p(x), _p(_c(W, np.float32)),
                            None if b is None else _p(_c(b, np.float32)), M, K, N, _p(y))
        return y

    def activation(self, x, relu=False):
        x = _c(x, np.float32).copy()
        self.lib.ref_apply_activation(_p(x), C.c_int64(x.size), int(relu))
        return x

    def rfft2(self, x):
        x = _c(x, np.float32)
        H, W = x.shape
        out = np.empty((H, W // 2 + 1, 2), np.float32)
        self.lib.ref_rfft2(_p(x), H, W, _p(out))
        return out

    def irfft2(self, xc, H, W):
        out = np.empty((H, W), np.float32)
        self.lib.ref_irfft2(_p(_c(xc, np.float32)), H, W, _p(out))
        return out

    def spectral_conv2d(self, h, wr, wi):
        h = _c(h, np.float32)
        b, w, H, W = h.shape
        out = np.empty_like(h)
        self.lib.ref_spectral_conv2d(_p(h), b, w, H, W, wr.shape[2], wr.shape[3],
                                     _p(_c(wr, np.float32)), _p(_c(wi, np.float32)), _p(out))
        return out

    def quantise_activation(self, A, scale, zp):
        A = _c(A, np.float32)
        M, K = A.reshape(-1, A.shape[-1]).shape
        out = np.empty(A.shape, np.int8)
        self.lib.ref_quantise_activation(_p(A), _p(out, _i8p), M, K, C.c_float(scale),
                                         C.c_int32(zp))
        return out

    def linear_forward_batched(self, Wq, sW, zpW, sumW, bias, sA, zpA, A):
        A = _c(A, np.float32)
        M, K = A.shape
        N = Wq.shape[0]
        out = np.empty((M, N), np.float32)
        bias_c = None if bias is None else _c(bias, np.float32)
        rc = self.lib.ref_linear_forward_batched(
            _p(_c(Wq, np.int8), _i8p), _p(_c(sW, np.float32)), _p(_c(zpW, np.int32), _i32p),
            _p(_c(sumW, np.int32), _i32p), _p(bias_c), K, N, C.c_float(sA), C.c_int32(zpA),
            M, _p(A), _p(out))
        if rc != 0:
            raise RuntimeError("ref_linear_forward_batched failed")
        return out
