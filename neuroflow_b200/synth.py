"""Seeded synthetic inputs and random-init models with the shapes of the benchmark
configurations (no dataset or checkpoint is available offline).

* Gaussian random fields: periodic, spectrum ~ (|k|^2 + tau^2)^-2, unit std.
* Weights: spectral U(-1, 1)/(in*out); Linear Kaiming-uniform as PyTorch's default
  init (U(+-1/sqrt(fan_in)) for weight and bias).
* Calibration: forward hooks on every Linear output of the float32 model, min/max over
  a separate calibration batch, as the reference's `calibrate`
  (neuroflow/quant/static_quant.py:609-741) does.  The float32 forward here follows
  neuroflow/nn/fno2d.py:150-180 (torch.fft, exact GELU as torch's F.gelu).
This module is a fixture producer for tests and bench.py, not part of the inference
path.
"""
from __future__ import annotations

import math

import numpy as np

from . import ir, quant


def grf2d(rng: np.random.Generator, n: int, H: int, W: int, tau: float = 3.0) -> np.ndarray:
    """(n, H, W) periodic GRF with spectrum (|k|^2 + tau^2)^-2, normalised to unit std."""
    kh = np.fft.fftfreq(H, d=1.0 / H)[:, None]
    kw = np.fft.rfftfreq(W, d=1.0 / W)[None, :]
    amp = (kh ** 2 + kw ** 2 + tau ** 2) ** -1.0  # sqrt of the (.)^-2 power spectrum
    out = np.empty((n, H, W), np.float32)
    for i in range(n):
        z = rng.standard_normal((H, W // 2 + 1)) + 1j * rng.standard_normal((H, W // 2 + 1))
        f = np.fft.irfft2(z * amp, s=(H, W))
        f = (f - f.mean()) / (f.std() + 1e-12)
        out[i] = f.astype(np.float32)
    return out


def grf3d(rng: np.random.Generator, n: int, S: int, tau: float = 2.0) -> np.ndarray:
    k0 = np.fft.fftfreq(S, d=1.0 / S)
    kd = np.fft.rfftfreq(S, d=1.0 / S)
    amp = (k0[:, None, None] ** 2 + k0[None, :, None] ** 2 + kd[None, None, :] ** 2
           + tau ** 2) ** -1.0
    out = np.empty((n, S, S, S), np.float32)
    for i in range(n):
        z = rng.standard_normal(amp.shape) + 1j * rng.standard_normal(amp.shape)
        f = np.fft.irfftn(z * amp, s=(S, S, S), axes=(0, 1, 2))
        f = (f - f.mean()) / (f.std() + 1e-12)
        out[i] = f.astype(np.float32)
    return out


def fno2d_inputs(rng: np.random.Generator, n: int, H: int, W: int, in_ch: int = 3) -> np.ndarray:
    """(n, H, W, in_ch): field + grid coordinates in [0, 1) (+ extra GRFs if in_ch > 3)."""
    x = np.empty((n, H, W, in_ch), np.float32)
    x[..., 0] = grf2d(rng, n, H, W)
    if in_ch >= 2:
        x[..., 1] = (np.arange(H, dtype=np.float32) / H)[None, :, None]
    if in_ch >= 3:
        x[..., 2] = (np.arange(W, dtype=np.float32) / W)[None, None, :]
    for c in range(3, in_ch):
        x[..., c] = grf2d(rng, n, H, W)
    return x


def _kaiming_linear(rng, out_f: int, in_f: int):
    bound = 1.0 / math.sqrt(in_f)
    w = rng.uniform(-bound, bound, size=(out_f, in_f)).astype(np.float32)
    b = rng.uniform(-bound, bound, size=(out_f,)).astype(np.float32)
    return w, b


def fno2d_weights(rng, in_ch, out_ch, width, mh, mw, L):
    wts = {}
    wts["lift.weight"], wts["lift.bias"] = _kaiming_linear(rng, width, in_ch)
    s = 1.0 / (width * width)
    for i in range(L):
        wts[f"specs.{i}.weights_real"] = (s * rng.uniform(-1, 1, (width, width, mh, mw))).astype(np.float32)
        wts[f"specs.{i}.weights_imag"] = (s * rng.uniform(-1, 1, (width, width, mh, mw))).astype(np.float32)
        wts[f"locs.{i}.weight"], wts[f"locs.{i}.bias"] = _kaiming_linear(rng, width, width)
    wts["proj_q.weight"], wts["proj_q.bias"] = _kaiming_linear(rng, width, width)
    wts["proj_out.weight"], wts["proj_out.bias"] = _kaiming_linear(rng, out_ch, width)
    return wts


def fno2d_linear_outputs(wts: dict, x: np.ndarray, L: int, mh: int, mw: int) -> dict:
    """Float32 FNO2d forward (neuroflow/nn/fno2d.py:150-180) returning every Linear's
    output, the statistics `calibrate` hooks."""
    import torch
    import torch.nn.functional as F

    def lin(t, name):
        return t @ torch.from_numpy(wts[name + ".weight"]).T + torch.from_numpy(wts[name + ".bias"])

    obs = {}
    with torch.no_grad():
        h = lin(torch.from_numpy(x), "lift")
        obs["lift.output"] = h.numpy().copy()
        h = h.permute(0, 3, 1, 2)
        Hh, Ww = h.shape[-2], h.shape[-1]
        for i in range(L):
            xf = torch.fft.rfftn(h, dim=(-2, -1))[..., :mh, :mw]
            wgt = torch.complex(torch.from_numpy(wts[f"specs.{i}.weights_real"]),
                                torch.from_numpy(wts[f"specs.{i}.weights_imag"]))
            of = torch.einsum("bimn,iomn->bomn", xf, wgt)
            of = F.pad(of, (0, (Ww // 2 + 1) - mw, 0, Hh - mh))
            x1 = torch.fft.irfftn(of, s=(Hh, Ww), dim=(-2, -1))
            x2 = lin(h.permute(0, 2, 3, 1), f"locs.{i}")
            obs[f"locs.{i}.output"] = x2.numpy().copy()
            h = F.gelu(x1 + x2.permute(0, 3, 1, 2))
        q = lin(h.permute(0, 2, 3, 1), "proj_q")
        obs["proj_q.output"] = q.numpy().copy()
        y = lin(F.gelu(q), "proj_out")
        obs["proj_out.output"] = y.numpy().copy()
    return obs


def fno2d_model(seed: int, in_ch=3, out_ch=1, width=64, mh=12, mw=12, L=4, H=128, W=128,
                n_calib=32, per_channel=True, calib_chunk=8) -> ir.Model:
    """A random-init FNO2d with a calibrated NIRQ block (per-channel weights,
    per-tensor activations), ready for ir.write."""
    rng = np.random.default_rng(seed)
    wts = fno2d_weights(rng, in_ch, out_ch, width, mh, mw, L)
    crng = np.random.default_rng(seed + 1)
    mins, maxs = {}, {}
    done = 0
    while done < n_calib:
        nb = min(calib_chunk, n_calib - done)
        xc = fno2d_inputs(crng, nb, H, W, in_ch)
        for k, v in fno2d_linear_outputs(wts, xc, L, mh, mw).items():
            mins[k] = min(mins.get(k, np.inf), float(v.min()))
            maxs[k] = max(maxs.get(k, -np.inf), float(v.max()))
        done += nb
    qp = quant.weight_qparams(wts, per_channel=per_channel)
    for k in mins:
        qp[k] = quant.tensor_qparams(np.array([mins[k], maxs[k]], np.float32))
    cfg = dict(in_channels=in_ch, out_channels=out_ch, width=width, modes_h=mh, modes_w=mw,
               n_layers=L, pad_factor=1)
    return ir.Model(op="FNO2d", config=cfg, weights=wts, qparams=qp, quant_enabled=True)


# ------------------------------------------------------------------------- FNO1d
def grf1d(rng: np.random.Generator, n_samples: int, n: int, n_modes: int = 32) -> np.ndarray:
    """(n_samples, n) periodic field: sum of `n_modes` cos/sin pairs with coefficients
    ~ N(0, k^-2), normalised to unit std."""
    xs = np.arange(n, dtype=np.float64) / n
    k = np.arange(1, n_modes + 1, dtype=np.float64)
    basis_c = np.cos(2 * np.pi * k[:, None] * xs[None, :])
    basis_s = np.sin(2 * np.pi * k[:, None] * xs[None, :])
    out = np.empty((n_samples, n), np.float32)
    for i in range(n_samples):
        a = rng.standard_normal(n_modes) / k
        b = rng.standard_normal(n_modes) / k
        f = a @ basis_c + b @ basis_s
        f = (f - f.mean()) / (f.std() + 1e-12)
        out[i] = f.astype(np.float32)
    return out


def fno1d_inputs(rng: np.random.Generator, n_samples: int, n: int, in_ch: int = 2) -> np.ndarray:
    """(n_samples, n, in_ch): field u0 + the grid x in [0, 1) (+ extra fields)."""
    x = np.empty((n_samples, n, in_ch), np.float32)
    x[..., 0] = grf1d(rng, n_samples, n)
    if in_ch >= 2:
        x[..., 1] = (np.arange(n, dtype=np.float32) / n)[None, :]
    for c in range(2, in_ch):
        x[..., c] = grf1d(rng, n_samples, n)
    return x


def fno1d_weights(rng, in_ch, out_ch, width, modes, L):
    wts = {}
    wts["lift.weight"], wts["lift.bias"] = _kaiming_linear(rng, width, in_ch)
    s = 1.0 / (width * width)
    for i in range(L):
        wts[f"specs.{i}.weights_real"] = (s * rng.uniform(-1, 1, (width, width, modes))).astype(np.float32)
        wts[f"specs.{i}.weights_imag"] = (s * rng.uniform(-1, 1, (width, width, modes))).astype(np.float32)
        wts[f"locs.{i}.weight"], wts[f"locs.{i}.bias"] = _kaiming_linear(rng, width, width)
    wts["proj_q.weight"], wts["proj_q.bias"] = _kaiming_linear(rng, width, width)
    wts["proj_out.weight"], wts["proj_out.bias"] = _kaiming_linear(rng, out_ch, width)
    return wts


def fno1d_linear_outputs(wts: dict, x: np.ndarray, L: int, modes: int, pad_factor: int = 1) -> dict:
    """Float32 FNO1d forward (neuroflow/nn/fno.py:126-150) returning every Linear's
    output (batch, n, features), the tensors `calibrate` hooks."""
    import torch
    import torch.nn.functional as F

    def lin(t, name):
        return t @ torch.from_numpy(wts[name + ".weight"]).T + torch.from_numpy(wts[name + ".bias"])

    obs = {}
    with torch.no_grad():
        h = lin(torch.from_numpy(x), "lift")
        obs["lift.output"] = h.numpy().copy()
        h = h.permute(0, 2, 1)
        pad_len = 0
        if pad_factor > 1:
            pad_len = (pad_factor - (h.shape[-1] % pad_factor)) % pad_factor
            h = F.pad(h, (0, pad_len))
        n = h.shape[-1]
        for i in range(L):
            xf = torch.fft.rfft(h, dim=-1)[..., :modes]
            wgt = torch.complex(torch.from_numpy(wts[f"specs.{i}.weights_real"]),
                                torch.from_numpy(wts[f"specs.{i}.weights_imag"]))
            of = F.pad(torch.einsum("bim,iom->bom", xf, wgt), (0, (n // 2 + 1) - modes))
            x1 = torch.fft.irfft(of, n=n, dim=-1)
            x2 = lin(h.permute(0, 2, 1), f"locs.{i}")
            obs[f"locs.{i}.output"] = x2.numpy().copy()
            h = F.gelu(x1 + x2.permute(0, 2, 1))
        if pad_len > 0:
            h = h[..., :-pad_len]
        q = lin(h.permute(0, 2, 1), "proj_q")
        obs["proj_q.output"] = q.numpy().copy()
        y = lin(F.gelu(q), "proj_out")
        obs["proj_out.output"] = y.numpy().copy()
    return obs


def fno1d_model(seed: int, in_ch=2, out_ch=1, width=64, modes=16, L=4, n=1024, n_calib=32,
                per_token=True, per_channel=True, quantised=True, pad_factor=0,
                calib_chunk=32) -> ir.Model:
    """A random-init FNO1d (configs[0] shape by default).  With `quantised`, a calibrated
    NIRQ block: per-channel (or per-tensor) weights and per-token (or per-tensor)
    activations, as `quantise_model(per_channel_weights, per_token_activations)`
    exports them."""
    rng = np.random.default_rng(seed)
    wts = fno1d_weights(rng, in_ch, out_ch, width, modes, L)
    cfg = dict(in_channels=in_ch, out_channels=out_ch, width=width, modes=modes, n_layers=L,
               pad_factor=pad_factor, _=0)
    if not quantised:
        return ir.Model(op="FNO1d", config=cfg, weights=wts, quant_enabled=False)
    crng = np.random.default_rng(seed + 1)
    obs = {}
    done = 0
    while done < n_calib:
        nb = min(calib_chunk, n_calib - done)
        xc = fno1d_inputs(crng, nb, n, in_ch)
        for k, v in fno1d_linear_outputs(wts, xc, L, modes, pad_factor).items():
            obs.setdefault(k, []).append(v)
        done += nb
    qp = quant.weight_qparams(wts, per_channel=per_channel)
    for k, vs in obs.items():
        st = np.concatenate(vs, axis=0)
        qp[k] = quant.per_token_qparams(st) if per_token else quant.tensor_qparams(st)
    return ir.Model(op="FNO1d", config=cfg, weights=wts, qparams=qp, quant_enabled=True)


# ------------------------------------------------------------------ TokenMixer2D
TM2D_PARTS = ("ln1", "q_proj", "k_proj", "v_proj", "o_proj", "ln2", "ffn0", "ffn1")
TM2D_INT8_PARTS = ("q_proj", "k_proj", "v_proj", "o_proj", "ffn0", "ffn1")


def tm2d_model(seed: int, in_dim=3, out_dim=1, latent=128, h=64, w=64, n_patches=4096,
               n_heads=4, n_layers=4, activation="gelu") -> ir.Model:
    """A random-init TokenMixer2D (configs[4] shape by default): LayerNorm gamma = 1,
    beta = 0, every Linear Kaiming-uniform.  The NIRQ block carries per-channel weight
    qparams of the six INT8 layers (q, k, v, o, ffn0, ffn1); the reference runtime
    ignores NIRQ for this op, the INT8 executor reads them."""
    rng = np.random.default_rng(seed)
    wts = {}
    wts["slice_embed.proj.weight"], wts["slice_embed.proj.bias"] = _kaiming_linear(rng, latent, in_dim)
    for i in range(n_layers):
        pre = f"blocks.{i}."
        for part in TM2D_PARTS:
            if part.startswith("ln"):
                wts[pre + part + ".weight"] = np.ones(latent, np.float32)
                wts[pre + part + ".bias"] = np.zeros(latent, np.float32)
            else:
                o, k = {"ffn0": (2 * latent, latent), "ffn1": (latent, 2 * latent)}.get(part, (latent, latent))
                wts[pre + part + ".weight"], wts[pre + part + ".bias"] = _kaiming_linear(rng, o, k)
    wts["unslice.proj.weight"], wts["unslice.proj.bias"] = _kaiming_linear(rng, latent, in_dim + latent)
    wts["head.weight"], wts["head.bias"] = _kaiming_linear(rng, out_dim, latent)
    qp = {}
    for i in range(n_layers):
        for part in TM2D_INT8_PARTS:
            name = f"blocks.{i}.{part}.weight"
            qp[name] = quant.per_channel_qparams(wts[name], 0)
    cfg = dict(in_dim=in_dim, out_dim=out_dim, latent_dim=latent, h=h, w=w, n_patches=n_patches,
               n_heads=n_heads, n_layers=n_layers)
    return ir.Model(op="TokenMixer2D", config=cfg, activation=activation, weights=wts, qparams=qp,
                    quant_enabled=True)


def tm2d_inputs(rng: np.random.Generator, n: int, h: int, w: int, in_dim: int = 3) -> np.ndarray:
    """(n, h, w, in_dim): a GRF field (spectrum as configs[2]) + grid coordinates."""
    return fno2d_inputs(rng, n, h, w, in_dim)


# ------------------------------------------------------------------------- FNO3d
def fno3d_inputs(rng: np.random.Generator, n: int, S: int, in_ch: int = 4) -> np.ndarray:
    """(n, S, S, S, in_ch): a 3-D GRF (spectrum (|k|^2 + 4)^-2) + grid coordinates."""
    x = np.empty((n, S, S, S, in_ch), np.float32)
    x[..., 0] = grf3d(rng, n, S)
    g = np.arange(S, dtype=np.float32) / S
    if in_ch >= 2:
        x[..., 1] = g[None, :, None, None]
    if in_ch >= 3:
        x[..., 2] = g[None, None, :, None]
    if in_ch >= 4:
        x[..., 3] = g[None, None, None, :]
    for c in range(4, in_ch):
        x[..., c] = grf3d(rng, n, S)
    return x


def fno3d_weights(rng, in_ch, out_ch, width, modes, L):
    wts = {}
    wts["lift.weight"], wts["lift.bias"] = _kaiming_linear(rng, width, in_ch)
    s = 1.0 / (width * width)
    for i in range(L):
        for part in ("weights_real", "weights_imag"):
            wts[f"specs.{i}.{part}"] = (s * rng.uniform(-1, 1, (width, width) + tuple(modes))).astype(np.float32)
        wts[f"locs.{i}.weight"], wts[f"locs.{i}.bias"] = _kaiming_linear(rng, width, width)
    wts["proj_q.weight"], wts["proj_q.bias"] = _kaiming_linear(rng, width, width)
    wts["proj_out.weight"], wts["proj_out.bias"] = _kaiming_linear(rng, out_ch, width)
    return wts


def fno3d_linear_outputs(wts: dict, x: np.ndarray, L: int, modes) -> dict:
    """Float32 FNO3d forward (neuroflow/nn/fno3d.py structure: torch.fft, exact GELU)
    returning every Linear's output."""
    import torch
    import torch.nn.functional as F

    def lin(t, name):
        return t @ torch.from_numpy(wts[name + ".weight"]).T + torch.from_numpy(wts[name + ".bias"])

    mh, mw, md = modes
    obs = {}
    with torch.no_grad():
        h = lin(torch.from_numpy(x), "lift")
        obs["lift.output"] = h.numpy().copy()
        h = h.permute(0, 4, 1, 2, 3)
        S = h.shape[-3:]
        for i in range(L):
            xf = torch.fft.rfftn(h, dim=(-3, -2, -1))[..., :mh, :mw, :md]
            wgt = torch.complex(torch.from_numpy(wts[f"specs.{i}.weights_real"]),
                                torch.from_numpy(wts[f"specs.{i}.weights_imag"]))
            of = torch.einsum("bixyz,ioxyz->boxyz", xf, wgt)
            of = F.pad(of, (0, S[2] // 2 + 1 - md, 0, S[1] - mw, 0, S[0] - mh))
            x1 = torch.fft.irfftn(of, s=S, dim=(-3, -2, -1))
            x2 = lin(h.permute(0, 2, 3, 4, 1), f"locs.{i}")
            obs[f"locs.{i}.output"] = x2.numpy().copy()
            h = F.gelu(x1 + x2.permute(0, 4, 1, 2, 3))
        q = lin(h.permute(0, 2, 3, 4, 1), "proj_q")
        obs["proj_q.output"] = q.numpy().copy()
        y = lin(F.gelu(q), "proj_out")
        obs["proj_out.output"] = y.numpy().copy()
    return obs


def fno3d_model(seed: int, in_ch=4, out_ch=1, width=32, modes=(8, 8, 8), L=4, S=64,
                n_calib=4, calib_chunk=2) -> ir.Model:
    """A random-init FNO3d (configs[3] shape by default) with FP8 E4M3 per-tensor scales
    (amax / 448, compute_fp8_e4m3_qparams, static_quant.py:338-352) for every Linear
    output over a separate calibration batch and for every Linear weight, as NIRQ
    kind-3 entries.  The reference runtime ignores NIRQ for FNO3d."""
    rng = np.random.default_rng(seed)
    wts = fno3d_weights(rng, in_ch, out_ch, width, modes, L)
    crng = np.random.default_rng(seed + 1)
    amax = {}
    done = 0
    while done < n_calib:
        nb = min(calib_chunk, n_calib - done)
        xc = fno3d_inputs(crng, nb, S, in_ch)
        for k, v in fno3d_linear_outputs(wts, xc, L, modes).items():
            amax[k] = max(amax.get(k, 0.0), float(np.abs(v).max()))
        done += nb
    qp = {k: quant.fp8_qparams(np.array([v], np.float32)) for k, v in amax.items()}
    for name, t in wts.items():
        if name.endswith(".weight"):
            qp[name] = quant.fp8_qparams(t)
    cfg = dict(in_channels=in_ch, out_channels=out_ch, width=width, modes_h=modes[0],
               modes_w=modes[1], modes_d=modes[2], n_layers=L, pad_factor=1)
    return ir.Model(op="FNO3d", config=cfg, weights=wts, qparams=qp, quant_enabled=True)


# ------------------------------------------------------------------------- DeepONet
def deeponet_model(seed: int, in_branch=1, in_trunk=1, latent=32, out_ch=1, hidden_branch=64,
                   hidden_trunk=64, n_branch=3, n_trunk=3, activation="gelu") -> ir.Model:
    """A random-init DeepONet (the reference's default widths): branch and trunk MLPs
    with Kaiming-uniform Linears (the branch's last layer out_ch * latent wide), output
    bias U(-0.1, 0.1).  Hidden widths are what the loader infers from the second-to-last
    layer of each net."""
    rng = np.random.default_rng(seed)
    wts = {}
    for net, n, k0, hid, last in (("branch", n_branch, in_branch, hidden_branch, out_ch * latent),
                                  ("trunk", n_trunk, in_trunk, hidden_trunk, latent)):
        k = k0
        for i in range(n):
            o = last if i == n - 1 else hid
            wts[f"{net}.layers.{i}.weight"], wts[f"{net}.layers.{i}.bias"] = _kaiming_linear(rng, o, k)
            k = o
    wts["bias.weight"] = rng.uniform(-0.1, 0.1, out_ch).astype(np.float32)
    cfg = dict(in_branch=in_branch, in_trunk=in_trunk, latent_dim=latent, out_channels=out_ch,
               n_layers_branch=n_branch, n_layers_trunk=n_trunk)
    return ir.Model(op="DeepONet", config=cfg, activation=activation, weights=wts)


def deeponet_inputs(rng: np.random.Generator, n: int, n_sensor: int, n_query: int, in_branch=1,
                    in_trunk=1):
    """u (n, n_sensor, in_branch): GRF values at the sensors (+ further GRF channels);
    y (n, n_query, in_trunk): query coordinates in [0, 1) (+ uniform extra features)."""
    u = np.empty((n, n_sensor, in_branch), np.float32)
    for c in range(in_branch):
        u[..., c] = grf1d(rng, n, n_sensor)
    y = rng.uniform(0.0, 1.0, (n, n_query, in_trunk)).astype(np.float32)
    return u, y


# ------------------------------------------------------------------------- GraphOp
def line_graph(n: int):
    """CSR of a line graph with self-loops, each node listing itself, then its left and
    right neighbours (neuroflow/nn/graph_op.py's convention)."""
    off, idx = [0], []
    for i in range(n):
        nb = [i] + ([i - 1] if i > 0 else []) + ([i + 1] if i < n - 1 else [])
        idx += nb
        off.append(len(idx))
    return np.array(off, np.int64), np.array(idx, np.int64)


def grid8_graph(h: int, w: int):
    """CSR of an h x w grid with self-loops and 8-connectivity: itself first, then the
    in-grid neighbours in (di, dj) row-major order (neuroflow/nn/graph_op2d.py's
    convention)."""
    off, idx = [0], []
    for i in range(h):
        for j in range(w):
            nb = [i * w + j]
            for di in (-1, 0, 1):
                for dj in (-1, 0, 1):
                    if (di or dj) and 0 <= i + di < h and 0 <= j + dj < w:
                        nb.append((i + di) * w + j + dj)
            idx += nb
            off.append(len(idx))
    return np.array(off, np.int64), np.array(idx, np.int64)


def graphop_model(seed: int, in_dim=1, out_dim=1, hidden=32, n_layers=1, n_nodes=64, h=None, w=None,
                  activation="gelu") -> ir.Model:
    """A random-init GraphOp (n_nodes on a line graph) or, with h and w, GraphOp2D (an
    8-connected grid); deg_inv = 1 / max(deg, 1) as float32, the adjacency stored as
    float tensors as the reference's exporter writes it."""
    rng = np.random.default_rng(seed)
    two_d = h is not None
    off, idx = grid8_graph(h, w) if two_d else line_graph(n_nodes)
    nn_ = (h * w) if two_d else n_nodes
    deg = np.maximum(np.diff(off).astype(np.float32), 1.0)
    wts = {}
    wts["lift.weight"], wts["lift.bias"] = _kaiming_linear(rng, hidden, in_dim)
    for i in range(n_layers):
        p = f"blocks.{i}."
        wts[p + "lin_self.weight"], wts[p + "lin_self.bias"] = _kaiming_linear(rng, hidden, hidden)
        wts[p + "lin_neigh.weight"], wts[p + "lin_neigh.bias"] = _kaiming_linear(rng, hidden, hidden)
    wts["head.weight"], wts["head.bias"] = _kaiming_linear(rng, out_dim, hidden)
    wts["graph.adj_offsets"] = off.astype(np.float32)
    wts["graph.adj_indices"] = idx.astype(np.float32)
    wts["graph.deg_inv"] = (np.float32(1.0) / deg).astype(np.float32)
    if two_d:
        cfg = dict(in_dim=in_dim, out_dim=out_dim, h=h, w=w, hidden_dim=hidden, n_layers=n_layers)
        return ir.Model(op="GraphOp2D", config=cfg, activation=activation, weights=wts)
    cfg = dict(in_dim=in_dim, out_dim=out_dim, n_nodes=n_nodes, hidden_dim=hidden, n_layers=n_layers)
    return ir.Model(op="GraphOp", config=cfg, activation=activation, weights=wts)


def tokenmixer_model(seed: int, in_dim=2, out_dim=1, latent=64, n_points=1024, n_patches=64,
                     n_heads=4, n_layers=2, activation="gelu") -> ir.Model:
    """A random-init 1D TokenMixer: the TokenMixer2D weights on n_points points."""
    m = tm2d_model(seed, in_dim=in_dim, out_dim=out_dim, latent=latent, h=1, w=n_points,
                   n_patches=n_patches, n_heads=n_heads, n_layers=n_layers, activation=activation)
    cfg = dict(in_dim=in_dim, out_dim=out_dim, latent_dim=latent, n_points=n_points,
               n_patches=n_patches, n_heads=n_heads, n_layers=n_layers)
    return ir.Model(op="TokenMixer", config=cfg, activation=activation, weights=m.weights,
                    qparams=m.qparams, quant_enabled=m.quant_enabled)
