"""Generate the golden fixtures under tests/golden/ from the REFERENCE itself.

Run in a container that has the reference tree (read-only) and its compiled sources
(oracle/_ref, `make -C oracle ref`):

    python tests/golden/make_golden.py <path of the reference checkout>

What it writes (small files, committed):
  fno2d_q.nneuroir      a tiny FNO2d (width 16, 4x4 modes, 2 layers, 16x16) built by
                        the reference's PyTorch model, calibrated by its
                        `quantise_model(per_channel_weights=True)` and exported by its
                        `export_all` (NIRQ per-channel weights + per-tensor activations)
  fno2d_q.npz           input x, the reference C++ runtime's output y (fake-quant FP32
                        FNO2d, oracle/_ref), and the reference Python qparams
  fno2d_plain.nneuroir  the same model without NIRQ, with its runtime output
  calib.npz             its calibration batch and the reference's calibration of it with
                        the 99th-percentile rule and FP8 E4M3 scales (quantise_model)
  fno1d_pt.nneuroir     a tiny FNO1d (width 16, 6 modes, 2 layers, n = 64) calibrated with
                        `quantise_model(per_channel_weights=True,
                        per_token_activations=True)` (NIRQ kind 2) and exported by
                        `export_all`
  fno1d_pc.nneuroir     the same network calibrated with per-tensor activations
  fno1d.npz             input x and the reference runtime's outputs for both files, with
                        and without EnableInt8Gemm
  tm2d.nneuroir         a tiny TokenMixer2D (8x8 grid, 16 patches, latent 16, 2 heads,
                        2 blocks) built by the reference's PyTorch model and exported by
                        `export_all`
  tm2d.npz              input x and the reference runtime's RunTokenMixer2D output
  deeponet.nneuroir     a tiny DeepONet (latent 16, 2 outputs, 3-layer nets of 32 / 24),
  graphop.nneuroir      GraphOp (40-node line graph, hidden 16, 2 blocks),
  graphop2d.nneuroir    GraphOp2D (8x8 grid graph, hidden 16, 2 blocks) and
  tokenmixer.nneuroir   TokenMixer (64 points, 16 patches, latent 16), each built by the
                        reference's PyTorch model and exported by `export_all`
  ops.npz               their inputs and the reference runtime's RunDeepONet /
                        RunGraphOp / RunGraphOp2D / RunTokenMixer outputs
  int8_gemm.npz         LinearForwardBatched vectors (reference C++): W codes, scales,
                        zero points, sum_w, A, C for K = N = 64, plus QuantiseActivation
  fft.npz               Rfft2/Irfft2 of a 16x32 field (reference C++)
  gelu.npz              ApplyActivation GELU on 4096 values (reference C++)
  qparams.npz           compute_tensor_qparams / compute_per_channel_qparams KATs
                        (reference Python)
Nothing here is read from the reference at test time: the tests read these files.
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if len(sys.argv) < 2:
    sys.exit("usage: python tests/golden/make_golden.py <reference project root>")
REF = sys.argv[1]
sys.dont_write_bytecode = True  # never write into the reference tree
sys.path.insert(0, REF)
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from neuroflow.ir.export import export_all, export_to_binary, export_to_neuroir  # noqa: E402
from neuroflow.nn.fno import FNO1d, FNO1dConfig  # noqa: E402
from neuroflow.nn.fno2d import FNO2d, FNO2dConfig  # noqa: E402
from neuroflow.nn.tokenmixer2d import TokenMixer2D, TokenMixer2DConfig  # noqa: E402
from neuroflow.quant import (compute_per_channel_qparams, compute_tensor_qparams,  # noqa: E402
                             quant_to_ir, quantise_model)

from oracle.cpu import Reference  # noqa: E402


def main():
    ref = Reference()
    rng = np.random.default_rng(2024)

    # --- FNO2d with NIRQ ---------------------------------------------------------
    torch.manual_seed(0)
    cfg = FNO2dConfig(in_channels=3, out_channels=1, width=16, modes_h=4, modes_w=4,
                      n_layers=2, activation="gelu", pad_factor=1)
    model = FNO2d(cfg).eval()
    calib = torch.randn(4, 16, 16, 3)
    qm = quantise_model(model, [calib], per_channel_weights=True, per_token_activations=False)
    quant = quant_to_ir(qm)
    with tempfile.TemporaryDirectory() as d:
        _, p = export_all(model, d, basename="fno2d_q", quant=quant)
        blob = open(p, "rb").read()
        _, p2 = export_all(model, d, basename="fno2d_plain")
        blob_plain = open(p2, "rb").read()
    open(os.path.join(HERE, "fno2d_q.nneuroir"), "wb").write(blob)
    open(os.path.join(HERE, "fno2d_plain.nneuroir"), "wb").write(blob_plain)
    x = rng.standard_normal((2, 16, 16, 3)).astype(np.float32)
    y_q = ref.run(os.path.join(HERE, "fno2d_q.nneuroir"), x, 1)
    y_plain = ref.run(os.path.join(HERE, "fno2d_plain.nneuroir"), x, 1)
    act = {k: (v.scale, v.zero_point) for k, v in qm.activation_qparams.items()}
    np.savez_compressed(os.path.join(HERE, "fno2d_q.npz"), x=x, y_q=y_q, y_plain=y_plain,
                        act_keys=np.array(sorted(act)),
                        act_scale=np.array([act[k][0] for k in sorted(act)], np.float32),
                        act_zp=np.array([act[k][1] for k in sorted(act)], np.int32))
    # the same model's calibration by the reference: its calibration batch, min/max
    # (above), the 99th-percentile rule and the FP8 E4M3 scales
    qm99 = quantise_model(model, [calib], per_channel_weights=True, per_token_activations=False,
                          percentile=99.0, fp8_activations=True)
    keys = sorted(qm99.activation_qparams)
    np.savez_compressed(os.path.join(HERE, "calib.npz"), calib=calib.numpy(), keys=np.array(keys),
                        p99_scale=np.array([qm99.activation_qparams[k].scale for k in keys], np.float32),
                        p99_zp=np.array([qm99.activation_qparams[k].zero_point for k in keys], np.int32),
                        fp8_scale=np.array([qm99.fp8_qparams[k].scale for k in keys], np.float32))

    # --- FNO1d, per-token and per-tensor activations ------------------------------
    torch.manual_seed(1)
    cfg1 = FNO1dConfig(in_channels=2, out_channels=1, width=16, modes=6, n_layers=2,
                       activation="gelu", pad_factor=1)
    m1 = FNO1d(cfg1).eval()
    calib1 = torch.randn(4, 64, 2)
    x1 = rng.standard_normal((3, 64, 2)).astype(np.float32)
    outs = {"x": x1}
    for tag, per_token in (("pt", True), ("pc", False)):
        qm1 = quantise_model(m1, [calib1], per_channel_weights=True,
                             per_token_activations=per_token)
        with tempfile.TemporaryDirectory() as d:
            _, p1 = export_all(m1, d, basename=f"fno1d_{tag}", quant=quant_to_ir(qm1))
            blob1 = open(p1, "rb").read()
        path1 = os.path.join(HERE, f"fno1d_{tag}.nneuroir")
        open(path1, "wb").write(blob1)
        outs[f"y_{tag}"] = ref.run(path1, x1, 1)
        outs[f"y_{tag}_int8"] = ref.run(path1, x1, 1, enable_int8=True)
    np.savez_compressed(os.path.join(HERE, "fno1d.npz"), **outs)

    # --- LinearForwardBatched ------------------------------------------------------
    K = N = 64
    M = 300
    W = rng.uniform(-0.125, 0.125, (N, K)).astype(np.float32)
    pc = compute_per_channel_qparams(torch.from_numpy(W), 0)
    sW = np.asarray(pc.scales, np.float32)
    zW = np.asarray(pc.zero_points, np.int32)
    Wq = np.clip(np.round(W / sW[:, None]) + zW[:, None], -128, 127).astype(np.int8)
    import ctypes as C
    sumW = np.empty(N, np.int32)
    ref.lib.ref_precompute_sum_w(Wq.ctypes.data_as(C.c_void_p), zW.ctypes.data_as(C.c_void_p),
                                 K, N, sumW.ctypes.data_as(C.c_void_p))
    A = (rng.standard_normal((M, K)) * 1.7).astype(np.float32)
    qa = compute_tensor_qparams(torch.from_numpy(A))
    Cout = ref.linear_forward_batched(Wq, sW, zW, sumW, None, float(qa.scale), int(qa.zero_point), A)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    Cb = ref.linear_forward_batched(Wq, sW, zW, sumW, bias, float(qa.scale), int(qa.zero_point), A)
    Aq = ref.quantise_activation(A, float(qa.scale), int(qa.zero_point))
    np.savez_compressed(os.path.join(HERE, "int8_gemm.npz"), Wq=Wq, sW=sW, zW=zW, sumW=sumW,
                        A=A, sA=np.float32(qa.scale), zA=np.int32(qa.zero_point), C=Cout,
                        bias=bias, Cb=Cb, Aq=Aq)

    # --- FFT, GELU --------------------------------------------------------------
    f = rng.standard_normal((16, 32)).astype(np.float32)
    F = ref.rfft2(f)
    g = ref.irfft2(F, 16, 32)
    np.savez_compressed(os.path.join(HERE, "fft.npz"), x=f, rfft2=F, irfft2=g)
    z = np.concatenate([np.linspace(-8, 8, 2048), rng.standard_normal(2048) * 3]).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "gelu.npz"), z=z, gelu=ref.activation(z))

    # --- qparam KATs (reference Python) ----------------------------------------------
    cases = [np.linspace(-1, 1, 1001, dtype=np.float32), np.full(7, 0.5, np.float32),
             np.linspace(0.2, 3.0, 50, dtype=np.float32),
             np.linspace(-3.0, -0.1, 50, dtype=np.float32),
             (rng.standard_normal(500) * 2 + 0.3).astype(np.float32)]
    ts, tz = [], []
    for c in cases:
        q = compute_tensor_qparams(torch.from_numpy(c))
        ts.append(q.scale)
        tz.append(q.zero_point)
    Wpc = rng.standard_normal((16, 24)).astype(np.float32)
    Wpc[3] = np.abs(Wpc[3]) + 0.1      # all-positive row (zp clipped low)
    Wpc[5] = -np.abs(Wpc[5]) - 0.1     # all-negative row (zp clipped high)
    pcq = compute_per_channel_qparams(torch.from_numpy(Wpc), 0)
    np.savez_compressed(os.path.join(HERE, "qparams.npz"),
                        **{f"case{i}": c for i, c in enumerate(cases)},
                        t_scale=np.array(ts, np.float64), t_zp=np.array(tz, np.int32),
                        W=Wpc, pc_scale=np.asarray(pcq.scales, np.float32),
                        pc_zp=np.asarray(pcq.zero_points, np.int32))
    # --- TokenMixer2D (appended last so the streams above are unchanged) ------------
    torch.manual_seed(2)
    tm = TokenMixer2D(TokenMixer2DConfig(in_dim=3, out_dim=1, h=8, w=8, n_patches=16,
                                         latent_dim=16, n_heads=2, n_layers=2)).eval()
    with tempfile.TemporaryDirectory() as d:
        _, pt = export_all(tm, d, basename="tm2d")
        blob_t = open(pt, "rb").read()
    path_t = os.path.join(HERE, "tm2d.nneuroir")
    open(path_t, "wb").write(blob_t)
    xt = rng.standard_normal((2, 8, 8, 3)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "tm2d.npz"), x=xt,
                        y=ref.run(path_t, xt, 1, tokenmixer2d=True))

    # --- DeepONet, GraphOp, GraphOp2D, TokenMixer (appended last) -------------------
    from neuroflow.nn.deeponet import DeepONet, DeepONetConfig
    from neuroflow.nn.graph_op import GraphOp, GraphOpConfig
    from neuroflow.nn.graph_op2d import GraphOp2D, GraphOp2DConfig
    from neuroflow.nn.tokenmixer import TokenMixer, TokenMixerConfig

    def export(model, name):
        with tempfile.TemporaryDirectory() as d:
            _, pth = export_all(model, d, basename=name)
            blob_o = open(pth, "rb").read()
        path_o = os.path.join(HERE, name + ".nneuroir")
        open(path_o, "wb").write(blob_o)
        return path_o

    outs = {}
    torch.manual_seed(3)
    dn = DeepONet(DeepONetConfig(in_branch=1, in_trunk=1, latent_dim=16, out_channels=2,
                                 hidden_branch=32, hidden_trunk=24, n_layers_branch=3,
                                 n_layers_trunk=3)).eval()
    path_d = export(dn, "deeponet")
    outs["don_u"] = rng.standard_normal((2, 20, 1)).astype(np.float32)
    outs["don_y"] = rng.uniform(0, 1, (2, 30, 1)).astype(np.float32)
    outs["don_out"] = ref.run_deeponet(path_d, outs["don_u"], outs["don_y"], 2)
    torch.manual_seed(4)
    go = GraphOp(GraphOpConfig(in_dim=2, out_dim=1, n_nodes=40, hidden_dim=16, n_layers=2)).eval()
    path_g = export(go, "graphop")
    outs["gop_x"] = rng.standard_normal((2, 40, 2)).astype(np.float32)
    outs["gop_y"] = ref.run_other(path_g, "GraphOp", outs["gop_x"], 1)
    torch.manual_seed(5)
    g2 = GraphOp2D(GraphOp2DConfig(in_dim=1, out_dim=2, h=8, w=8, hidden_dim=16, n_layers=2)).eval()
    path_g2 = export(g2, "graphop2d")
    outs["g2_x"] = rng.standard_normal((2, 8, 8, 1)).astype(np.float32)
    outs["g2_y"] = ref.run_other(path_g2, "GraphOp2D", outs["g2_x"], 2)
    torch.manual_seed(6)
    tk = TokenMixer(TokenMixerConfig(in_dim=2, out_dim=1, n_points=64, n_patches=16,
                                     latent_dim=16, n_heads=2, n_layers=1)).eval()
    path_tk = export(tk, "tokenmixer")
    outs["tk_x"] = rng.standard_normal((2, 64, 2)).astype(np.float32)
    outs["tk_y"] = ref.run_other(path_tk, "TokenMixer", outs["tk_x"], 1)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **outs)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
