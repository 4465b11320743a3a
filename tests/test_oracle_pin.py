"""CPU: the C restatement (oracle/) pinned against the reference.

1. Against the committed golden fixtures (tests/golden/, made by make_golden.py from the
   reference's own Python exporter/quantiser and its C++ runtime): bit-exact.
2. Against the reference sources compiled in place (oracle/_ref, with the reference
   build's own flags) on fresh random inputs, when that library is present (it is
   built by __graft_entry__.build() where the reference tree exists): bit-exact.
"""
import os

import numpy as np
import pytest

from neuroflow_b200 import ir, quant, synth
from oracle.cpu import REF_SO, Oracle, Reference

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
needs_ref = pytest.mark.skipif(not os.path.exists(REF_SO),
                               reason="oracle/_ref not built (needs the reference tree)")


def _g(name):
    return np.load(os.path.join(GOLD, name))


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---------------------------------------------------------------- golden fixtures
def test_golden_fno2d_fake_quant_network():
    d = _g("fno2d_q.npz")
    m = ir.read(os.path.join(GOLD, "fno2d_q.nneuroir"))
    assert m.op == "FNO2d" and m.quant_enabled
    y = Oracle().fno2d_forward(m, d["x"], mode=0)
    assert np.array_equal(_bits(y), _bits(d["y_q"]))


def test_golden_fno2d_plain_network():
    d = _g("fno2d_q.npz")
    m = ir.read(os.path.join(GOLD, "fno2d_plain.nneuroir"))
    assert not m.quant_enabled
    y = Oracle().fno2d_forward(m, d["x"], mode=0)
    assert np.array_equal(_bits(y), _bits(d["y_plain"]))


@pytest.mark.parametrize("tag", ["pt", "pc"])
def test_golden_fno1d_networks(tag):
    """FNO1d models calibrated and exported by the reference's own Python package
    (per-token activations "pt", per-tensor "pc"), run by the reference runtime with
    and without EnableInt8Gemm: the restatement reproduces every output bit."""
    d = _g("fno1d.npz")
    m = ir.read(os.path.join(GOLD, f"fno1d_{tag}.nneuroir"))
    assert m.op == "FNO1d" and m.quant_enabled
    kinds = {type(m.qparams[k]).__name__ for k in m.qparams if k.endswith(".output")}
    assert kinds == ({"PerToken"} if tag == "pt" else {"PerTensor"})
    o = Oracle()
    assert np.array_equal(_bits(o.fno1d_forward(m, d["x"])), _bits(d[f"y_{tag}"]))
    assert np.array_equal(_bits(o.fno1d_forward(m, d["x"], int8=True)), _bits(d[f"y_{tag}_int8"]))


def test_golden_tm2d_network():
    """A TokenMixer2D built by the reference's PyTorch model and exported by its
    exporter; the reference runtime's RunTokenMixer2D output, every bit."""
    d = _g("tm2d.npz")
    m = ir.read(os.path.join(GOLD, "tm2d.nneuroir"))
    assert m.op == "TokenMixer2D" and m.config["n_patches"] == 16
    assert np.array_equal(_bits(Oracle().tm2d_forward(m, d["x"])), _bits(d["y"]))


def test_e4m3_known_answers():
    """The reference's own FP8 known-answer cases (cpp/tests/test_fp8_e4m3.cpp:50-140)
    and the F6 band: [7.5, 8) * 2^-9 stays at code 7 (an IEEE-style encoder gives 2^-6)."""
    o = Oracle()
    kat = [(0.0, 0x00), (-0.0, 0x80), (1.0, 0x38), (-1.0, 0xB8), (448.0, 0x7E),
           (-448.0, 0xFE), (1.0625, 0x38), (1.1875, 0x3A), (1.10, 0x39), (1000.0, 0x7E),
           (-1000.0, 0xFE), (float("inf"), 0x7E), (float("-inf"), 0xFE),
           (float("nan"), 0x7F), (7.6 / 512, 0x07), (7.99 / 512, 0x07), (1.0 / 64, 0x08),
           (3.0 / 512, 0x03)]
    for v, b in kat:
        assert o.lib.nfo_fp32_to_e4m3(v) == b, (v, hex(o.lib.nfo_fp32_to_e4m3(v)))
    assert o.lib.nfo_e4m3_to_fp32(0x38) == 1.0 and o.lib.nfo_e4m3_to_fp32(0x7E) == 448.0
    assert o.lib.nfo_e4m3_to_fp32(0x08) == 1.0 / 64
    assert np.isnan(o.lib.nfo_e4m3_to_fp32(0x7F)) and np.isnan(o.lib.nfo_e4m3_to_fp32(0xFF))


def test_golden_linear_forward_batched_and_quantiser():
    d = _g("int8_gemm.npz")
    o = Oracle()
    c, acc, codes = o.linear_forward_batched(d["Wq"], d["sW"], d["zW"], d["sumW"], None,
                                             float(d["sA"]), int(d["zA"]), d["A"])
    assert np.array_equal(_bits(c), _bits(d["C"]))
    assert np.array_equal(codes, d["Aq"])
    cb, _, _ = o.linear_forward_batched(d["Wq"], d["sW"], d["zW"], d["sumW"], d["bias"],
                                        float(d["sA"]), int(d["zA"]), d["A"])
    assert np.array_equal(_bits(cb), _bits(d["Cb"]))
    # the precomputed row sums of the fixture equal the restated rule
    assert np.array_equal(d["sumW"],
                          (d["Wq"].astype(np.int32) - d["zW"][:, None]).sum(axis=1))


def test_golden_fft_and_gelu():
    d = _g("fft.npz")
    o = Oracle()
    assert np.array_equal(_bits(o.rfft2(d["x"])), _bits(d["rfft2"]))
    assert np.array_equal(_bits(o.irfft2(d["rfft2"], 16, 32)), _bits(d["irfft2"]))
    g = _g("gelu.npz")
    assert np.array_equal(_bits(o.activation(g["z"])), _bits(g["gelu"]))


def test_golden_qparam_rules():
    d = _g("qparams.npz")
    for i in range(5):
        q = quant.tensor_qparams(d[f"case{i}"])
        assert np.float32(q.scale) == np.float32(d["t_scale"][i])
        assert q.zero_point == d["t_zp"][i]
    pc = quant.per_channel_qparams(d["W"], 0)
    assert np.array_equal(_bits(pc.scales), _bits(d["pc_scale"]))
    assert np.array_equal(pc.zero_points, d["pc_zp"])


def test_golden_ir_bytes_roundtrip():
    for name in ("fno2d_q.nneuroir", "fno2d_plain.nneuroir"):
        raw = open(os.path.join(GOLD, name), "rb").read()
        m = ir.read_bytes(raw)
        assert ir.write_bytes(m) == raw
        assert m.config["width"] == 16 and m.config["n_layers"] == 2


def test_golden_ir_through_the_cpp_loader():
    from neuroflow_b200 import _nfx
    op, cfg, nw, q = _nfx.load_neuroir(os.path.join(GOLD, "fno2d_q.nneuroir"))
    assert op == "FNO2d" and cfg[:7] == [3, 1, 16, 4, 4, 2, 1] and nw == 14 and q
    # the other op families' reference-exported files: op, config block, weight count
    for name, want_op, want_cfg, want_nw in (
            ("deeponet", "DeepONet", [1, 1, 16, 2, 3, 3, 0], 13),
            ("graphop", "GraphOp", [2, 1, 40, 16, 2, 0, 0, 0], 15),
            ("graphop2d", "GraphOp2D", [1, 2, 8, 8, 16, 2, 0, 0], 15),
            ("tokenmixer", "TokenMixer", [2, 1, 16, 64, 16, 2, 1, 0], 22)):
        path = os.path.join(GOLD, name + ".nneuroir")
        op, cfg, nw, q = _nfx.load_neuroir(path)
        assert (op, cfg[:len(want_cfg)], nw, q) == (want_op, want_cfg, want_nw, False), name
        assert ir.write_bytes(ir.read(path)) == open(path, "rb").read()


def test_cpp_loader_error_codes(tmp_path):
    from neuroflow_b200 import _nfx
    raw = open(os.path.join(GOLD, "fno2d_q.nneuroir"), "rb").read()
    cases = {
        "missing": (None, 2, "cannot open IR file"),
        "magic": (b"NIRX" + raw[4:], 3, "bad magic"),
        "version": (raw[:4] + b"\x04\x00" + raw[6:], 3, "unsupported IR binary version"),
        "opcode": (raw[:6] + b"\x09" + raw[7:], 5, "unknown op_code"),
        "truncated": (raw[:5000], 3, "truncated"),
        "name": (raw.replace(b"locs.1.weight", b"locs.1.weighX"), 3, "weight name mismatch"),
        "nirq_kind": (raw[:raw.index(b"NIRQ") + 9] + b"\x07" + raw[raw.index(b"NIRQ") + 10:], 3,
                      "unsupported qparam kind"),
    }
    for key, (blob, code, msg) in cases.items():
        p = tmp_path / f"{key}.nneuroir"
        if blob is not None:
            p.write_bytes(blob)
        with pytest.raises(_nfx.NfxError) as ei:
            _nfx.load_neuroir(str(p))
        assert ei.value.code == code, key
        assert msg in str(ei.value), key
    # a file without NIRQ ends right after the weights and loads fine
    p = tmp_path / "plain.nneuroir"
    p.write_bytes(raw[:raw.index(b"NIRQ")])
    assert _nfx.load_neuroir(str(p))[3] is False


# ---------------------------------------------------------- compiled reference sources
@needs_ref
def test_ref_fft_all_sizes_bitexact():
    o, r = Oracle(), Reference()
    rng = np.random.default_rng(0)
    for H, W in [(2, 2), (4, 8), (8, 64), (32, 32), (128, 128), (256, 16)]:
        x = (rng.standard_normal((H, W)) * 10 ** rng.uniform(-2, 2)).astype(np.float32)
        a, b = o.rfft2(x), r.rfft2(x)
        assert np.array_equal(_bits(a), _bits(b)), (H, W)
        assert np.array_equal(_bits(o.irfft2(a, H, W)), _bits(r.irfft2(a, H, W))), (H, W)


@needs_ref
def test_ref_spectral_conv_linear_gelu_bitexact():
    o, r = Oracle(), Reference()
    rng = np.random.default_rng(1)
    h = rng.standard_normal((2, 16, 32, 16)).astype(np.float32)
    wr = rng.standard_normal((16, 16, 12, 6)).astype(np.float32) / 256
    wi = rng.standard_normal((16, 16, 12, 6)).astype(np.float32) / 256
    assert np.array_equal(_bits(o.spectral_conv2d(h, wr, wi)), _bits(r.spectral_conv2d(h, wr, wi)))
    x = rng.standard_normal((100, 64)).astype(np.float32)
    W = rng.standard_normal((33, 64)).astype(np.float32)
    b = rng.standard_normal(33).astype(np.float32)
    assert np.array_equal(_bits(o.linear(x, W, b)), _bits(r.linear(x, W, b)))
    z = (rng.standard_normal(100000) * 4).astype(np.float32)
    assert np.array_equal(_bits(o.activation(z)), _bits(r.activation(z)))
    assert np.array_equal(_bits(o.activation(z, relu=True)), _bits(r.activation(z, relu=True)))


@needs_ref
def test_ref_linear_every_length_bitexact():
    """The vector-block / fused-tail split of the reference build's Linear, for every
    dot-product length that occurs (in_ch, width, tails)."""
    o, r = Oracle(), Reference()
    rng = np.random.default_rng(5)
    for K in list(range(1, 41)) + [48, 63, 64, 100, 128, 256]:
        x = rng.standard_normal((64, K)).astype(np.float32)
        W = rng.standard_normal((5, K)).astype(np.float32)
        b = rng.standard_normal(5).astype(np.float32)
        assert np.array_equal(_bits(o.linear(x, W, b)), _bits(r.linear(x, W, b))), K


@needs_ref
@pytest.mark.parametrize("variant", ["plain", "per_token", "per_tensor", "padded"])
def test_ref_fno1d_network_bitexact(tmp_path, variant):
    kw = {"plain": dict(quantised=False), "per_token": dict(per_token=True),
          "per_tensor": dict(per_token=False), "padded": dict(per_token=True, pad_factor=32)}[variant]
    n = 16 if variant == "padded" else 64
    m = synth.fno1d_model(7, in_ch=5, width=20, modes=6, L=3, n=n, n_calib=4, **kw)
    p = str(tmp_path / "m.nneuroir")
    ir.write(p, m)
    x = synth.fno1d_inputs(np.random.default_rng(4), 3, n, in_ch=5)
    r, o = Reference(), Oracle()
    for int8 in (False, True):
        want = r.run(p, x, 1, enable_int8=int8)
        assert np.array_equal(_bits(o.fno1d_forward(m, x, int8=int8)), _bits(want)), int8


@needs_ref
@pytest.mark.parametrize("kw", [
    dict(latent=16, n_heads=2, h=6, w=8, n_patches=12, n_layers=2),
    dict(latent=24, n_heads=3, h=5, w=4, n_patches=20, n_layers=1, in_dim=5, out_dim=2),
    dict(latent=16, n_heads=1, h=3, w=7, n_patches=21, n_layers=1),
    dict(latent=32, n_heads=4, h=8, w=16, n_patches=128, n_layers=2)])
def test_ref_tm2d_network_bitexact(tmp_path, kw):
    """Ragged patch counts (the attention-times-V sum's fused tail), pooled patches
    (pp > 1), odd latent widths (LayerNorm and Linear tails)."""
    m = synth.tm2d_model(3, **kw)
    p = str(tmp_path / "m.nneuroir")
    ir.write(p, m)
    x = np.random.default_rng(1).standard_normal(
        (2, kw["h"], kw["w"], kw.get("in_dim", 3))).astype(np.float32)
    want = Reference().run(p, x, kw.get("out_dim", 1), tokenmixer2d=True)
    assert np.array_equal(_bits(Oracle().tm2d_forward(m, x)), _bits(want))


@needs_ref
def test_ref_e4m3_encoder_sweep_bitexact():
    """Every 97th float32 bit pattern (44 M values over all signs, exponents, NaN and
    infinity) and every decode, against the reference header's encoder/decoder."""
    import ctypes as C
    o, r = Oracle(), Reference()
    u = np.arange(0, 1 << 32, 97, dtype=np.uint64).astype(np.uint32)
    f = u.view(np.float32)
    want = np.empty(f.size, np.uint8)
    r.lib.ref_fp32_to_e4m3(f.ctypes.data_as(C.c_void_p), want.ctypes.data_as(C.c_void_p),
                           C.c_int64(f.size))
    assert np.array_equal(o.fp32_to_e4m3(f), want)
    codes = np.arange(256, dtype=np.uint8)
    dec = np.empty(256, np.float32)
    r.lib.ref_e4m3_to_fp32(codes.ctypes.data_as(C.c_void_p), dec.ctypes.data_as(C.c_void_p),
                           C.c_int64(256))
    mine = np.array([o.lib.nfo_e4m3_to_fp32(int(c)) for c in codes], np.float32)
    assert np.array_equal(_bits(mine), _bits(dec))


@needs_ref
@pytest.mark.parametrize("kw", [dict(width=8, modes=(3, 3, 2), L=2, S=8),
                                dict(width=12, modes=(2, 4, 3), L=1, S=16, in_ch=5)])
def test_ref_fno3d_network_bitexact(tmp_path, kw):
    m = synth.fno3d_model(4, n_calib=2, **kw)
    p = str(tmp_path / "m.nneuroir")
    ir.write(p, m)
    x = synth.fno3d_inputs(np.random.default_rng(1), 2, kw["S"], kw.get("in_ch", 4))
    want = Reference().run(p, x, 1)
    o = Oracle()
    assert np.array_equal(_bits(o.fno3d_forward(m, x)), _bits(want))
    # the FP8 variant stays within the E4M3 rounding of the FP32 network
    rel = np.linalg.norm(o.fno3d_forward(m, x, fp8=True) - want) / np.linalg.norm(want)
    assert rel < 0.1


@needs_ref
def test_ref_linear_forward_batched_bitexact():
    o, r = Oracle(), Reference()
    for K, N in [(32, 32), (64, 64), (128, 64), (256, 256)]:
        c = quant.gemm_case(K * 7 + N, 257, K, N)
        A = (np.random.default_rng(K).standard_normal((257, K)) * 2).astype(np.float32)
        qa = quant.tensor_qparams(A)
        for bias in (None, c["bias"]):
            want = r.linear_forward_batched(c["Wq"], c["sW"], c["zW"], c["sum_w"], bias,
                                            qa.scale, qa.zero_point, A)
            got, _, _ = o.linear_forward_batched(c["Wq"], c["sW"], c["zW"], c["sum_w"], bias,
                                                 qa.scale, qa.zero_point, A)
            assert np.array_equal(_bits(got), _bits(want)), (K, N)


@needs_ref
@pytest.mark.parametrize("per_channel", [True, False])
def test_ref_fno2d_network_bitexact(tmp_path, per_channel):
    m = synth.fno2d_model(9, in_ch=5, width=20, mh=5, mw=4, L=3, H=16, W=32, n_calib=2,
                          per_channel=per_channel)
    p = str(tmp_path / "m.nneuroir")
    ir.write(p, m)
    x = synth.fno2d_inputs(np.random.default_rng(3), 2, 16, 32, in_ch=5)
    want = Reference().run(p, x, 1)
    got = Oracle().fno2d_forward(m, x, mode=0)
    assert np.array_equal(_bits(got), _bits(want))


# ------------------------------------------------------------- INT8 composition
def test_int8_mode_close_to_fake_quant_network():
    """The INT8 path differs from the FP32 fake-quant network only by the activation
    quantisation of the layer inputs: outputs agree to a few output steps."""
    m = synth.fno2d_model(4, width=16, mh=4, mw=4, L=2, H=16, W=16, n_calib=2)
    x = synth.fno2d_inputs(np.random.default_rng(8), 2, 16, 16)
    o = Oracle()
    y0 = o.fno2d_forward(m, x, mode=0)
    y1, taps = o.fno2d_forward(m, x, mode=1, taps=True)
    step = m.qparams["proj_out.output"].scale
    assert np.abs(y1 - y0).max() <= 16 * step
    # layer-0 codes are the lift output's codes
    assert taps["codes_in.0"].min() >= -128 and taps["codes_in.0"].max() <= 127
    assert len(np.unique(taps["codes_in.1"])) > 20


# ------------------------------------------ DeepONet, GraphOp, GraphOp2D, TokenMixer
def test_golden_other_op_families():
    """DeepONet, GraphOp, GraphOp2D and TokenMixer models built by the reference's
    PyTorch modules and exported by its exporter; the reference runtime's RunDeepONet /
    RunGraphOp / RunGraphOp2D / RunTokenMixer outputs, every bit.  The Python reader
    sees the weight order the reference loader insists on."""
    d = _g("ops.npz")
    o = Oracle()
    m = ir.read(os.path.join(GOLD, "deeponet.nneuroir"))
    assert m.op == "DeepONet" and list(m.weights) == ir.expected_weight_names(m.op, m.config)
    assert np.array_equal(_bits(o.deeponet_forward(m, d["don_u"], d["don_y"])), _bits(d["don_out"]))
    for name, x, y in (("graphop", "gop_x", "gop_y"), ("graphop2d", "g2_x", "g2_y")):
        m = ir.read(os.path.join(GOLD, name + ".nneuroir"))
        assert list(m.weights) == ir.expected_weight_names(m.op, m.config)
        assert np.array_equal(_bits(o.graphop_forward(m, d[x])), _bits(d[y]))
    m = ir.read(os.path.join(GOLD, "tokenmixer.nneuroir"))
    assert m.op == "TokenMixer" and list(m.weights) == ir.expected_weight_names(m.op, m.config)
    assert np.array_equal(_bits(o.tokenmixer_forward(m, d["tk_x"])), _bits(d["tk_y"]))


@needs_ref
@pytest.mark.parametrize("act", ["relu", "gelu"])
@pytest.mark.parametrize("kw", [
    dict(),
    dict(in_branch=3, in_trunk=2, latent=45, out_ch=3, hidden_branch=48, hidden_trunk=72,
         n_branch=2, n_trunk=4),
    dict(latent=7, n_branch=1, n_trunk=1, out_ch=2)])
def test_ref_deeponet_bitexact(tmp_path, act, kw):
    """Latent widths with an unfused-only (32), mixed (45) and fused-only (7) dot
    product; one-layer nets (no hidden width)."""
    m = synth.deeponet_model(1, activation=act, **kw)
    p = str(tmp_path / "d.nneuroir")
    ir.write(p, m)
    u, y = synth.deeponet_inputs(np.random.default_rng(2), 3, 37, 53, m.config["in_branch"],
                                 m.config["in_trunk"])
    want = Reference().run_deeponet(p, u, y, m.config["out_channels"])
    assert np.array_equal(_bits(Oracle().deeponet_forward(m, u, y)), _bits(want))


@needs_ref
@pytest.mark.parametrize("act", ["relu", "gelu"])
@pytest.mark.parametrize("kw", [
    dict(), dict(in_dim=3, out_dim=2, hidden=40, n_layers=3, n_nodes=100),
    dict(h=16, w=16), dict(in_dim=2, out_dim=3, hidden=64, n_layers=2, h=8, w=32)])
def test_ref_graphop_bitexact(tmp_path, act, kw):
    m = synth.graphop_model(3, activation=act, **kw)
    p = str(tmp_path / "g.nneuroir")
    ir.write(p, m)
    shape = (2, kw["h"], kw["w"]) if "h" in kw else (2, m.config["n_nodes"])
    x = np.random.default_rng(4).standard_normal(shape + (m.config["in_dim"],)).astype(np.float32)
    want = Reference().run_other(p, m.op, x, m.config["out_dim"])
    assert np.array_equal(_bits(Oracle().graphop_forward(m, x)), _bits(want))


@needs_ref
@pytest.mark.parametrize("act", ["relu", "gelu"])
def test_ref_tokenmixer_bitexact(tmp_path, act):
    """The 1D TokenMixer is the TokenMixer2D network on n_points points."""
    m = synth.tokenmixer_model(7, activation=act, n_points=256, n_patches=32, latent=32,
                               n_heads=2, n_layers=2)
    m.quant_enabled = False
    p = str(tmp_path / "t.nneuroir")
    ir.write(p, m)
    x = np.random.default_rng(8).standard_normal((2, 256, 2)).astype(np.float32)
    want = Reference().run_other(p, "TokenMixer", x, 1)
    assert np.array_equal(_bits(Oracle().tokenmixer_forward(m, x)), _bits(want))
