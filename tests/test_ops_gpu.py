"""DeepONet, GraphOp, GraphOp2D and TokenMixer on the GPU runtime (the reference's
RunDeepONet / RunGraphOp / RunGraphOp2D / RunTokenMixer, runtime.cpp:103-153, on
DeepONet::Forward fno.cpp:1289-1406, GraphOp::Forward :1653-1741, GraphOp2D::Forward
:1969-2060 and TokenMixer::Forward :1460-1644).

ReLU networks are bit-identical to the CPU restatement (pinned bit-exact to the
reference runtime).  GELU networks differ only by CUDA's tanhf against glibc's (a few
ulps per activation): rtol 1e-5 of the reference's outputs, including those of models
that the reference's own PyTorch modules built and its exporter wrote."""
import os
import subprocess

import numpy as np
import pytest

from neuroflow_b200 import ir, synth
from oracle.cpu import Oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "neuroflow_b200")


def _close(got, want):
    return np.allclose(got, want, rtol=1e-5, atol=1e-6 * float(np.abs(want).max()))


def _write(tmp_path, m, name="m.nneuroir"):
    p = str(tmp_path / name)
    ir.write(p, m)
    return p


@pytest.mark.gpu
def test_reference_exported_models_match_the_reference_runtime():
    """tests/golden: built by the reference's PyTorch modules (GELU), exported by its
    exporter, outputs of the reference C++ runtime."""
    import neuroflow_cpp
    d = np.load(os.path.join(GOLD, "ops.npz"))
    got = neuroflow_cpp.infer_deeponet_arrays(os.path.join(GOLD, "deeponet.nneuroir"), d["don_u"], d["don_y"])
    assert got.shape == d["don_out"].shape and _close(got, d["don_out"])
    for name, x, y in (("graphop", "gop_x", "gop_y"), ("graphop2d", "g2_x", "g2_y"),
                       ("tokenmixer", "tk_x", "tk_y")):
        got = neuroflow_cpp.infer_arrays(os.path.join(GOLD, name + ".nneuroir"), d[x])
        assert got.shape == d[y].shape and _close(got, d[y]), name


@pytest.mark.gpu
@pytest.mark.parametrize("act", ["relu", "gelu"])
@pytest.mark.parametrize("kw,B,ns,nq", [
    (dict(), 4, 100, 200),
    (dict(in_branch=3, in_trunk=2, latent=45, out_ch=3, hidden_branch=48, hidden_trunk=72,
          n_branch=2, n_trunk=4), 3, 37, 53),
    (dict(latent=7, n_branch=1, n_trunk=1, out_ch=2), 2, 5, 300),
    (dict(latent=128, out_ch=3, hidden_branch=256, hidden_trunk=128), 2, 64, 130),  # 384-wide branch output
])
def test_deeponet_matches_oracle(tmp_path, act, kw, B, ns, nq):
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.deeponet_model(5, activation=act, **kw)
    p = _write(tmp_path, m)
    u, y = synth.deeponet_inputs(np.random.default_rng(6), B, ns, nq, m.config["in_branch"],
                                 m.config["in_trunk"])
    want = Oracle().deeponet_forward(m, u, y)
    got = np.zeros_like(want)
    InferenceRuntime(p).run_deeponet(u, y, got)
    if act == "relu":
        assert np.array_equal(got, want)
    else:
        assert _close(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("act", ["relu", "gelu"])
@pytest.mark.parametrize("kw,B", [
    (dict(), 3), (dict(in_dim=3, out_dim=2, hidden=40, n_layers=3, n_nodes=100), 2),
    (dict(h=16, w=16), 2), (dict(in_dim=2, out_dim=3, hidden=64, n_layers=2, h=8, w=32), 3),
    (dict(hidden=256, n_layers=2, h=12, w=20), 2), (dict(hidden=130, n_layers=1, h=16, w=16), 1),
])
def test_graphop_matches_oracle(tmp_path, act, kw, B):
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.graphop_model(9, activation=act, **kw)
    p = _write(tmp_path, m)
    shape = (B, kw["h"], kw["w"]) if "h" in kw else (B, m.config["n_nodes"])
    x = np.random.default_rng(10).standard_normal(shape + (m.config["in_dim"],)).astype(np.float32)
    want = Oracle().graphop_forward(m, x)
    got = np.zeros_like(want)
    rt = InferenceRuntime(p)
    (rt.run_graphop2d if m.op == "GraphOp2D" else rt.run_graphop)(x, got)
    if act == "relu":
        assert np.array_equal(got, want)
    else:
        assert _close(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("act", ["relu", "gelu"])
def test_tokenmixer_matches_oracle(tmp_path, act):
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.tokenmixer_model(7, activation=act, n_points=1024, n_patches=64, latent=64,
                               n_heads=2, n_layers=2)
    p = _write(tmp_path, m)
    x = np.random.default_rng(8).standard_normal((3, 1024, 2)).astype(np.float32)
    want = Oracle().tokenmixer_forward(m, x)
    got = np.zeros_like(want)
    InferenceRuntime(p).run_tokenmixer(x, got)
    assert _close(got, want)


@pytest.mark.gpu
def test_device_variants_equal_host_variants(tmp_path):
    import torch
    from neuroflow_b200.runtime import InferenceRuntime
    m = synth.deeponet_model(2, latent=32, out_ch=2)
    rt = InferenceRuntime(_write(tmp_path, m, "d.nneuroir"))
    u, y = synth.deeponet_inputs(np.random.default_rng(1), 3, 50, 70)
    host = np.zeros((3, 70, 2), np.float32)
    rt.run_deeponet(u, y, host)
    dout = torch.empty((3, 70, 2), device="cuda")
    rt.run_deeponet_device(torch.from_numpy(u).cuda(), torch.from_numpy(y).cuda(), dout)
    torch.cuda.synchronize()
    assert np.array_equal(dout.cpu().numpy(), host)
    g = synth.graphop_model(3, h=8, w=8, hidden=32, n_layers=2)
    rt = InferenceRuntime(_write(tmp_path, g, "g.nneuroir"))
    x = np.random.default_rng(2).standard_normal((2, 8, 8, 1)).astype(np.float32)
    host = np.zeros((2, 8, 8, 1), np.float32)
    rt.run_graphop2d(x, host)
    dy = torch.empty((2, 8, 8, 1), device="cuda")
    rt.run_other_device("graphop2d", torch.from_numpy(x).cuda(), dy)
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy(), host)


@pytest.mark.gpu
def test_errors_follow_the_reference(tmp_path):
    from neuroflow_b200.runtime import InferenceRuntime
    d = synth.deeponet_model(1, latent=8, out_ch=1)
    rt = InferenceRuntime(_write(tmp_path, d, "d.nneuroir"))
    u = np.zeros((2, 5, 1), np.float32)
    y = np.zeros((2, 6, 1), np.float32)
    for (uu, yy, oo, msg) in (
            (u[0], y, np.zeros((2, 6, 1), np.float32), "expected 3D u"),
            (u, y[0], np.zeros((2, 6, 1), np.float32), "expected 3D y"),
            (np.zeros((2, 5, 2), np.float32), y, np.zeros((2, 6, 1), np.float32), "branch feature dim"),
            (u, np.zeros((2, 6, 3), np.float32), np.zeros((2, 6, 1), np.float32), "trunk feature dim"),
            (u, y, np.zeros((2, 7, 1), np.float32), "output buffer shape mismatch"),
            (u, np.zeros((3, 6, 1), np.float32), np.zeros((2, 6, 1), np.float32), "batch sizes differ")):
        with pytest.raises(RuntimeError, match=msg):
            rt.run_deeponet(uu, yy, oo)
    with pytest.raises(RuntimeError, match="GraphOp not initialized"):
        rt.run_graphop(np.zeros((1, 4, 1), np.float32), np.zeros((1, 4, 1), np.float32))
    with pytest.raises(RuntimeError, match="runtime does not support op: DeepONet"):
        rt.run(np.zeros((1, 4, 1), np.float32), np.zeros((1, 4, 1), np.float32))
    g = synth.graphop_model(1, h=4, w=4)
    rt = InferenceRuntime(_write(tmp_path, g, "g.nneuroir"))
    with pytest.raises(RuntimeError, match="GraphOp2D: h / w mismatch"):
        rt.run_graphop2d(np.zeros((1, 4, 5, 1), np.float32), np.zeros((1, 4, 5, 1), np.float32))
    with pytest.raises(RuntimeError, match="GraphOp2D: expected 4D x"):
        rt.run_graphop2d(np.zeros((1, 16, 1), np.float32), np.zeros((1, 16, 1), np.float32))
    with pytest.raises(RuntimeError, match="DeepONet not initialized"):
        rt.run_deeponet(u, y, np.zeros((2, 6, 1), np.float32))
    # a graph index outside the node range: refused (the reference reads out of bounds)
    g.weights["graph.adj_indices"] = g.weights["graph.adj_indices"].copy()
    g.weights["graph.adj_indices"][5] = 16.0
    rt = InferenceRuntime(_write(tmp_path, g, "bad.nneuroir"))
    with pytest.raises(RuntimeError, match="adjacency offsets or indices out of range"):
        rt.run_graphop2d(np.zeros((1, 4, 4, 1), np.float32), np.zeros((1, 4, 4, 1), np.float32))
    t = synth.tokenmixer_model(1, n_points=64, n_patches=16, latent=16, n_heads=2, n_layers=1)
    rt = InferenceRuntime(_write(tmp_path, t, "t.nneuroir"))
    with pytest.raises(RuntimeError, match="TokenMixer: n_points mismatch"):
        rt.run_tokenmixer(np.zeros((1, 32, 2), np.float32), np.zeros((1, 32, 1), np.float32))
    with pytest.raises(RuntimeError, match="TokenMixer2D not initialized"):
        rt.run_tokenmixer2d(np.zeros((1, 8, 8, 2), np.float32), np.zeros((1, 8, 8, 1), np.float32))


@pytest.mark.gpu
def test_cli_and_infer_run_the_other_ops(tmp_path):
    """nflow_infer and `infer` dispatch GraphOp2D and TokenMixer models to their Run
    calls as the reference's `infer` does (pybind_module.cpp:95-105)."""
    import neuroflow_cpp
    d = np.load(os.path.join(GOLD, "ops.npz"))
    for name, x in (("graphop2d", "g2_x"), ("tokenmixer", "tk_x"), ("graphop", "gop_x")):
        path = os.path.join(GOLD, name + ".nneuroir")
        want = neuroflow_cpp.infer_arrays(path, d[x])
        xin, yout = str(tmp_path / "x.npy"), str(tmp_path / "y.npy")
        np.save(xin, d[x])
        assert neuroflow_cpp.infer(path, xin, yout) == "ok"
        assert np.array_equal(np.load(yout), want)
        r = subprocess.run([os.path.join(PKG, "nflow_infer"), "--model", path, "--input", xin,
                            "--output", yout], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        assert np.array_equal(np.load(yout), want)
