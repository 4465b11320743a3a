"""Batch partitioned across two GPUs, against one GPU running the whole batch
(needs 2 GPUs; skipped on a one-GPU machine).

* RuntimeGroup (one process, nfx_group_*): host-buffer Run (each device copies its own
  slice) and device-buffer Run (NCCL scatter of the inputs, gather of the outputs into
  the first device's buffer), even and uneven batches.
* run_sharded (one process per GPU, nfx_runtime_run_sharded*): all-gather to every rank
  and gather to a root, device and host buffers.
Every result must be bit-identical to the single-GPU run: the slices run the same
kernels on the same samples."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _two_gpus():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.device_count() >= 2
    except Exception:
        return False


needs2 = pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")


def _model(tmp_path, H=32, W=32):
    from neuroflow_b200 import ir, synth
    m = synth.fno2d_model(8, width=64, mh=12, mw=12, L=2, H=H, W=W, n_calib=2, calib_chunk=2)
    p = os.path.join(str(tmp_path), "m.nneuroir")
    ir.write(p, m)
    return m, p


@pytest.mark.gpu
@needs2
@pytest.mark.parametrize("B", [5, 8])
def test_group_matches_one_gpu(tmp_path, B):
    import torch
    from neuroflow_b200 import synth
    from neuroflow_b200.runtime import InferenceRuntime, RuntimeGroup
    m, p = _model(tmp_path)
    x = synth.fno2d_inputs(np.random.default_rng(B), B, 32, 32)
    one = InferenceRuntime(p, 0)
    one.enable_int8_gemm()
    want = np.zeros((B, 32, 32, 1), np.float32)
    one.run(x, want)
    g = RuntimeGroup(p, [0, 1])
    g.enable_int8_gemm()
    assert g.is_int8_gemm_enabled()
    got = np.full_like(want, np.nan)
    g.run(x, got)
    assert np.array_equal(got, want)
    torch.cuda.set_device(0)
    dx = torch.from_numpy(x).cuda(0)
    dy = torch.full((B, 32, 32, 1), float("nan"), device="cuda:0")
    for _ in range(2):
        g.run_device(dx, dy)
        torch.cuda.synchronize(0)
        g.check()
        assert np.array_equal(dy.cpu().numpy(), want)
    g.close()


def _rank_main(rank, path, x, uid_q, out_q):
    import torch
    sys.path.insert(0, ROOT)
    from neuroflow_b200.runtime import Comm, InferenceRuntime, comm_unique_id
    try:
        torch.cuda.set_device(rank)
        rt = InferenceRuntime(path, rank)
        rt.enable_int8_gemm()
        if rank == 0:
            uid = comm_unique_id()
            uid_q.put(uid)             # for rank 1
        else:
            uid = uid_q.get(timeout=120)
        comm = Comm(uid, 2, rank, rank)
        B = x.shape[0]
        dx = torch.from_numpy(x).cuda(rank)
        res = {}
        for root in (-1, 0):
            dy = torch.full((B,) + x.shape[1:3] + (1,), float("nan"), device=f"cuda:{rank}")
            rt.run_sharded(comm, dx, dy, root=root)
            torch.cuda.synchronize(rank)
            rt.check()
            res[f"dev{root}"] = dy.cpu().numpy()
            yh = np.full((B,) + x.shape[1:3] + (1,), np.nan, np.float32)
            rt.run_sharded_host(comm, x, yh, root=root)
            res[f"host{root}"] = yh
        comm.close()
        out_q.put((rank, res, None))
    except Exception as e:  # report instead of hanging the other rank's join
        out_q.put((rank, None, repr(e)))


@pytest.mark.gpu
@needs2
@pytest.mark.parametrize("B", [5, 6])
def test_sharded_two_processes_match_one_gpu(tmp_path, B):
    import torch.multiprocessing as mp
    from neuroflow_b200 import synth
    from neuroflow_b200.runtime import InferenceRuntime
    m, p = _model(tmp_path)
    x = synth.fno2d_inputs(np.random.default_rng(40 + B), B, 32, 32)
    one = InferenceRuntime(p, 0)
    one.enable_int8_gemm()
    want = np.zeros((B, 32, 32, 1), np.float32)
    one.run(x, want)
    one.close()
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, p, x, uid_q, out_q)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = {}
    try:
        for _ in range(2):
            rank, res, err = out_q.get(timeout=240)
            assert err is None, f"rank {rank}: {err}"
            results[rank] = res
    finally:
        for pr in procs:
            pr.join(60)
            if pr.is_alive():
                pr.kill()
    from neuroflow_b200 import _nfx
    for rank in (0, 1):
        res = results[rank]
        assert np.array_equal(res["dev-1"], want) and np.array_equal(res["host-1"], want)
        b0, nb = _nfx.batch_slice(B, 2, rank)
        if rank == 0:
            assert np.array_equal(res["dev0"], want) and np.array_equal(res["host0"], want)
        else:   # a non-root rank's device y holds its own slice; its host y is untouched
            assert np.array_equal(res["dev0"][b0:b0 + nb], want[b0:b0 + nb])
            assert np.isnan(res["host0"]).all()
