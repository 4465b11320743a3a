"""Host logic of the batch partition across GPUs, on CPU.

A batch of B samples on G GPUs runs as contiguous slices of ceil(B / G) samples
(nfx_batch_slice, the rule nfx_group_* and nfx_runtime_run_sharded* use); the outputs
are gathered back in rank order.  The gloo test runs that partition as two ranks, each
computing its slice with the CPU restatement, gathers the slices (to every rank, and to
a root) and checks the reassembled batch against one run over the whole batch."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("B,G", [(256, 8), (256, 2), (5, 2), (3, 4), (1, 8), (0, 2), (257, 8)])
def test_batch_slices_partition_the_batch(B, G):
    from neuroflow_b200 import _nfx
    per = -(-B // G) if B else 0
    nxt = 0
    for r in range(G):
        b0, nb = _nfx.batch_slice(B, G, r)
        assert b0 == min(B, r * per) and 0 <= nb <= per
        if nb:
            assert b0 == nxt
        nxt = b0 + nb
    assert nxt == B


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, path, x, out):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from neuroflow_b200 import _nfx, ir
    from oracle.cpu import Oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=60))
    try:
        m = ir.read(path)
        b0, nb = _nfx.batch_slice(len(x), ws, rank)
        mine = Oracle().fno2d_forward(m, x[b0:b0 + nb], mode=1) if nb else None
        every = [None] * ws
        dist.all_gather_object(every, (b0, mine))          # root < 0: every rank gets y
        at_root = [None] * ws if rank == 0 else None
        dist.gather_object((b0, mine), at_root, dst=0)      # root 0
        def assemble(parts):
            parts = [p for p in parts if p[1] is not None]
            parts.sort(key=lambda p: p[0])
            return np.concatenate([p[1] for p in parts])
        out.put((rank, assemble(every), assemble(at_root) if rank == 0 else None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [5, 4])
def test_sharded_slices_gathered_equal_whole_batch_gloo(tmp_path, B):
    import torch.multiprocessing as mp
    from neuroflow_b200 import ir, synth
    from oracle.cpu import Oracle
    m = synth.fno2d_model(6, width=16, mh=4, mw=4, L=2, H=16, W=16, n_calib=2, calib_chunk=2)
    path = str(tmp_path / "m.nneuroir")
    ir.write(path, m)
    x = synth.fno2d_inputs(np.random.default_rng(B), B, 16, 16)
    want = Oracle().fno2d_forward(m, x, mode=1)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, path, x, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted((q.get(timeout=120) for _ in range(2)), key=lambda t: t[0])
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    for rank, every, at_root in got:
        assert np.array_equal(every, want)
        if rank == 0:
            assert np.array_equal(at_root, want)
