"""Benchmark: FNO2d INT8 inference on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nfx|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one process per GPU)

One step = one forward pass of the FNO2d INT8 executor over the global batch of 256
samples (128x128 grid, 3 input channels, width 64, 12x12 modes, 4 layers, out_ch 1).
At N > 1 the batch is partitioned across the ranks (strong scaling): every rank holds
the whole batch, computes its contiguous slice of ceil(256 / N) samples with replicated
weights, and NCCL all-gathers the fp32 outputs into every rank's buffer inside the
timed region (InferenceRuntime.run_sharded).  The weak-scaling rate (every rank its own
256 samples, no collective) is reported as "weak_scaling".  Inputs are seeded synthetic
Gaussian random fields; weights are random-init and calibrated on a separate 32-sample
batch (no dataset or checkpoint is available offline).  The per-step working set at
256 samples per GPU (268 MB of int8 codes per layer boundary + 50 MB of input) is
larger than the 126 MB L2, so no L2 flush is needed between steps; at N = 8 (32
samples per GPU, 34 MB of codes) the slice fits in L2, which the line states.

`value`: samples/s of the whole job with inputs resident in HBM, device-timed with
CUDA events, max over ranks.  `e2e`: the same metric through the public host-buffer
API (pinned host x -> device -> host y every step; at N > 1 run_sharded_host, each
rank copying its input slice in and rank 0 copying the gathered outputs out).
`--impl reference`: the reference's own CPU runtime (compiled from its sources into
oracle/_ref) on all host cores, one InferenceRuntime per thread.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(in_channels=3, out_channels=1, width=64, modes_h=12, modes_w=12, n_layers=4,
           H=128, W=128, batch=256, n_calib=32)
METRIC = "FNO2d INT8 samples/s"
UNIT = "samples/s"
WORKLOAD = "configs[2] FNO2d INT8 per-channel, 128x128, width 64, 12x12 modes, 4 layers"
# algorithmic bytes per sample of the whole network (int8 codes at each layer boundary,
# read twice per layer, written once; fp32 input and output): 16 P + 14 P C
P = CFG["H"] * CFG["W"]
BYTES_PER_SAMPLE = 16 * P + 14 * P * CFG["width"]


def model_path(seed: int = 0) -> str:
    from neuroflow_b200 import ir, synth
    key = hashlib.sha1(json.dumps([CFG, seed, "v1"], sort_keys=True).encode()).hexdigest()[:12]
    path = os.path.join(tempfile.gettempdir(), f"nfx_bench_fno2d_{key}.nneuroir")
    if not os.path.exists(path):
        m = synth.fno2d_model(seed, in_ch=CFG["in_channels"], out_ch=CFG["out_channels"],
                              width=CFG["width"], mh=CFG["modes_h"], mw=CFG["modes_w"],
                              L=CFG["n_layers"], H=CFG["H"], W=CFG["W"], n_calib=CFG["n_calib"])
        tmp = path + f".{os.getpid()}"
        ir.write(tmp, m)
        os.replace(tmp, path)
    return path


def inputs(seed: int, n: int) -> np.ndarray:
    from neuroflow_b200 import synth
    return synth.fno2d_inputs(np.random.default_rng(seed), n, CFG["H"], CFG["W"],
                              CFG["in_channels"])


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def max_over_ranks(x: float, ws: int, device) -> float:
    """The largest of the ranks' values (a time), on every rank; x itself for one rank.
    `device` holds the one-element tensor of the reduction (a GPU for NCCL, the CPU
    for gloo)."""
    if ws <= 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(ws: int, batch_per_rank: int, steps: int, seconds: float) -> float:
    """Whole-job samples/s: every rank ran `steps` steps of its own batch in at most
    `seconds` (weak scaling)."""
    return ws * batch_per_rank * steps / seconds


def cpu_reference(path: str, x: np.ndarray, nthreads: int, target_s: float = 8.0):
    """Reference runtime on the host cores: returns (samples/s, sample description)."""
    from oracle.cpu import Reference
    ref = Reference()
    t1 = ref.bench(path, x[:1], CFG["out_channels"], 1, 1)          # one sample, one thread
    reps = max(1, int(round(target_s / max(t1, 1e-3))))
    n = min(len(x), nthreads)
    wall = ref.bench(path, x[:n], CFG["out_channels"], n, reps)
    return n * reps / wall, n, reps, t1


def gemm_rows(device, Ms, Ks):
    """configs[1] GEMM cases: achieved GB/s of nfx_int8_gemm (bias and bias + GELU).
    Each case rotates over enough distinct A / C buffers that every launch reads and
    writes memory outside L2 (> 256 MB per rotation), and replays its launches from a
    CUDA graph (device time per launch, CUDA events)."""
    import torch
    from neuroflow_b200 import _nfx, quant
    hbm, src = peaks()
    rows = []
    for M in Ms:
        for K in Ks:
            N = K
            c = quant.gemm_case(K, 4096, K, N)  # weights + qparams
            t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device)
                 for k, v in c.items() if k in ("Wq", "sW", "zW", "sum_w", "bias")}
            per_call = M * K + 4 * M * N + 8 * M
            nbuf = max(1, min(512, -(-(256 << 20) // per_call)))
            rng = np.random.default_rng(K + M)
            bufs = []
            for _ in range(nbuf):
                A = torch.from_numpy(rng.integers(-128, 128, (M, K), dtype=np.int8)).to(device)
                sA = torch.from_numpy(rng.uniform(0.005, 0.02, M).astype(np.float32)).to(device)
                zA = torch.from_numpy(rng.integers(-20, 20, M).astype(np.int32)).to(device)
                bufs.append((A, sA, zA, torch.empty((M, N), dtype=torch.float32, device=device)))
            reps = max(20, min(2000, int(2.5e9 // per_call)))
            for act in (0, 1):
                def call(i):
                    A, sA, zA, C_ = bufs[i % nbuf]
                    _nfx.int8_gemm(A, t["Wq"], t["sW"], t["zW"], t["sum_w"], bias=t["bias"],
                                   scale_a=sA, zp_a=zA, act=act, out=C_)
                for i in range(max(3, nbuf)):
                    call(i)
                torch.cuda.synchronize()
                # the launches are replayed from a CUDA graph, so that small M measures
                # the GPU and not the host's launch rate
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for i in range(reps):
                        call(i)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) / reps * 1e3
                del g
                byts = M * K + N * K + 4 * M * N + 16 * N + 8 * M
                gbs = byts / (us * 1e-6) / 1e9
                rows.append({"M": M, "K": K, "N": N, "epilogue": "bias+GELU" if act else "bias",
                             "us": round(us, 2), "GBps": round(gbs, 1),
                             "frac": round(gbs / hbm, 3), "buffers": nbuf})
            del bufs
            torch.cuda.empty_cache()
    return rows


def run_gemm(args):
    """the standalone INT8 GEMM of the local 1x1 layer over the whole sweep
    (M in {4096, 65536, 1048576}, K = N in {32, 64, 128, 256}, bias and bias + GELU
    epilogues), one JSON line."""
    import torch
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    hbm, src = peaks()
    rows = gemm_rows(device, [args.gemm_m] if args.gemm_m else (4096, 65536, 1 << 20),
                     [args.gemm_k] if args.gemm_k else (32, 64, 128, 256))
    big = [r for r in rows if r["M"] == max(x["M"] for x in rows) and r["epilogue"] == "bias"]
    line = {"metric": "INT8 GEMM HBM GB/s (configs[1], largest M, bias epilogue, mean over K = N)",
            "value": round(float(np.mean([r["GBps"] for r in big])), 1), "unit": "GB/s",
            "n_gpus": 1, "higher_is_better": True, "dtype": "int8", "data": "synthetic",
            "peak": hbm, "peak_source": src,
            "config": {"workload": "configs[1] INT8 GEMM sweep (algorithmic bytes: A + W + "
                                   "fp32 C + per-channel and per-row qparams)"},
            "sweep": rows}
    print(json.dumps(line), flush=True)


def make_comm(ws: int, rank: int, local: int):
    """The library's NCCL communicator for the sharded Run (None for one rank): rank 0
    makes the unique id, the process group's broadcast hands it to the others."""
    if ws <= 1:
        return None
    import torch.distributed as dist
    from neuroflow_b200.runtime import Comm, comm_unique_id
    box = [comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return Comm(box[0], ws, rank, local)


def run_nfx(args, ws, rank, local):
    """One step = the forward of the global batch (configs[2]: 256 samples).  At N > 1
    the batch is partitioned: every rank holds the whole input batch, computes its
    contiguous slice of ceil(256 / N) samples and the outputs are all-gathered with NCCL
    into every rank's y inside the timed region (strong scaling); the weak-scaling rate
    (every rank its own 256 samples, no collective) is reported beside it."""
    import torch
    from neuroflow_b200 import _nfx
    from neuroflow_b200.runtime import InferenceRuntime

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B = args.batch                       # global batch
    path = model_path(0)
    x_host = inputs(100, B)              # the same batch on every rank
    rt = InferenceRuntime(path, local)
    rt.enable_int8_gemm()
    if not rt.is_int8_gemm_enabled():
        raise RuntimeError("INT8 path not enabled for the bench model")
    comm = make_comm(ws, rank, local)
    b0, nb = _nfx.batch_slice(B, ws, rank)
    dx = torch.from_numpy(x_host).to(device)
    dy = torch.empty((B, CFG["H"], CFG["W"], CFG["out_channels"]), dtype=torch.float32,
                     device=device)
    stream = torch.cuda.Stream(device)
    if ws > 1:
        import torch.distributed as dist

    def step():
        if comm is None:
            rt.run_device(dx, dy, stream)
        else:
            rt.run_sharded(comm, dx, dy, -1, stream)

    # a slice whose per-step working set fits in the 126 MB L2 (32 samples per GPU at
    # N = 8: 34 MB of codes per layer boundary) gets an L2 flush between timed steps
    # (a 256 MB write, outside the timed intervals: each step is timed by its own pair
    # of events and the intervals are summed)
    flush = None
    if nb * P * CFG["width"] * 2 < 256 << 20:
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def timed(fn, steps):
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if flush is None:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            return e0.elapsed_time(e1)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for a, b in ev:
            with torch.cuda.stream(stream):
                flush.zero_()
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    rt.check()

    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        # keep the GPU busy while the clock sampler starts (untimed, like the warm-up;
        # the same count on every rank)
        for _ in range(args.preheat):
            step()
        torch.cuda.synchronize()
        rt.profile(True)
        ms = timed(step, args.steps)
    if ws > 1:
        dist.barrier()
    prof = rt.profile_read()
    rt.profile(False)
    rt.check()
    ms = max_over_ranks(ms, ws, device)
    value = B * args.steps / (ms * 1e-3)

    weak = None
    if ws > 1:
        # every rank its own full batch, no collective (the previous bench line)
        def own():
            rt.run_device(dx, dy, stream)
        for _ in range(args.warmup):
            own()
        wms = max_over_ranks(timed(own, args.steps), ws, device)
        weak = {"value": round(job_rate(ws, B, args.steps, wms * 1e-3), 1), "unit": UNIT,
                "batch_per_gpu": B, "ms_per_step": round(wms / args.steps, 3)}
        rt.check()

    # end to end through the host-buffer API (pinned host memory): the whole batch in,
    # the whole output back (at N > 1 each rank copies its input slice in, the outputs
    # are gathered to rank 0, which copies them out)
    xp = torch.from_numpy(x_host).pin_memory()
    yp = torch.empty(tuple(dy.shape), dtype=torch.float32).pin_memory()
    xn, yn = xp.numpy(), yp.numpy()
    e2e_steps = 0 if args.no_e2e else max(3, args.steps // 2)

    def e2e_step():
        if comm is None:
            rt.run(xn, yn)
        else:
            rt.run_sharded_host(comm, xn, yn, 0)
    for _ in range(max(1, args.warmup) if e2e_steps else 0):
        e2e_step()
    if ws > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = max(time.perf_counter() - t0, 1e-9)
    e2e_s = max_over_ranks(e2e_s, ws, device)
    e2e = B * e2e_steps / e2e_s if e2e_steps else None

    # the same with ordinary (pageable) numpy buffers, which the runtime stages through
    # its own pinned memory (one GPU)
    e2e_pageable = None
    if e2e_steps and ws == 1:
        xq = np.ascontiguousarray(x_host)
        yq = np.zeros(tuple(dy.shape), np.float32)
        for _ in range(max(1, args.warmup)):
            rt.run(xq, yq)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            rt.run(xq, yq)
        e2e_pageable = B * e2e_steps / max(time.perf_counter() - t0, 1e-9)

    result = None
    if rank == 0:
        hbm, src = peaks()
        # dominant kernel of the step (rank 0's launches over its slice)
        top = max(prof.items(), key=lambda kv: kv[1][1])
        name, (launches, tot_ms) = top
        per_launch_s = tot_ms / launches * 1e-3
        M = nb * P
        C = CFG["width"]
        alg = {  # algorithmic bytes per launch of each kernel
            "fno2d_layer": 2 * M * C,                      # codes in + codes out
            "fno2d_spec_fwd": M * C,                       # codes in
            "fno2d_proj": M * C + 4 * M * CFG["out_channels"],
            "fno2d_lift": 4 * M * CFG["in_channels"] + M * C,
            "fno2d_spec_mix": 0,
        }[name]
        achieved = alg / per_launch_s / 1e9
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            tj = json.load(open(tp))
            t = tj.get("bytes_per_launch", {}).get(name)
            if t is not None:
                traffic = int(t * nb / tj.get("batch", nb))
        share = {k: round(v[1] / sum(vv[1] for vv in prof.values()), 3) for k, v in prof.items()}
        total_launches = sum(v[0] for v in prof.values())
        result = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": B, "batch_per_gpu": nb,
                       "grid": [CFG["H"], CFG["W"]], "in_channels": CFG["in_channels"],
                       "out_channels": CFG["out_channels"], "width": C, "modes": [12, 12],
                       "n_layers": CFG["n_layers"],
                       "parallelism": f"batch x{ws}" + (", NCCL all-gather of the outputs"
                                                        if ws > 1 else ""),
                       "l2": ("working set > L2 (268 MB codes per layer boundary at 256 "
                              "samples)") if flush is None else
                             "L2 flushed between timed steps (256 MB write, untimed)"},
            "e2e": {"value": round(e2e, 1) if e2e else None, "unit": UNIT,
                    "h2d_bytes_per_step": int(x_host.nbytes), "d2h_bytes_per_step": int(4 * B * P),
                    "host_buffers": "pinned",
                    "pageable_value": round(e2e_pageable, 1) if e2e_pageable else None},
            "roofline": {"bound": "hbm", "kernel": name, "achieved": round(achieved, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 3),
                         "peak_source": src, "traffic": traffic,
                         "algorithmic_bytes_per_launch": alg,
                         "launch_us": round(per_launch_s * 1e6, 1)},
            "network_roofline": {"bytes_per_sample": BYTES_PER_SAMPLE,
                                 "achieved_GBps": round(value / ws * BYTES_PER_SAMPLE / 1e9, 1),
                                 "frac": round(value / ws * BYTES_PER_SAMPLE / 1e9 / hbm, 3)},
            "kernel_share": share,
            "gpu_launches": total_launches,
            "clocks": clk.summary(),
        }
        if weak is not None:
            result["weak_scaling"] = weak
    if comm is not None:
        if ws > 1:
            dist.barrier()
        comm.close()
    return result, rt, x_host, path


# Other BASELINE configurations, timed the same way (device-resident inputs, CUDA
# events on the launch stream) for the per-config numbers; not the driver's line.
AUX = {
    "fno1d": dict(metric="FNO1d samples/s", op="FNO1d", batch=64,
                  workload="configs[0] FNO1d, n=1024, width 64, 16 modes, 4 layers, per-channel "
                           "weights, per-token activations (the reference runs its FP32 Linear "
                           "with per-token fake-quant for this IR; EnableInt8Gemm declines)"),
    "fno1d_int8": dict(metric="FNO1d INT8 samples/s", op="FNO1d", batch=64,
                       workload="configs[0] geometry with per-tensor activations: the reference's "
                                "INT8 LinearForwardBatched dispatch (EnableInt8Gemm)",
                       # 12 P + 14 P C with P = 1024, C = 64
                       bytes_per_sample=12 * 1024 + 14 * 1024 * 64),
    "fno2d_fp32": dict(metric="FNO2d FP32 fake-quant samples/s", op="FNO2d", batch=256,
                       workload="configs[2] geometry without EnableInt8Gemm: the reference FNO2d "
                                "Run (fp32 with fake-quant at the four .output boundaries)"),
    "fno3d": dict(metric="FNO3d FP32 samples/s", op="FNO3d", batch=16,
                  workload="configs[3] geometry, FP32 (the reference FNO3d Run: 64^3 grid, "
                           "width 32, 8x8x8 modes, 4 layers)"),
    "fno3d_fp8": dict(metric="FNO3d FP8-E4M3 samples/s", op="FNO3d", batch=16,
                      workload="configs[3] FNO3d FP8-E4M3 per-tensor (E4M3 codes between "
                               "layers, amax/448 scales from a 4-sample calibration batch)",
                      # 20 P + 14 P C with P = 64^3, C = 32 (one-byte codes between layers)
                      bytes_per_sample=20 * 64 ** 3 + 14 * 64 ** 3 * 32),
    "tm2d": dict(metric="TokenMixer2D FP32 samples/s", op="TokenMixer2D", batch=32,
                 workload="configs[4] TokenMixer2D, 64x64 grid = 4096 tokens, latent 128, "
                          "4 heads, 4 blocks (the reference RunTokenMixer2D arithmetic)"),
    "tm2d_int8": dict(metric="TokenMixer2D INT8 samples/s", op="TokenMixer2D", batch=32,
                      workload="configs[4] with the INT8 per-token q/k/v/o/ffn layers"),
}


def aux_model(name: str) -> str:
    from neuroflow_b200 import ir, synth
    key = hashlib.sha1(json.dumps([name, "v1"]).encode()).hexdigest()[:12]
    path = os.path.join(tempfile.gettempdir(), f"nfx_bench_{name}_{key}.nneuroir")
    if os.path.exists(path):
        return path
    if name in ("fno1d", "fno1d_int8"):
        m = synth.fno1d_model(0, per_token=(name == "fno1d"))
    elif name == "fno2d_fp32":
        return model_path(0)
    elif name in ("fno3d", "fno3d_fp8"):
        m = synth.fno3d_model(0)
    else:
        m = synth.tm2d_model(0)
    tmp = path + f".{os.getpid()}"
    ir.write(tmp, m)
    os.replace(tmp, path)
    return path


def run_aux(args):
    import torch
    from neuroflow_b200 import synth
    from neuroflow_b200.runtime import InferenceRuntime
    spec = AUX[args.workload]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    B = args.batch if args.batch else spec["batch"]
    rng = np.random.default_rng(100)
    if spec["op"] == "FNO1d":
        x = synth.fno1d_inputs(rng, B, 1024)
    elif spec["op"] == "FNO2d":
        x = inputs(100, B)
    elif spec["op"] == "FNO3d":
        x = synth.fno3d_inputs(rng, B, 64)
    else:
        x = synth.tm2d_inputs(rng, B, 64, 64)
    rt = InferenceRuntime(aux_model(args.workload), 0)
    if args.workload in ("fno1d", "fno1d_int8", "tm2d_int8"):
        rt.enable_int8_gemm()
    if args.workload == "fno3d_fp8":
        rt.enable_fp8()
        if not rt.is_fp8_enabled():
            raise RuntimeError("FP8 path not enabled for the bench model")
    dx = torch.from_numpy(x).to(device)
    dy = torch.empty(tuple(x.shape[:-1]) + (1,), dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device)
    run = rt.run_tokenmixer2d_device if spec["op"] == "TokenMixer2D" else rt.run_device
    for _ in range(args.warmup):
        run(dx, dy, stream)
    torch.cuda.synchronize()
    rt.check()
    rt.profile(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            run(dx, dy, stream)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    prof = rt.profile_read()
    rt.profile(False)
    rt.check()
    tot = sum(v[1] for v in prof.values())
    line = {"metric": spec["metric"], "value": round(B * args.steps / (ms * 1e-3), 1),
            "unit": "samples/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "data": "synthetic", "config": {"workload": spec["workload"], "batch": B},
            "kernel_share": {k: round(v[1] / tot, 3) for k, v in prof.items()},
            "gpu_launches": sum(v[0] for v in prof.values()), "clocks": clk.summary()}
    if "bytes_per_sample" in spec:
        hbm, src = peaks()
        gbs = line["value"] * spec["bytes_per_sample"] / 1e9
        line["network_roofline"] = {"bytes_per_sample": spec["bytes_per_sample"],
                                    "achieved_GBps": round(gbs, 1), "peak": hbm,
                                    "peak_source": src, "frac": round(gbs / hbm, 4)}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="nfx", choices=["nfx", "reference"])
    ap.add_argument("--gemm-m", type=int, default=0, help="--workload gemm: one M only")
    ap.add_argument("--gemm-k", type=int, default=0, help="--workload gemm: one K = N only")
    ap.add_argument("--preheat", type=int, default=40,
                    help="untimed steps run after the clock sampler starts")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="samples per GPU (default: the configuration's batch, 256 for the "
                         "headline; smaller values only for profiling captures)")
    ap.add_argument("--workload", default="fno2d_int8", choices=["fno2d_int8", "gemm"] + sorted(AUX),
                    help="fno2d_int8 (default): the headline configs[2] line; the others time "
                         "the remaining BASELINE configurations on one GPU")
    args = ap.parse_args()
    if args.workload == "gemm" and args.impl == "nfx":
        run_gemm(args)
        return
    if args.workload != "fno2d_int8" and args.impl == "nfx":
        run_aux(args)
        return

    if args.impl == "reference":
        # host-only arm: no process group; under torchrun rank 0 alone runs and prints
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        if int(os.environ.get("RANK", "0")) != 0:
            return
        path = model_path(0)
        n = os.cpu_count() or 1
        x = inputs(100, max(1, n))
        from oracle.cpu import Reference
        ref = Reference()
        for _ in range(args.warmup):
            ref.bench(path, x[:1], CFG["out_channels"], 1, 1)
        t = 0.0
        for _ in range(args.steps):
            t += ref.bench(path, x, CFG["out_channels"], n, 1)
        v = n * args.steps / t
        line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT,
                "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "dtype": "fp32",
                "config": {"workload": WORKLOAD, "batch_per_step": n},
                "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": n,
                                 "kind": "reference",
                                 "sample": f"{n} samples per step through the reference "
                                           "InferenceRuntime::Run (FNO2d fake-quant fp32 path; "
                                           "the reference has no INT8 FNO2d), one runtime per "
                                           "thread"},
                "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if not args.batch:
        args.batch = CFG["batch"]
    ws, rank, local = dist_setup(args.gpus)
    result, rt, x_host, path = run_nfx(args, ws, rank, local)
    if rank == 0:
        if ws == 1 and not args.no_gemm:
            import torch
            result["gemm_sweep"] = gemm_rows(torch.device("cuda", local), (65536, 1 << 20),
                                             (32, 64, 128, 256))
        if ws == 1 and not args.no_cpu_baseline:
            n = os.cpu_count() or 1
            v, nthr, reps, t1 = cpu_reference(path, x_host, n)
            result["cpu_baseline"] = {
                "value": round(v, 3), "unit": UNIT, "cores": nthr, "kind": "reference",
                "sample": f"{nthr * reps} samples ({nthr} threads x {reps}) of the same "
                          "workload through the reference InferenceRuntime::Run (fake-quant "
                          "fp32 FNO2d; the reference has no INT8 FNO2d); single-thread "
                          f"{t1:.2f} s/sample"}
        print(json.dumps(result), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
