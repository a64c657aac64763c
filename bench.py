"""Training-step benchmark of go-tensor's B200 backend.

Workloads (`--workload`, default `wide_mlp`), one per benchmark config, each
with seeded synthetic inputs of the config's shape and distribution and
PyTorch-style uniform initial weights (nn/module.go:43-49, nn/conv.go:20-28):

  wide_mlp    Linear(4096,4096)-ReLU-Linear(4096,4096)-ReLU-Linear(4096,1000),
              float32, batch 8192, N(0,1) inputs, SGD lr 0.01 momentum 0.9
              weight decay 1e-4 (the headline)
  mlp         Linear(784,128)-ReLU-Linear(128,10), float32, batch 64,
              U[0,1) inputs, Adam lr 1e-3
  cnn         Conv2d(1,32,3,p1)-ReLU-MaxPool2d(2)-Conv2d(32,64,3,p1)-ReLU-
              MaxPool2d(2)-Flatten-Linear(3136,128)-ReLU-Dropout(0)-
              Linear(128,10), float32, batch 256, U[0,1) inputs, Adam
  conv_stack  four Conv2d(3x3,p1)-ReLU-MaxPool2d(2) blocks of 64/128/256/512
              channels on [3,32,32], Flatten-Linear(2048,10), float32, batch
              1024, N(0,1) inputs, Adam
  fp64_mlp    Linear(1024,1024)-Tanh-Linear(1024,1024)-Sigmoid-Linear(1024,10),
              float64, batch 4096, U[-1,1) inputs, Adam

Labels are uniform over the classes. A step is one forward + backward +
optimizer update of the whole global batch, which is sharded over the GPUs
(strong scaling) with gradients averaged over NCCL.

    python bench.py [--workload W] [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU. Rank 0 prints one JSON line.
`--impl reference` times go-tensor's CPU path (the oracle's restatement of
internal/cpu and the tensor/nn/optim layers, all host threads) on a bounded
sample of the same workload and prints the same metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "go-tensor_b200"))
sys.path.insert(0, ROOT)

METRIC = "train samples/sec (fwd+bwd+step)"

# Per-sample GEMM flops (forward, dW, and dX for every layer but the first;
# convolutions as 2 N OH OW O C KH KW with padded taps counted), the
# algorithmic work the GEMM roofline divides.
WORKLOADS = {
    "wide_mlp": {
        "name": "wide_mlp_4096-4096-4096-1000_b8192_sgd", "batch": 8192, "sample": [4096], "classes": 1000,
        "dtype": "f32", "x": "normal", "opt": "sgd", "gemm_flops": 192_348_160,
        "layers": [("Linear", (4096, 4096)), ("ReLU", ()), ("Linear", (4096, 4096)), ("ReLU", ()),
                   ("Linear", (4096, 1000))]},
    "mlp": {
        "name": "mlp_784-128-10_b64_adam", "batch": 64, "sample": [784], "classes": 10, "dtype": "f32",
        "x": "uniform01", "opt": "adam", "gemm_flops": 409_088,
        "layers": [("Linear", (784, 128)), ("ReLU", ()), ("Linear", (128, 10))]},
    "cnn": {
        "name": "cnn_28x28_c32-64_fc128_b256_adam", "batch": 256, "sample": [1, 28, 28], "classes": 10,
        "dtype": "f32", "x": "uniform01", "opt": "adam", "gemm_flops": 24_995_328,
        "layers": [("Conv2d", (1, 32, 3, 1, 1)), ("ReLU", ()), ("MaxPool2d", (2, 0)),
                   ("Conv2d", (32, 64, 3, 1, 1)), ("ReLU", ()), ("MaxPool2d", (2, 0)), ("Flatten", ()),
                   ("Linear", (3136, 128)), ("ReLU", ()), ("Dropout", (0.0,)), ("Linear", (128, 10))]},
    "conv_stack": {
        "name": "conv_stack_32x32_c64-128-256-512_b1024_adam", "batch": 1024, "sample": [3, 32, 32],
        "classes": 10, "dtype": "f32", "x": "normal", "opt": "adam", "gemm_flops": 346_939_392,
        "layers": [("Conv2d", (3, 64, 3, 1, 1)), ("ReLU", ()), ("MaxPool2d", (2, 0)),
                   ("Conv2d", (64, 128, 3, 1, 1)), ("ReLU", ()), ("MaxPool2d", (2, 0)),
                   ("Conv2d", (128, 256, 3, 1, 1)), ("ReLU", ()), ("MaxPool2d", (2, 0)),
                   ("Conv2d", (256, 512, 3, 1, 1)), ("ReLU", ()), ("MaxPool2d", (2, 0)), ("Flatten", ()),
                   ("Linear", (2048, 10))]},
    "fp64_mlp": {
        "name": "fp64_mlp_1024-1024-1024-10_b4096_adam", "batch": 4096, "sample": [1024], "classes": 10,
        "dtype": "f64", "x": "uniform11", "opt": "adam", "gemm_flops": 10_547_200,
        "layers": [("Linear", (1024, 1024)), ("Tanh", ()), ("Linear", (1024, 1024)), ("Sigmoid", ()),
                   ("Linear", (1024, 10))]},
}
SGD_CFG = (0.01, 0.9, 1e-4)   # lr, momentum, weight decay
ADAM_LR = 1e-3
# Optimizer bytes per parameter: SGD with momentum and weight decay reads p,
# g, v and writes p, v; Adam reads p, g, m, v and writes p, m, v.
OPT_BYTES = {("sgd", "f32"): 20, ("adam", "f32"): 28, ("adam", "f64"): 56, ("sgd", "f64"): 40}
# FP64 peak: the HGX B200 datasheet's FP64 / FP64 tensor-core figure (the
# measured-peaks file has no float64 entry).
FP64_PEAK_TFLOPS = 37.0
CPU_SAMPLE_ROWS = {"wide_mlp": 256, "mlp": 64, "cnn": 64, "conv_stack": 32, "fp64_mlp": 512}


def make_layers(gm, spec):
    return [getattr(gm, kind)(*args) for kind, args in spec]


def init_params(model, spec, seed=1):
    """U(+-1/sqrt(fan_in)) for every weight and bias, fan_in of its layer."""
    rng = np.random.default_rng(seed)
    fans = []
    for kind, args in spec:
        if kind == "Linear":
            fans += [args[0], args[0]]
        elif kind == "Conv2d":
            fans += [args[0] * args[2] * args[2]] * 2
    sd = {}
    for (name, shape, _), fan in zip(model.params, fans):
        b = 1 / np.sqrt(fan)
        sd[name] = rng.uniform(-b, b, shape).astype(model.np_dtype)
    return sd


def make_batch(wl, rows, seed):
    rng = np.random.default_rng(seed)
    shape = [rows] + wl["sample"]
    n = int(np.prod(shape))
    x = {"normal": lambda: rng.standard_normal(n), "uniform01": lambda: rng.random(n),
         "uniform11": lambda: rng.uniform(-1, 1, n)}[wl["x"]]()
    y = rng.integers(0, wl["classes"], rows).astype(np.int32)
    return x.reshape(shape).astype(np.float64 if wl["dtype"] == "f64" else np.float32), y


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


CLOCK_FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def clocks_sampler(index: int):
    """Starts nvidia-smi sampling GPU `index` every 50 ms (timestamped), well
    before the timed regions so that its start-up delay costs no samples."""
    out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
    try:
        p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={CLOCK_FIELDS}",
                              "--format=csv,noheader,nounits", "-lms", "50"], stdout=out, stderr=subprocess.DEVNULL)
    except OSError:
        return None, out.name
    # NVML's start-up can hold the driver for a moment; let it finish (first
    # sample written) before anything is timed.
    deadline = time.time() + 10
    while time.time() < deadline and p.poll() is None and os.path.getsize(out.name) == 0:
        time.sleep(0.05)
    return p, out.name


def clocks_summary(proc, path, windows):
    """Median SM clock, max clock and active throttle reasons over the samples
    taken inside `windows` (host-time intervals of the timed regions). A
    timed region shorter than the 50 ms sampling period (the small configs)
    may hold no sample: then the samples within 100 ms of a region are used,
    and the line says so (`window_margin_ms`)."""
    import datetime as _dt
    if proc is None:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
    proc.terminate()
    try:
        proc.wait(timeout=5)
    except subprocess.TimeoutExpired:
        proc.kill()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    rows = []
    with open(path) as f:
        for line in f:
            c = [x.strip() for x in line.split(",")]
            if len(c) < 10:
                continue
            try:
                t = _dt.datetime.strptime(c[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                mhz, mx = float(c[2]), float(c[3])
            except ValueError:
                continue
            try:
                pw = float(c[4])
            except ValueError:
                pw = None
            rows.append((t, mhz, mx, pw, {n for n, v in zip(names, c[6:10]) if v.lower() == "active"}))
    os.unlink(path)
    out = {}
    for margin in (0.0, 0.1):
        picked = [r for r in rows if any(lo - margin <= r[0] <= hi + margin for lo, hi in windows)]
        if picked:
            if margin:
                out["window_margin_ms"] = 1000 * margin
            break
    else:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples near the timed regions"]}
    sm = [r[1] for r in picked]
    power = [r[3] for r in picked if r[3] is not None]
    reasons = set().union(*(r[4] for r in picked))
    out.update({"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[2] for r in picked),
                "reasons": sorted(reasons), "samples": len(sm), "sm_mhz_min": min(sm),
                "power_w_max": max(power) if power else None})
    return out


# ---------------------------------------------------------------------------
# CPU leg: the oracle's restatement of go-tensor's CPU path

def cpu_step_time(wl, rows: int, steps: int, warmup: int, threads: int):
    """Times the oracle's training loop on `rows` samples of the workload:
    per step, the forward + backward (loss, ZeroGrad, Backward) and, apart,
    the optimizer update of all parameters. Returns two lists of seconds."""
    from oracle import gotensor_ref as T
    from oracle import nn_ref as nn
    from oracle import optim_ref as optim
    T.SetDefaultDType(T.Float64 if wl["dtype"] == "f64" else T.Float32)
    T._factories[T.CPU_TYPE] = lambda index: T.CPUBackend(threads)
    T._backends.clear()
    T.ManualSeed(1)
    model = nn.NewSequential(*[getattr(nn, "New" + kind)(*args) for kind, args in wl["layers"]])
    if wl["opt"] == "sgd":
        opt = optim.NewSGD(model.Parameters(), optim.SGDConfig(LR=SGD_CFG[0], Momentum=SGD_CFG[1],
                                                               WeightDecay=SGD_CFG[2]))
    else:
        opt = optim.NewAdam(model.Parameters(), optim.AdamConfig(LR=ADAM_LR))
    xb, yb = make_batch(wl, rows, 1)
    x = T.New(xb.astype(np.float64).reshape(-1), *xb.shape)
    y = [int(v) for v in yb]
    fb, st = [], []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        loss = nn.CrossEntropyLoss(model.Forward(x), y)
        opt.ZeroGrad()
        loss.Backward()
        loss.Item()
        t1 = time.perf_counter()
        opt.Step()
        model.Parameters()[0].Float64s()[:1]  # the update has landed
        t2 = time.perf_counter()
        if i >= warmup:
            fb.append(t1 - t0)
            st.append(t2 - t1)
    return fb, st


def cpu_baseline(wl_key, steps, warmup, threads):
    """Samples/s of the CPU path at the workload's full global batch: the
    forward + backward cost (linear in the rows, as the row-split MatMul of
    internal/cpu/linalg.go:65-81 is) measured on a sample of rows and scaled
    to the batch, plus the optimizer update, which does not depend on the
    batch, measured at its full size. Returns (value, seconds per step,
    description)."""
    wl = WORKLOADS[wl_key]
    rows = min(CPU_SAMPLE_ROWS[wl_key], wl["batch"])
    fb, st = cpu_step_time(wl, rows, steps, warmup, threads)
    t_fb, t_st = statistics.median(fb), statistics.median(st)
    t_step = t_fb * wl["batch"] / rows + t_st
    desc = (f"forward+backward timed on {rows} of the {wl['batch']} rows and scaled to the batch "
            f"({t_fb * 1e3:.1f} ms x {wl['batch'] // rows}), plus the optimizer update of all parameters timed "
            f"at full size ({t_st * 1e3:.1f} ms); median of {len(fb)} steps after {warmup} warm-up; oracle "
            "restatement of go-tensor's CPU backend and tensor/nn/optim (Go is absent)")
    if rows == wl["batch"]:
        desc = (f"the full batch of {rows} rows, median of {len(fb)} steps after {warmup} warm-up; oracle "
                "restatement of go-tensor's CPU backend and tensor/nn/optim (Go is absent)")
    return wl["batch"] / t_step, t_step, desc


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    # keep the arm to a few minutes: the sampled steps of the large configs take seconds each
    steps = max(1, min(args.steps, 5))
    warmup = 1
    value, t_step, desc = cpu_baseline(args.workload, steps, warmup, threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": wl["dtype"],
        "data": "synthetic (seeded inputs of the config's shape and distribution, uniform labels)",
        "config": {"workload": wl["name"], "global_batch": wl["batch"]},
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": desc + f"; {steps} timed steps (the arm caps them at 5)"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU leg

def init_dist(n_gpus):
    from gotensor.dist import env_ranks
    rank, world, local = env_ranks()
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def allgather_max(x, world):
    from gotensor.dist import max_over_ranks
    return max_over_ranks(x)


def barrier(world):
    from gotensor.dist import barrier as _barrier
    _barrier()


def run_ours(args):
    import torch

    from gotensor import FLOAT32, FLOAT64
    from gotensor import model as gm
    from gotensor._lib import check, cuda_lib
    wl = WORKLOADS[args.workload]
    f64 = wl["dtype"] == "f64"
    es = 8 if f64 else 4
    rank, world, local = init_dist(args.gpus)
    torch.cuda.set_device(local)
    from gotensor.dist import exchange_unique_id, shard
    lo, hi = shard(wl["batch"], rank, world)
    B = hi - lo
    model = gm.Model(make_layers(gm, wl["layers"]), [B] + wl["sample"], dtype=FLOAT64 if f64 else FLOAT32,
                     device=local)
    lib, ctx = cuda_lib(), model.ctx.ptr
    model.load_state_dict(init_params(model, wl["layers"], 1))  # same weights on every rank
    if wl["opt"] == "sgd":
        model.sgd(*SGD_CFG)
    else:
        model.adam(lr=ADAM_LR)
    if world > 1:
        # rank 0's stdout carries exactly one JSON line: keep NCCL's version banner off it
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        model.dp_init(rank, world, exchange_unique_id(rank), timeout_ms=120000, bucket_bytes=args.bucket_mb << 20)
    model.enable_graph(not args.no_graph)

    # This rank's shard of the batch, in pinned host memory for the e2e leg.
    x_np, y_np = make_batch(wl, B, 100 + rank)
    xh = torch.from_numpy(x_np).pin_memory()
    yh = torch.from_numpy(y_np).pin_memory()
    loss_h = torch.zeros(1, dtype=torch.float64 if f64 else torch.float32).pin_memory()
    h2d = xh.numel() * es + yh.numel() * 4
    model.set_batch(x_np, y_np)

    def steps_resident(k):
        for _ in range(k):
            model.train_step()

    def steps_e2e(k):
        # Every step's batch goes host -> device (pinned memory, copy stream)
        # and its loss comes back. The upload of batch i+1 overlaps step i;
        # the first upload has nothing to overlap.
        model.stage_batch(xh.data_ptr(), yh.data_ptr())
        for i in range(k):
            if i + 1 < k:
                model.stage_batch(xh.data_ptr(), yh.data_ptr())
            model.train_step()
            check(lib.gt_download_async(ctx, loss_h.data_ptr(), model.lib.gth_loss_device(model.ptr), es))

    def timed(fn, k):
        """Device time of fn(k) (k steps) on the model's stream, max over ranks."""
        barrier(world)
        model.ctx.sync()
        torch.cuda.synchronize()
        check(lib.gt_mark(ctx, 0))
        fn(k)
        check(lib.gt_mark(ctx, 1))
        ms = ctypes.c_float()
        check(lib.gt_elapsed_ms(ctx, 0, 1, ctypes.byref(ms)))
        model.ctx.sync()
        torch.cuda.synchronize()
        barrier(world)
        return allgather_max(ms.value, world)

    proc, cpath = clocks_sampler(local)
    steps_resident(max(args.warmup, 3))
    model.ctx.sync()
    launches_per_step = model.step_launches
    before = lib.gt_launch_count()
    windows = []
    t0 = time.time()
    ms_total = timed(steps_resident, args.steps)
    windows.append((t0, time.time()))
    launches = lib.gt_launch_count() - before
    if launches == 0:  # graph replays launch without passing through the library's counter
        launches = launches_per_step * args.steps
    value = wl["batch"] * args.steps / (ms_total / 1e3)
    loss = model.loss()

    steps_e2e(2)
    t0 = time.time()
    ms_e2e = timed(steps_e2e, args.steps)
    windows.append((t0, time.time()))
    clocks = clocks_summary(proc, cpath, windows)
    e2e = wl["batch"] * args.steps / (ms_e2e / 1e3)

    # Roofline of the dominant kernel, the GEMM (tcgen05 3xTF32 for float32,
    # the FP64 pipe for float64): K more steps of the same workload with every
    # GEMM launch bracketed by CUDA events on the model's stream (graph replay
    # off: events inside a replayed graph keep only the last replay's times).
    roof = step_roofline(lib, model, args.steps, wl, args.workload)
    roof["roofline"]["step_ms_graph"] = ms_total / args.steps

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        threads = os.cpu_count() or 1
        cval, _, desc = cpu_baseline(args.workload, 2, 1, threads)
        cpu = {"value": cval, "unit": "samples/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        opt_desc = (f"sgd(lr={SGD_CFG[0]}, momentum={SGD_CFG[1]}, wd={SGD_CFG[2]})" if wl["opt"] == "sgd"
                    else f"adam(lr={ADAM_LR})")
        line = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": wl["dtype"],
            "data": "synthetic (seeded inputs of the config's shape and distribution, uniform labels, "
                    "PyTorch-style uniform init)",
            "config": {"workload": wl["name"], "global_batch": wl["batch"], "per_gpu_batch": B,
                       "parallelism": f"dp{world}", "optimizer": opt_desc, "graph": not args.no_graph,
                       "l2": l2_note(args.workload, model),
                       "gemm": roof["path"]},
            "gemm_launches": roof["launches"],
            "loss_after": loss,
            "e2e": {"value": e2e, "unit": "samples/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": es},
            "gpu_launches": int(launches),
            "roofline": roof["roofline"],
            "optimizer_roofline": roof["optimizer"],
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    barrier(world)
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def l2_note(key, model):
    """Why no L2 flush is needed between timed steps: the step's working set
    (parameters, gradients, optimizer state, activations) against the 126 MB L2."""
    es = model.np_dtype().itemsize
    state = model.num_params * es * (3 if WORKLOADS[key]["opt"] == "sgd" else 4)
    if key in ("wide_mlp", "conv_stack", "fp64_mlp", "cnn"):
        return (f"per-step working set exceeds L2: parameters, gradients and optimizer state "
                f"{state / 1e6:.0f} MB plus activations")
    return (f"the whole working set ({state / 1e6:.1f} MB of parameters and state plus activations) fits in "
            "L2: a small-batch, launch-latency-bound config, timed as it runs")


# dram__bytes_read.sum + dram__bytes_write.sum of the GEMM launches of one
# training step of the wide MLP, from one ncu capture of
# `bench.py --workload wide_mlp --steps 1 --warmup 3 --skip-cpu` (launches
# 16-31: the second warm-up step, replayed from the CUDA graph).
GEMM_TRAFFIC_BYTES_PER_STEP = {"wide_mlp": 4_234_614_272}
GEMM_LAUNCHES_PER_STEP = {"wide_mlp": 8}
# The wide MLP's SGD update: DRAM traffic of its launch in the same capture.
OPT_TRAFFIC_BYTES = {"wide_mlp": 698_175_488}


def _peak_3xtf32():
    hbm, bf16, kind = peaks()
    # 3xTF32: three TF32 products per fp32 MAC; TF32 runs at half the bf16 rate.
    return bf16 / 2 / 3, f"3xTF32 peak = {kind} bf16 burst {bf16:.0f} TF/s / 2 (TF32 rate) / 3 (products)"


def _peak_3xtf32_sustained():
    """The same from the sustained (power-capped) bf16 figure, or None."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]) / 2 / 3
    except Exception:
        return None


def step_roofline(lib, model, steps, wl, key):
    """Runs `steps` training steps with the GEMM launch timer on; returns the
    flop rate of all GEMM launches (total algorithmic flops / total kernel
    time) against the GEMM peak of the dtype, the optimizer kernel's bytes per
    second against HBM, and the per-shape breakdown."""
    from gotensor._lib import check
    ctx = model.ctx.ptr
    f64 = wl["dtype"] == "f64"
    if f64:
        peak, note, sustained = FP64_PEAK_TFLOPS, "FP64 peak = 37 TF/s (HGX B200 datasheet; nominal)", None
    else:
        peak, note = _peak_3xtf32()
        note += " (of measured)"
        sustained = _peak_3xtf32_sustained()
    model.enable_graph(False)
    check(lib.gt_gemm_timer_start(ctx, steps * 64 + 64))
    pass_ms, opt_ms, t = ctypes.c_float(), 0.0, ctypes.c_float()
    check(lib.gt_mark(ctx, 4))
    for _ in range(steps):
        # train_step without a graph: forward_backward, then optimizer_step;
        # marks 6/7 bracket the optimizer kernel (read back every step)
        model.forward_backward()
        check(lib.gt_mark(ctx, 6))
        model.optimizer_step()
        check(lib.gt_mark(ctx, 7))
        check(lib.gt_elapsed_ms(ctx, 6, 7, ctypes.byref(t)))
        opt_ms += t.value
    check(lib.gt_mark(ctx, 5))
    check(lib.gt_elapsed_ms(ctx, 4, 5, ctypes.byref(pass_ms)))
    hbm, _, hbm_kind = peaks()
    nparams = model.num_params
    bpp = OPT_BYTES[(wl["opt"], wl["dtype"])]
    # The update alone: `steps` optimizer steps back to back on the stream
    # (the steps above interleave it with the host's launches of the next
    # step, which leaves small updates waiting on launch latency).
    check(lib.gt_mark(ctx, 6))
    for _ in range(steps):
        model.optimizer_step()
    check(lib.gt_mark(ctx, 7))
    check(lib.gt_elapsed_ms(ctx, 6, 7, ctypes.byref(t)))
    opt_alone_ms = t.value / steps
    opt_gbs = bpp * nparams / (opt_alone_ms / 1e3) / 1e9
    kern = ("sgd_kernel (momentum + weight decay, one pass)" if wl["opt"] == "sgd"
            else "adam_kernel (one pass; bias corrections from a device step counter, then the counter's increment)")
    optimizer = {"bound": "hbm", "kernel": kern, "achieved": opt_gbs, "peak": hbm, "unit": "GB/s",
                 "frac": opt_gbs / hbm, "bytes_per_launch": bpp * nparams, "ms_per_launch": opt_alone_ms,
                 "ms_per_step_in_pass": opt_ms / steps, "traffic": OPT_TRAFFIC_BYTES.get(key),
                 "note": f"{bpp} B/param x {nparams} params; {steps} updates back to back, CUDA events on the "
                         f"model's stream; peak = {hbm_kind} copy bandwidth (of {hbm_kind})"}
    n, dropped = ctypes.c_int64(), ctypes.c_int64()
    check(lib.gt_gemm_timer_count(ctx, ctypes.byref(n), ctypes.byref(dropped)))
    if dropped.value:
        raise SystemExit(f"GEMM timer dropped {dropped.value} launches")
    shapes = {}
    last_step = []  # (M x N x K, ms) of every GEMM of the pass's last step, in launch order
    total_ms = total_flops = 0.0
    paths = set()
    mnk = (ctypes.c_int64 * 3)()
    path = ctypes.c_int()
    ms = ctypes.c_float()
    for i in range(n.value):
        check(lib.gt_gemm_timer_read(ctx, i, mnk, ctypes.byref(path), ctypes.byref(ms)))
        key_s = f"{mnk[0]}x{mnk[1]}x{mnk[2]}"
        if i >= n.value - n.value // steps:
            last_step.append((key_s, round(ms.value, 4)))
        flops = 2.0 * mnk[0] * mnk[1] * mnk[2]
        e = shapes.setdefault(key_s, {"launches": 0, "times": [], "flops": flops, "path": path.value})
        e["launches"] += 1
        e["times"].append(ms.value)
        total_flops += flops
        paths.add(path.value)
    check(lib.gt_gemm_timer_stop(ctx))
    # A shape's time per launch is the median over its launches in the pass:
    # a launch whose bracket caught a one-off stall (the pool growing its
    # workspace, say) does not stand for the kernel.
    for v in shapes.values():
        v["ms"] = statistics.median(v["times"]) * v["launches"]
        total_ms += v["ms"]
    per_step = n.value // steps
    achieved = total_flops / (total_ms / 1e3) / 1e12
    traffic = None
    if GEMM_TRAFFIC_BYTES_PER_STEP.get(key) and per_step == GEMM_LAUNCHES_PER_STEP.get(key):
        traffic = GEMM_TRAFFIC_BYTES_PER_STEP[key] / GEMM_LAUNCHES_PER_STEP[key]
    names = {1: "SIMT (FFMA; float64 on DFMA or the FP64 tensor path, mma.sync f64)", 2: "tcgen05 3xTF32",
             4: "tcgen05 3xTF32 implicit-GEMM convolution",
             5: "SIMT weight gradient from the pooled gradient (first conv; window maxima only)",
             6: "SIMT thin GEMM (a classifier's 10 classes: a warp per row, or a thread per column)",
             7: "SIMT direct convolution + ReLU + 2x2 pool (first conv, K = C*9)"}
    breakdown = {k: {"launches_per_step": v["launches"] // steps, "ms_per_launch": v["ms"] / v["launches"],
                     "ms_max": max(v["times"]),
                     "tflops": v["flops"] * v["launches"] / (v["ms"] / 1e3) / 1e12,
                     "path": names.get(v["path"], str(v["path"]))} for k, v in shapes.items()}
    step_ms = pass_ms.value / steps
    alg = wl["gemm_flops"] * model.input_shape[0]
    return {"path": " + ".join(sorted(names.get(p, str(p)) for p in paths)), "launches": per_step,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": ("every GEMM launch of the step (forward, dW, dX), M x N x K below; float64 "
                                    "on the FP64 pipe" if f64 else
                                    "every GEMM launch of the step (forward, dW, dX; convolutions as GEMMs), "
                                    "M x N x K below"),
                         "flops_per_launch": total_flops / max(n.value, 1), "ms_per_launch": total_ms / max(n.value, 1),
                         "algorithmic_gemm_flops_per_step": alg,
                         "algorithmic_tflops_over_step": alg / (step_ms / 1e3) / 1e12,
                         "gemm_share_of_step": total_ms / pass_ms.value, "step_ms_timed_pass": step_ms,
                         "by_shape": breakdown, "last_step_launches": last_step,
                         "peak_note": note, "peak_sustained": sustained,
                         "frac_of_sustained": (achieved / sustained) if sustained else None},
            "optimizer": optimizer}


IN, HID, OUT = 4096, 4096, 1000  # the wide MLP's widths, for the isolated GEMM and eval modes
GLOBAL_BATCH = 8192
WORKLOAD = WORKLOADS["wide_mlp"]["name"]


def gemm_isolated(lib, model, B, reps):
    """The backward GEMMs of one 4096x4096 layer at batch B (dW, then dX),
    `reps` times each after two warm-up launches, alone on the model's stream."""
    from gotensor._lib import check
    ctx = model.ctx
    peak, note = _peak_3xtf32()
    fp = model.ctx.alloc
    x = fp(B * HID * 4)
    dy = fp(B * HID * 4)
    w = fp(HID * HID * 4)
    dw = fp(HID * HID * 4)
    dx = fp(B * HID * 4)
    rng = np.random.default_rng(5)
    for p, n in ((x, B * HID), (dy, B * HID), (w, HID * HID)):
        # realistic operands: tensor-core power (and so clocks) depend on the data
        h = rng.standard_normal(n, dtype=np.float32)
        check(lib.gt_upload(ctx.ptr, p, h.ctypes.data, n * 4))
    for _ in range(2):
        check(lib.gt_linear_bwd_weight(ctx.ptr, 0, x, dy, dw, None, B, HID, HID))
        check(lib.gt_linear_bwd_data(ctx.ptr, 0, dy, w, x, 1, dx, B, HID, HID))
    check(lib.gt_mark(ctx.ptr, 2))
    for _ in range(reps):
        check(lib.gt_linear_bwd_weight(ctx.ptr, 0, x, dy, dw, None, B, HID, HID))
        check(lib.gt_linear_bwd_data(ctx.ptr, 0, dy, w, x, 1, dx, B, HID, HID))
    check(lib.gt_mark(ctx.ptr, 3))
    ms = ctypes.c_float()
    check(lib.gt_elapsed_ms(ctx.ptr, 2, 3, ctypes.byref(ms)))
    per_launch_ms = ms.value / (2 * reps)
    flops = 2.0 * B * HID * HID
    achieved = flops / (per_launch_ms / 1e3) / 1e12
    for p in (x, dy, w, dw, dx):
        ctx.release(p)
    return {"kernel": f"backward GEMMs of a 4096x4096 layer (dW and dX, M=K=4096, batch {B}), alone",
            "per_launch_ms": per_launch_ms, "achieved_tflops": achieved, "peak_tflops": peak,
            "frac": achieved / peak, "gemm_path": lib.gt_gemm_path_taken(), "peak_note": note}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="wide_mlp")
    ap.add_argument("--batch", type=int, default=0,
                    help="global batch override (a small case of the workload, for profiling); default: the config's")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--bucket-mb", type=int, default=32)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--gemm-only", action="store_true",
                    help="time only the dominant kernel (the backward GEMMs at the workload's shapes), for profiling")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--checkpoint-only", action="store_true",
                    help="time checkpoints of the workload's model (safetensors F32 and GOTN, save and load)")
    ap.add_argument("--eval-only", action="store_true",
                    help="time evaluation instead (forward + Argmax + correct count on the device)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.batch:
        WORKLOADS[args.workload] = dict(WORKLOADS[args.workload], batch=args.batch,
                                        name=WORKLOADS[args.workload]["name"] + f"_batch{args.batch}")
    if args.impl == "reference":
        return run_reference(args)
    if args.gemm_only:
        return run_gemm_only(args)
    if args.eval_only:
        return run_eval_only(args)
    if args.checkpoint_only:
        return run_checkpoint_only(args)
    return run_ours(args)


def run_gemm_only(args):
    """Times only the dominant kernel (the backward GEMMs at the workload's
    shapes) and prints one JSON line; the case the ncu --set full capture runs."""
    from gotensor import model as gm
    from gotensor._lib import cuda_lib
    lib = cuda_lib()
    model = gm.Model([gm.Linear(IN, HID), gm.ReLU(), gm.Linear(HID, OUT)], [GLOBAL_BATCH, IN])
    print(json.dumps(gemm_isolated(lib, model, GLOBAL_BATCH, args.reps)), flush=True)
    return 0


def run_checkpoint_only(args):
    """Checkpoints of the workload's model (37.7M float32 parameters) through
    the native writer and reader, to a file in memory-backed /dev/shm when
    there is one (so the file system does not dominate). Prints one JSON
    line with the wall time and file bytes per second of each."""
    from gotensor import model as gm
    from gotensor._lib import check
    model = gm.Model([gm.Linear(IN, HID), gm.ReLU(), gm.Linear(HID, HID), gm.ReLU(), gm.Linear(HID, OUT)],
                     [GLOBAL_BATCH, IN])
    rng = np.random.default_rng(1)
    model.set_flat_params(rng.standard_normal(model.num_params).astype(np.float32))
    lib = model.lib
    folder = "/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir()
    out = {}
    for fmt in ("safetensors_f32", "gotn_f64"):
        path = os.path.join(folder, f"gotensor_bench.{fmt}")
        if fmt.startswith("safetensors"):
            save = lambda: check(lib.gth_save_safetensors(model.ptr, path.encode(), b"F32", None, None, 0))
            load = lambda: check(lib.gth_load_safetensors(model.ptr, path.encode(), 1))
        else:
            save = lambda: check(lib.gth_save_gotn(model.ptr, path.encode()))
            load = lambda: check(lib.gth_load_gotn(model.ptr, path.encode()))
        res = {}
        for name, fn in (("save", save), ("load", load)):
            fn()
            times = []
            for _ in range(max(args.steps, 3)):
                t = time.perf_counter()
                fn()
                model.ctx.sync()
                times.append(time.perf_counter() - t)
            size = os.path.getsize(path)
            res[name] = {"ms": 1e3 * statistics.median(times), "file_bytes": size,
                         "gb_per_s": size / statistics.median(times) / 1e9}
        os.unlink(path)
        out[fmt] = res
    print(json.dumps({"metric": "checkpoint of the wide MLP (37.7M float32 parameters)", "folder": folder,
                      "results": out}), flush=True)
    return 0


def run_eval_only(args):
    """Evaluation of the workload's model at batch 8192 (NoGrad forward,
    Argmax of every row and the correct count on the device, one 8-byte
    count read back per batch), and the Argmax kernel alone on the 8192 x
    1000 logits against HBM bandwidth. Prints one JSON line."""
    import torch

    from gotensor import model as gm
    from gotensor._lib import check, cuda_lib
    lib = cuda_lib()
    model = gm.Model([gm.Linear(IN, HID), gm.ReLU(), gm.Linear(HID, HID), gm.ReLU(), gm.Linear(HID, OUT)],
                     [GLOBAL_BATCH, IN])
    rng = np.random.default_rng(1)
    model.set_flat_params((rng.standard_normal(model.num_params) * 0.01).astype(np.float32))
    model.set_batch(rng.standard_normal((GLOBAL_BATCH, IN)).astype(np.float32), rng.integers(0, OUT, GLOBAL_BATCH))
    ctx = model.ctx.ptr
    for _ in range(max(args.warmup, 3)):
        model.count_correct()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.count_correct()
    wall = (time.perf_counter() - t0) / args.steps
    # the Argmax kernel alone, CUDA events on the context's stream
    logits = model.ctx.alloc(GLOBAL_BATCH * OUT * 4)
    preds = model.ctx.alloc(GLOBAL_BATCH * 4)
    h = rng.standard_normal(GLOBAL_BATCH * OUT).astype(np.float32)
    check(lib.gt_upload(ctx, logits, h.ctypes.data, h.nbytes))
    for _ in range(3):
        check(lib.gt_argmax_rows(ctx, 0, logits, GLOBAL_BATCH, OUT, preds))
    check(lib.gt_mark(ctx, 0))
    reps = 50
    for _ in range(reps):
        check(lib.gt_argmax_rows(ctx, 0, logits, GLOBAL_BATCH, OUT, preds))
    check(lib.gt_mark(ctx, 1))
    ms = ctypes.c_float()
    check(lib.gt_elapsed_ms(ctx, 0, 1, ctypes.byref(ms)))
    per = ms.value / reps
    nbytes = GLOBAL_BATCH * OUT * 4 + GLOBAL_BATCH * 4
    hbm, _, kind = peaks()
    gbs = nbytes / (per / 1e3) / 1e9
    model.ctx.release(logits)
    model.ctx.release(preds)
    print(json.dumps({"metric": "eval samples/sec (forward + argmax + correct count)", "value": GLOBAL_BATCH / wall,
                      "unit": "samples/s", "ms_per_batch": wall * 1e3, "workload": WORKLOAD + "_eval",
                      "argmax_kernel": {"bound": "hbm", "ms": per, "bytes": nbytes, "achieved": gbs,
                                        "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                                        "note": f"logits 8192 x 1000 fp32 + int32 indices; peak = {kind} copy "
                                                "bandwidth (the logits fit in L2 across repetitions)"}}),
          flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
