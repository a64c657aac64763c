"""One rank of the data-parallel GPU tests (tests/test_gpu_dp.py), run as a
child process with RANK / WORLD_SIZE / LOCAL_RANK set; not a test module.

    python tests/dp_worker.py step OUT_DIR     # DP step + 5 SGD steps
    python tests/dp_worker.py lonely OUT_DIR   # world 2, the peer never joins
"""
import datetime
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "go-tensor_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

B, IN, HID, OUT = 512, 256, 512, 100


def step(out_dir):
    from gotensor import dist as gd
    from gotensor import model as gm
    rank, world, local = gd.env_ranks()
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rng = np.random.default_rng(3)  # identical batch and weights on every rank
    x = rng.standard_normal((B, IN)).astype(np.float32)
    y = rng.integers(0, OUT, B)
    layers = [gm.Linear(IN, HID), gm.ReLU(), gm.Linear(HID, HID), gm.ReLU(), gm.Linear(HID, OUT)]
    lo, hi = gd.shard(B, rank, world)
    model = gm.Model(layers, [hi - lo, IN], device=local)
    sd = {}
    for name, shape, _ in model.params:
        fan_in = IN if name.startswith("0.") else HID
        sd[name] = rng.uniform(-1, 1, shape).astype(np.float32) / np.float32(np.sqrt(fan_in))
    model.load_state_dict(sd)
    model.sgd(0.05, 0.9, 1e-4)
    if world > 1:
        # small buckets: the gradient goes out in several all-reduces
        model.dp_init(rank, world, gd.exchange_unique_id(rank), timeout_ms=60000, bucket_bytes=256 << 10)
    model.set_batch(x[lo:hi], y[lo:hi])
    model.forward_backward()
    grads, loss0 = model.flat_grads(), model.loss()
    model.enable_graph(True)  # steps 2.. are captured and replayed, all-reduces included
    for _ in range(5):
        model.train_step()
    params, loss = model.flat_params(), model.loss()
    np.savez(os.path.join(out_dir, f"rank{rank}_of{world}.npz"), grads=grads, params=params, loss0=loss0,
             loss=loss)
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def lonely(out_dir):
    from gotensor._lib import GTError, check, cuda_lib
    from gotensor.backend import CudaBackend
    from gotensor.model import unique_id
    be = CudaBackend(0)
    lib = cuda_lib()
    t0 = time.time()
    try:
        check(lib.gt_comm_init(be.ctx.ptr, 0, 2, unique_id(), 1500))
        err = None
    except GTError as e:
        err = str(e)
    waited = time.time() - t0
    # the context is still usable after the failed join
    v = be.ToHost(be.Unary(5, 0.0, be.FromHost(np.array([-1.0, 2.0], np.float32))))  # RELU
    with open(os.path.join(out_dir, "lonely.json"), "w") as f:
        json.dump({"error": err, "waited": waited, "relu": [float(a) for a in v]}, f)


if __name__ == "__main__":
    {"step": step, "lonely": lonely}[sys.argv[1]](sys.argv[2])
