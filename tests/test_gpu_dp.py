"""Data parallelism over NCCL, ranks as child processes (tests/dp_worker.py),
one per GPU.

* two GPUs, each training on half the batch with gradients averaged in
  several buckets during the backward pass, match one GPU training on the
  whole batch (mean of equal shard means = the global mean), and both ranks
  hold bitwise identical gradients and, after five captured-graph SGD steps,
  bitwise identical parameters;
* a rank whose peer never joins gets an error from gt_comm_init within its
  deadline instead of hanging, and its device context stays usable (the
  failure is made on the host: the second rank is simply never started).
"""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from gpu_common import assert_close

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
WORKER = os.path.join(HERE, "dp_worker.py")


def _gpus():
    import torch
    return torch.cuda.device_count()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(mode, out_dir, rank, world, port, extra_env=None):
    env = dict(os.environ, RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
               MASTER_PORT=str(port))
    env.update(extra_env or {})
    return subprocess.Popen([sys.executable, WORKER, mode, str(out_dir)], env=env, stdout=subprocess.PIPE,
                            stderr=subprocess.STDOUT, text=True)


def _wait(procs, timeout=240):
    outs = []
    try:
        for p in procs:
            out, _ = p.communicate(timeout=timeout)
            outs.append(out)
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    for p, out in zip(procs, outs):
        assert p.returncode == 0, out[-3000:]


@pytest.mark.skipif("_gpus() < 2", reason="needs two GPUs")
@pytest.mark.parametrize("extra_env", [{}, {"GT_DP_LAST_CHUNKS": "4"}], ids=["one_dw_gemm", "dw_in_row_chunks"])
def test_two_gpu_dp_matches_one_gpu(tmp_path, extra_env):
    """With GT_DP_LAST_CHUNKS=4 the first Linear's weight gradient (N = 512
    rows) is computed in 4 chunks of 128 rows, each averaged while the next is
    computed, and its bias rides in the first chunk's bucket."""
    _wait([_spawn("step", tmp_path, 0, 1, _free_port())])
    port = _free_port()
    _wait([_spawn("step", tmp_path, r, 2, port, extra_env) for r in range(2)])
    one = np.load(tmp_path / "rank0_of1.npz")
    r0, r1 = np.load(tmp_path / "rank0_of2.npz"), np.load(tmp_path / "rank1_of2.npz")
    # every rank holds the same averaged gradient and, after the steps, the same weights
    assert np.array_equal(r0["grads"], r1["grads"])
    assert np.array_equal(r0["params"], r1["params"])
    assert float(r0["loss0"]) == float(r1["loss0"])
    scale = float(np.abs(one["grads"]).max())
    assert np.max(np.abs(r0["grads"].astype(np.float64) - one["grads"])) <= 1e-4 * max(1.0, scale)
    assert_close(r0["loss0"], one["loss0"], 1e-5, "loss of the sharded batch")
    assert_close(r0["params"], one["params"], 1e-4, "weights after 5 SGD steps")
    assert_close(r0["loss"], one["loss"], 1e-4, "loss after 5 SGD steps")


def test_comm_init_fails_when_a_rank_never_joins(tmp_path):
    p = _spawn("lonely", tmp_path, 0, 1, _free_port(), {"NCCL_NVLS_ENABLE": "0"})
    _wait([p], timeout=120)
    res = json.loads((tmp_path / "lonely.json").read_text())
    assert res["error"] and "timed out" in res["error"], res
    assert res["waited"] < 30
    assert res["relu"] == [0.0, 2.0]
