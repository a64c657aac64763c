"""Host side of data parallelism (gotensor/dist.py) on CPU ranks: two gloo
processes stand in for two GPUs. Covers the shard split, the communicator id
exchange, the max-over-ranks timing reduction, and a rank that leaves before
the exchange: the surviving rank must fail within the process group's
timeout instead of waiting forever."""
import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp

from gotensor import dist as gd


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _ranks_agree(rank, world, port, out):
    dist = _init(rank, world, port)
    r, w, local = gd.env_ranks()
    uid = gd.exchange_unique_id(r, make_id=lambda: bytes(range(128)))
    lo, hi = gd.shard(8192, r, w)
    t = gd.max_over_ranks(10.0 * (r + 1))
    gd.barrier()
    out.put((r, w, local, uid, lo, hi, t))
    dist.destroy_process_group()


def _one_rank_leaves(rank, world, port, out):
    dist = _init(rank, world, port, timeout_s=5)
    if rank == 1:
        out.put((1, "left"))
        return  # exits without joining the exchange
    try:
        gd.exchange_unique_id(rank, make_id=lambda: bytes(128))
        out.put((0, "no error"))
    except Exception as e:  # gloo reports the lost peer or the timeout
        out.put((0, type(e).__name__))


def _run(fn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank did not exit")
    return sorted(res, key=lambda x: x[0])


def test_two_ranks_share_id_shards_and_max():
    res = _run(_ranks_agree, 2)
    assert [r[:3] for r in res] == [(0, 2, 0), (1, 2, 1)]
    assert res[0][3] == res[1][3] == bytes(range(128))
    assert [(r[4], r[5]) for r in res] == [(0, 4096), (4096, 8192)]
    assert res[0][6] == res[1][6] == 20.0


def test_surviving_rank_fails_when_a_peer_leaves():
    res = _run(_one_rank_leaves, 2)
    assert res[1] == (1, "left")
    assert res[0][1] != "no error"


def test_shard_validation():
    assert gd.shard(8192, 7, 8) == (7168, 8192)
    with pytest.raises(ValueError):
        gd.shard(8192, 0, 3)  # uneven split
    with pytest.raises(ValueError):
        gd.shard(8192, 2, 2)
    with pytest.raises(ValueError):
        gd.shard(0, 0, 1)


def test_env_ranks_defaults_and_validation(monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    assert gd.env_ranks() == (0, 1, 0)
    monkeypatch.setenv("RANK", "3")
    monkeypatch.setenv("WORLD_SIZE", "2")
    with pytest.raises(ValueError):
        gd.env_ranks()
