"""The C interfaces load and export every entry point their headers declare,
and the host-only parts of the runtime behave (no GPU needed)."""
import os
import re

import pytest

from gotensor import _lib
from gotensor.model import bucket_plan, row_chunk_plan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    return set(re.findall(r"^GT_API\s+[\w\s\*]+?\b(gth?_\w+)\s*\(", text, flags=re.M))


@pytest.mark.parametrize("header,loader,prefix", [("gt_cuda.h", _lib.cuda_lib, "gt_"),
                                                  ("gt_host.h", _lib.host_lib, "gth_")])
def test_library_exports_every_declared_symbol(header, loader, prefix):
    names = declared(header)
    assert len(names) > 20
    lib = loader()
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    api = _lib.CUDA_API if prefix == "gt_" else _lib.HOST_API
    assert names == set(api), (names ^ set(api))


def test_bucket_plan_covers_buffer_in_backward_order():
    sizes = [4096 * 4096, 4096, 4096 * 4096, 4096, 1000 * 4096, 1024]
    plan = bucket_plan(sizes, 6_500_000)
    total = sum(sizes)
    # contiguous, disjoint, from the end of the buffer to its start
    assert plan[0][1] == total and plan[-1][0] == 0
    for (lo, hi), (lo2, hi2) in zip(plan, plan[1:]):
        assert hi2 == lo and lo < hi
    # boundaries fall on tensor boundaries
    edges = {0}
    acc = 0
    for s in sizes:
        acc += s
        edges.add(acc)
    assert all(lo in edges and hi in edges for lo, hi in plan)
    # every bucket except the first-layer one reaches the size
    assert all(hi - lo >= 6_500_000 for lo, hi in plan[:-1])


def test_bucket_plan_single_bucket_and_tiny_sizes():
    assert bucket_plan([10, 20, 30], 1 << 30) == [(0, 60)]
    assert bucket_plan([10, 20, 30], 1) == [(30, 60), (10, 30), (0, 10)]
    assert bucket_plan([], 5) == []


def test_row_chunk_plan_splits_the_first_weight_bucket():
    """GT_DP_LAST_CHUNKS: the bucket that starts at the first Linear's weight is
    cut at row chunks; the chunk buckets tile it exactly, highest rows first,
    and the first of them keeps the bias that follows the weight."""
    # the data-parallel test model: Linear(256,512), Linear(512,512), Linear(512,100)
    # (each tensor padded to 64 elements, as the runtime lays them out)
    sizes = [512 * 256, 512, 512 * 512, 512, 100 * 512, 128]
    buckets = bucket_plan(sizes, (256 << 10) // 4)
    w_off, N, K = 0, 512, 256
    rows, plan = row_chunk_plan(buckets, w_off, N, K, 4)
    assert rows == [0, 128, 256, 384, 512]
    first = [b for b in buckets if b[0] == w_off][0]
    chunk_buckets = plan[len(buckets) - 1:]
    assert plan[:len(buckets) - 1] == [b for b in buckets if b[0] != w_off]
    assert chunk_buckets == [(w_off + 384 * K, first[1]), (w_off + 256 * K, w_off + 384 * K),
                             (w_off + 128 * K, w_off + 256 * K), (w_off, w_off + 128 * K)]
    assert first[1] > w_off + N * K  # the bias sits in the first chunk bucket issued
    # contiguous and covering the buffer
    assert plan[0][1] == sum(sizes) and plan[-1][0] == 0
    for (lo, hi), (lo2, hi2) in zip(plan, plan[1:]):
        assert hi2 == lo and lo < hi


@pytest.mark.parametrize("N,chunks,want", [(4096, 4, [0, 1024, 2048, 3072, 4096]),
                                           (4096, 3, [0, 1280, 2560, 3840, 4096]),
                                           (100, 2, [0, 32, 64, 96, 100])])
def test_row_chunk_plan_rounds_rows_to_tiles(N, chunks, want):
    rows, plan = row_chunk_plan([(0, N * 8 + 64)], 0, N, 8, chunks)
    assert rows == want
    assert plan[0] == (want[-2] * 8, N * 8 + 64) and plan[-1] == (0, want[1] * 8)


def test_row_chunk_plan_leaves_other_plans_alone():
    assert row_chunk_plan([(0, 100)], 0, 64, 1, 1) == ([], [(0, 100)])      # one chunk
    assert row_chunk_plan([(10, 100)], 0, 64, 1, 4) == ([], [(10, 100)])    # no bucket starts at the weight
    assert row_chunk_plan([(0, 1000)], 0, 16, 8, 4) == ([], [(0, 1000)])   # fewer rows than one chunk
