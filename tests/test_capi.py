"""The C interfaces load and export every entry point their headers declare,
and the host-only parts of the runtime behave (no GPU needed)."""
import os
import re

import pytest

from gotensor import _lib
from gotensor.model import bucket_plan

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
