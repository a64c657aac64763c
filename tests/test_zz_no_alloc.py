"""gt_xent_fwd_bwd_noalloc: the softmax cross-entropy for callers that cannot
allocate device memory during a step (for example a host whose own allocator
already holds the GPU's memory). It must give the same loss and gradients as
gt_xent_fwd_bwd, call after call, using only its built-in row buffer.

This file is collected last on purpose; it sets up its own device context, so
it also passes when run alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from gotensor import _lib
from gotensor._lib import FLOAT32, FLOAT64, GTError, check
from gotensor.backend import CudaBackend

pytestmark = pytest.mark.gpu


def _pool_usage(be):
    used, reserved = ctypes.c_uint64(), ctypes.c_uint64()
    be.Sync()
    check(_lib.cuda_lib().gt_pool_usage(be.ctx.ptr, ctypes.byref(used), ctypes.byref(reserved)))
    return used.value, reserved.value


def _run(be, fn, x_dev, labels_dev, B, C, dt, loss, dl):
    check(fn(be.ctx.ptr, dt, x_dev.ptr, labels_dev, B, C, loss.ptr, dl.ptr, None))
    be.Sync()
    return be.ToHost(loss), be.ToHost(dl)


@pytest.mark.parametrize("dt,npdt", [(FLOAT32, np.float32), (FLOAT64, np.float64)])
def test_noalloc_matches_pool_variant_on_consecutive_calls(dt, npdt):
    be = CudaBackend(0)
    lib = _lib.cuda_lib()
    rng = np.random.default_rng(4)
    # two calls in a row, the second smaller than the first: leftovers of the
    # first call in the shared buffer must not reach the second result
    for B, C in ((8192, 1000), (64, 10)):
        x = be.FromHost((rng.standard_normal((B, C)) * 3).astype(npdt))
        y = rng.integers(0, C, B).astype(np.int32)
        labels = be.ctx.alloc(4 * B)
        check(lib.gt_upload(be.ctx.ptr, labels, y.ctypes.data, 4 * B))
        loss, dl = be.Zeros(dt, 1), be.Zeros(dt, B * C)
        want_loss, want_dl = _run(be, lib.gt_xent_fwd_bwd, x, labels, B, C, dt, loss, dl)
        # the same two kernels on the same inputs: identical bits, and the
        # pool neither hands out nor grows by a byte during the call
        es = 4 if dt == FLOAT32 else 8
        check(lib.gt_zero(be.ctx.ptr, loss.ptr, es))  # so a call that wrote nothing cannot pass
        check(lib.gt_zero(be.ctx.ptr, dl.ptr, es * B * C))
        before = _pool_usage(be)
        got_loss, got_dl = _run(be, lib.gt_xent_fwd_bwd_noalloc, x, labels, B, C, dt, loss, dl)
        assert _pool_usage(be) == before
        assert got_loss.tobytes() == want_loss.tobytes()
        assert got_dl.tobytes() == want_dl.tobytes()
        be.ctx.release(labels)


def test_noalloc_rejects_batches_beyond_its_buffer():
    be = CudaBackend(0)
    lib = _lib.cuda_lib()
    too_many = 262144 + 1  # GT_XENT_NOALLOC_MAX_ROWS + 1
    err = lib.gt_xent_fwd_bwd_noalloc(be.ctx.ptr, FLOAT32, None, None, too_many, 10, None, None, None)
    with pytest.raises(GTError, match="exceeds"):
        check(err)
    be.Sync()  # nothing was launched; the context is still healthy
