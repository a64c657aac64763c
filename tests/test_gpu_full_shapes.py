"""The benchmark's largest single GEMMs at their full shapes against the
oracle's MatMul (internal/cpu/linalg.go:15-62 restated, fp32 accumulation)
on identical inputs, within the reference's device tolerance
|a-b| <= 1e-4 * max(1, |b|) (tensor/device_mps_test.go:19-21):

* the wide MLP's first-layer weight gradient, dW (4096 x 4096) = dY^T X over
  the whole batch of 8192 rows (the step's largest GEMM; on 148 SMs its 256
  output tiles take whole rounds plus a K-split tail);
* the conv stack's first-layer weight gradient at batch 1024, dW (64 x 27)
  over K = 1024 * 32 * 32 = 1,048,576 output positions, and its bias
  gradient (tensor/conv.go:40-59 backward: Permute, MatMul, sumTo).
"""
import ctypes

import numpy as np
import pytest

from gotensor import _lib
from gotensor._lib import check
from gpu_common import assert_close, cuda_backend
from oracle import gotensor_ref as T

pytestmark = pytest.mark.gpu

_keep = []


@pytest.fixture(autouse=True)
def _keep_alive():
    yield
    cuda_backend().Sync()
    _keep.clear()


def dev(a):
    s = cuda_backend().FromHost(np.ascontiguousarray(a))
    _keep.append(s)
    return s


def new(n, dt=T.Float32):
    s = cuda_backend().Zeros(dt, n)
    _keep.append(s)
    return s


def test_wide_mlp_first_layer_weight_gradient_full_shape():
    """dY carries the mean loss's 1/B factor, as every gradient of the step
    does. Unscaled N(0,1) operands would make the partial sums reach ~90, and
    the oracle's own sequential fp32 rounding (~K eps |partial sum|) would then
    exceed the 1e-4 floor by itself; the float64 check below holds the device
    to fp32-class error whatever the scale."""
    M, K, N = 8192, 4096, 4096  # batch, in, out
    rng = np.random.default_rng(21)
    x = rng.standard_normal((M, K)).astype(np.float32)
    dy = (rng.standard_normal((M, N)) / M).astype(np.float32)
    be = cuda_backend()
    dw, db = new(N * K), new(N)
    check(be.lib.gt_linear_bwd_weight(be.ctx.ptr, 0, dev(x).ptr, dev(dy).ptr, dw.ptr, db.ptr, M, K, N))
    got_w, got_b = be.ToHost(dw).reshape(N, K), be.ToHost(db)
    cpu = T.backend_for(T.CPU)
    # dW' (K, N) = X^T (K, M) @ dY (M, N), as the MatMul closure computes it
    # (tensor/ops.go:324-326); the Linear weight gradient is its transpose.
    want = cpu.ToHost(cpu.MatMul(cpu.FromHost(x.reshape(-1)), cpu.FromHost(dy.reshape(-1)), K, M, N, True, False))
    assert_close(got_w, want.reshape(K, N).T, 1e-4, "dW 4096x4096 over 8192 rows")
    want_b = cpu.ToHost(cpu.Reduce(0, cpu.FromHost(dy.reshape(-1)), 1, M, N))
    assert_close(got_b, want_b, 1e-4, "db over 8192 rows")
    # against the exact product: error relative to sum |dy||x| at fp32 level,
    # no worse than the oracle's own fp32 accumulation
    rows = rng.choice(N, 64, replace=False)  # 64 output rows (262,144 values) in float64
    exact = dy[:, rows].T.astype(np.float64) @ x.astype(np.float64)
    scale = np.abs(dy[:, rows]).T.astype(np.float64) @ np.abs(x).astype(np.float64)
    err = np.abs(got_w[rows] - exact) / scale
    err_oracle = np.abs(want.reshape(K, N).T[rows] - exact) / scale
    assert err.max() <= max(err_oracle.max(), 2.0 ** -20), (err.max(), err_oracle.max())


def test_conv_stack_first_conv_weight_gradient_full_batch():
    N, C, H, W, O, k = 1024, 3, 32, 32, 64, 3
    rng = np.random.default_rng(22)
    x = rng.standard_normal((N, C, H, W)).astype(np.float32)
    w = (rng.standard_normal((O, C, k, k)) / np.sqrt(C * k * k)).astype(np.float32)
    b = rng.standard_normal(O).astype(np.float32)
    dy = (rng.standard_normal((N, O, H, W)) / 1024).astype(np.float32)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, 1, 1)
    gg = _lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_])
    be = cuda_backend()
    dw, db = new(O * C * k * k), new(O)
    check(be.lib.gt_conv_bwd_weight(be.ctx.ptr, 0, dev(x).ptr, dev(dy).ptr, dw.ptr, db.ptr, ctypes.byref(gg), O))
    got_w, got_b = be.ToHost(dw), be.ToHost(db)
    T.SetDefaultDType(T.Float32)
    xs = T.FromFloat64(x.astype(np.float64).reshape(-1), N, C, H, W).ToDType(T.Float32)
    ws = T.FromFloat64(w.astype(np.float64).reshape(-1), O, C, k, k).ToDType(T.Float32).SetRequiresGrad(True)
    bs = T.FromFloat64(b.astype(np.float64), O).ToDType(T.Float32).SetRequiresGrad(True)
    T.Conv2d(xs, ws, bs, 1, 1).Backward(T.FromFloat64(dy.astype(np.float64).reshape(-1), N, O, H, W).ToDType(T.Float32))
    # dW sums 1,048,576 products of magnitude ~1e-3: compare at the reference's
    # tolerance and, more tightly, relative to the largest weight gradient
    want_w, want_b = ws.Grad().Float64s(), bs.Grad().Float64s()
    assert_close(got_w, want_w, 1e-4, "conv1 dW over 1,048,576 positions")
    assert_close(got_b, want_b, 1e-4, "conv1 db over 1,048,576 positions")
    scale = np.abs(want_w).max()
    assert np.max(np.abs(got_w - want_w)) <= 1e-4 * scale
