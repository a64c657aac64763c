"""The tcgen05 3xTF32 GEMM (forced path) against the oracle's fp32 matmul and,
at sizes the CPU oracle cannot finish quickly, against float64 host products
with an fp32-class error bound."""
import numpy as np
import pytest

from gotensor import _lib
from gpu_common import assert_close, cpu_backend, cuda_backend
from oracle import gotensor_ref as T

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _force_tc():
    lib = _lib.cuda_lib()
    lib.gt_debug_set_gemm_path(2)
    yield
    lib.gt_debug_set_gemm_path(0)


def run(m, k, n, ta, tb, rng, weight_like=True):
    # activations ~N(0,1); the other operand scaled like a Linear weight,
    # U(+-1/sqrt(k)) (nn/module.go:43-49), so outputs are O(1) as in training
    a = rng.standard_normal(m * k).astype(np.float32)
    if weight_like:
        b = rng.uniform(-1, 1, k * n).astype(np.float32) / np.float32(np.sqrt(k))
    else:
        b = rng.standard_normal(k * n).astype(np.float32)
    be = cuda_backend()
    ga, gb = be.FromHost(a), be.FromHost(b)
    got = be.ToHost(be.MatMul(ga, gb, m, k, n, ta, tb))
    assert _lib.cuda_lib().gt_gemm_path_taken() == 2
    return a, b, got


@pytest.mark.parametrize("mkn", [(128, 32, 128), (128, 8, 128), (1, 4, 1), (130, 36, 132), (256, 1000, 384),
                                 (64, 784, 128), (300, 1028, 10), (517, 96, 260)])
@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
def test_tc_matches_oracle(mkn, ta, tb):
    m, k, n = mkn
    # TMA needs every row pitch to be a multiple of 16 bytes
    if (ta and m % 4) or (not ta and k % 4) or (tb and k % 4) or (not tb and n % 4):
        pytest.skip("row pitch not a multiple of 16 bytes (the dispatcher uses SIMT there)")
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a, b, got = run(m, k, n, ta, tb, rng)
    want = cpu_backend().MatMul(T.CPUStorage(a), T.CPUStorage(b), m, k, n, ta, tb).data
    assert_close(got, want, 1e-4, f"tc {mkn} ta={ta} tb={tb}")


@pytest.mark.parametrize("mkn", [(4096, 4096, 1024), (1024, 8192, 4096), (8192, 1000, 512), (256, 1000, 384),
                                 (1024, 4096, 1000),  # 16 tiles: every tile in 4 K-splits
                                 (4096, 8192, 4096)])  # 256 tiles: the last round's 34 tiles in 2 K-splits
@pytest.mark.parametrize("ta,tb", [(False, True), (False, False), (True, False)])
def test_tc_large_against_float64(mkn, ta, tb):
    """The three operand layouts of a Linear layer's forward, dX and dW GEMMs at
    wide-MLP sizes, on unscaled N(0,1) operands (outputs ~sqrt(k) with heavy
    cancellation): the error vs the exact (float64) product, relative to
    sum |a||b|, stays at fp32 level, no worse than a plain fp32 dot product."""
    m, k, n = mkn
    rng = np.random.default_rng(m + k + n)
    a, b, got = run(m, k, n, ta, tb, rng, weight_like=False)
    A = a.reshape(k, m).T if ta else a.reshape(m, k)
    B = b.reshape(n, k).T if tb else b.reshape(k, n)
    exact = A.astype(np.float64) @ B.astype(np.float64)
    scale = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64)
    err = np.abs(got.reshape(m, n) - exact) / scale
    # fp32 reference: the same product with fp32 accumulation (numpy/BLAS sgemm)
    err32 = np.abs((A @ B).astype(np.float64) - exact) / scale
    assert err.max() <= max(4 * err32.max(), 2.0 ** -20), (err.max(), err32.max())


def test_tc_special_values_and_accuracy_beyond_tf32():
    """Values that tf32 alone cannot represent: 3xTF32 must recover them."""
    m = k = n = 128
    a = np.full(m * k, 1.0 + 2.0 ** -20, dtype=np.float32)
    b = np.full(k * n, 1.0 - 2.0 ** -21, dtype=np.float32)
    be = cuda_backend()
    got = be.ToHost(be.MatMul(be.FromHost(a), be.FromHost(b), m, k, n, False, False))
    exact = k * (1.0 + 2.0 ** -20) * (1.0 - 2.0 ** -21)
    assert np.abs(got - exact).max() <= 2 * np.spacing(np.float32(exact)), (got[0], exact)


def test_gemm_timer_records_each_launch_outside_capture():
    import ctypes
    from gotensor._lib import GTError, check
    lib = _lib.cuda_lib()
    be = cuda_backend()
    ctx = be.ctx.ptr
    rng = np.random.default_rng(9)
    a = be.FromHost(rng.standard_normal(256 * 512).astype(np.float32))
    b = be.FromHost(rng.standard_normal(512 * 384).astype(np.float32))
    check(lib.gt_gemm_timer_start(ctx, 2))
    try:
        for _ in range(3):  # the third is beyond the capacity: counted as dropped
            be.MatMul(a, b, 256, 512, 384, False, False)
        n, dropped = ctypes.c_int64(), ctypes.c_int64()
        check(lib.gt_gemm_timer_count(ctx, ctypes.byref(n), ctypes.byref(dropped)))
        assert (n.value, dropped.value) == (2, 1)
        mnk, path, ms = (ctypes.c_int64 * 3)(), ctypes.c_int(), ctypes.c_float()
        for i in range(2):
            check(lib.gt_gemm_timer_read(ctx, i, mnk, ctypes.byref(path), ctypes.byref(ms)))
            assert tuple(mnk) == (256, 384, 512) and path.value == 2 and ms.value > 0
        with pytest.raises(GTError, match="launch 2 of 2"):
            check(lib.gt_gemm_timer_read(ctx, 2, mnk, ctypes.byref(path), ctypes.byref(ms)))
        # a GEMM recorded into a graph is not timed (its events would only
        # hold the last replay)
        check(lib.gt_gemm_timer_start(ctx, 4))
        out = be.Zeros(_lib.FLOAT32, 256 * 384)
        check(lib.gt_capture_begin(ctx))
        err = lib.gt_matmul(ctx, _lib.FLOAT32, a.ptr, b.ptr, out.ptr, 256, 512, 384, 0, 0)
        g = ctypes.c_void_p()
        check(lib.gt_capture_end(ctx, ctypes.byref(g)))
        check(err)
        check(lib.gt_graph_launch(ctx, g))
        be.Sync()
        lib.gt_graph_free(g)
        check(lib.gt_gemm_timer_count(ctx, ctypes.byref(n), ctypes.byref(dropped)))
        assert (n.value, dropped.value) == (0, 0)
    finally:
        check(lib.gt_gemm_timer_stop(ctx))
    with pytest.raises(GTError, match="no timer"):
        check(lib.gt_gemm_timer_count(ctx, None, None))


def _f64_error(a, b, got, m, k, n, ta, tb):
    A = a.reshape(k, m).T if ta else a.reshape(m, k)
    B = b.reshape(n, k).T if tb else b.reshape(k, n)
    exact = A.astype(np.float64) @ B.astype(np.float64)
    scale = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64)
    err = np.abs(got.reshape(m, n) - exact) / scale
    err32 = np.abs((A @ B).astype(np.float64) - exact) / scale
    return err.max(), err32.max()


@pytest.mark.parametrize("splits", [2, 3, 8])
@pytest.mark.parametrize("ta,tb", [(False, True), (False, False), (True, False)])
def test_tc_split_k_against_float64_and_deterministic(splits, ta, tb):
    """K-split GEMMs (partials over consecutive K ranges, summed in split
    order): fp32-class error, and the same bits on every run whatever the
    order in which the units finish."""
    lib = _lib.cuda_lib()
    lib.gt_debug_set_gemm_splits(splits)
    try:
        m, k, n = 300, 4096, 520
        rng = np.random.default_rng(splits)
        a, b, got = run(m, k, n, ta, tb, rng, weight_like=False)
        err, err32 = _f64_error(a, b, got, m, k, n, ta, tb)
        assert err <= max(4 * err32, 2.0 ** -20), (err, err32)
        be = cuda_backend()
        ga, gb = be.FromHost(a), be.FromHost(b)
        for _ in range(2):
            again = be.ToHost(be.MatMul(ga, gb, m, k, n, ta, tb))
            assert np.array_equal(again, got)
    finally:
        lib.gt_debug_set_gemm_splits(0)


@pytest.mark.parametrize("splits", [2, 4])
def test_fused_epilogues_under_split_k(splits):
    """The fused Linear/Conv2d entry points when their GEMM is K-split: the
    bias, activation, derivative mask and NCHW order are applied once, to the
    summed result (checked against the oracle's op chains)."""
    import test_gpu_fused as F
    lib = _lib.cuda_lib()
    lib.gt_debug_set_gemm_splits(splits)
    try:
        F.test_linear_fwd(T.Float32, np.float32, 1e-4, 1, (257, 1024, 300))  # bias + ReLU
        F.test_linear_fwd(T.Float32, np.float32, 1e-4, 3, (64, 784, 128))  # sigmoid (generic epilogue)
        F.test_linear_bwd(T.Float32, np.float32, 1e-4, 1, (257, 1024, 300))  # ReLU mask on dX; dW
        F.test_conv_fwd_bwd(T.Float32, np.float32, 1e-4, (4, 32, 14, 14, 64, 3, 1, 1))  # NCHW store, bias by row
    finally:
        lib.gt_debug_set_gemm_splits(0)
        cuda_backend().Sync()
        F._keep.clear()


def test_sm_reserve_leaves_results_unchanged():
    """GEMMs launched with SMs reserved for other streams (the all-reduce of
    data parallelism) run on fewer SM pairs, in more rounds, with the same
    bits; an out-of-range reserve is refused."""
    from gotensor._lib import GTError, check
    lib = _lib.cuda_lib()
    be = cuda_backend()
    rng = np.random.default_rng(21)
    m, k, n = 2048, 512, 2048  # 64 tiles, no K-split either way
    a = be.FromHost(rng.standard_normal(m * k).astype(np.float32))
    b = be.FromHost(rng.standard_normal(k * n).astype(np.float32))
    want = be.ToHost(be.MatMul(a, b, m, k, n, False, False))
    try:
        for sms in (20, 100):
            check(lib.gt_set_gemm_sm_reserve(be.ctx.ptr, sms))
            got = be.ToHost(be.MatMul(a, b, m, k, n, False, False))
            assert np.array_equal(got, want), sms
        with pytest.raises(GTError, match="SMs"):
            check(lib.gt_set_gemm_sm_reserve(be.ctx.ptr, 10_000))
    finally:
        check(lib.gt_set_gemm_sm_reserve(be.ctx.ptr, 0))


def test_timed_out_wait_returns_an_error_and_the_context_recovers():
    """The error path of the tcgen05 GEMM's bounded barrier waits. With the
    wait limit lowered to 20 ms, one splitter warp per SM pair withholds its
    arrival for the first K-slice (a barrier that nothing completes): the MMA
    issuer's wait runs out, every other wait follows, the kernel frees its
    tensor memory and returns. gt_sync reports the timed-out site, and the
    next GEMM on the same context is correct. Nothing traps or hangs."""
    import time

    from gotensor._lib import GTError
    lib = _lib.cuda_lib()
    be = cuda_backend()
    be.Sync()
    rng = np.random.default_rng(9)
    m = k = n = 512
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    ga, gb = be.FromHost(a), be.FromHost(b)
    lib.gt_debug_set_tc_wait_limit_us(20000)
    try:
        lib.gt_debug_tc_withhold_arrive()
        t0 = time.time()
        be.MatMul(ga, gb, m, k, n, False, False)
        with pytest.raises(GTError, match=r"pipeline wait timed out \(site \d\)"):
            be.Sync()
        assert time.time() - t0 < 10
        be.Sync()  # the error was reported once and cleared
    finally:
        lib.gt_debug_set_tc_wait_limit_us(0)
    got = be.ToHost(be.MatMul(ga, gb, m, k, n, False, False))
    assert lib.gt_gemm_path_taken() == 2
    want = cpu_backend().MatMul(T.CPUStorage(a), T.CPUStorage(b), m, k, n, False, False).data
    assert_close(got, want, 1e-4, "GEMM after the timed-out one")


def test_timed_out_wait_in_the_tensor_memory_conv_kernel():
    """The same error path in the implicit convolution whose gathered A
    operand goes to tensor memory (a 64-wide input gradient: four gather
    warps per CTA, pairs of slices per barrier round, 512 tensor-memory
    columns). The leader CTA's gather warps withhold their arrival for the
    first round; the MMA issuer's wait runs out, the kernel frees its tensor
    memory and returns, gt_sync reports the site, and the same convolution
    then gives its earlier result bit for bit."""
    import ctypes
    import time

    from gotensor._lib import GTError, check
    lib = _lib.cuda_lib()
    be = cuda_backend()
    be.Sync()
    N, C, H, W, O = 4, 64, 16, 16, 128
    g = T.conv_geom("Conv2d", [N, C, H, W], 3, 3, 1, 1)
    gg = ctypes.byref(_lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_]))
    rng = np.random.default_rng(10)
    dy = be.FromHost(rng.standard_normal(N * O * H * W).astype(np.float32))
    w = be.FromHost(rng.standard_normal(O * C * 9).astype(np.float32))
    dx = be.Zeros(T.Float32, N * C * H * W)

    def run():
        check(lib.gt_conv_bwd_data(be.ctx.ptr, 0, dy.ptr, w.ptr, dx.ptr, gg, O))
        assert lib.gt_gemm_path_taken() == 4

    run()
    want = be.ToHost(dx)
    lib.gt_debug_set_tc_wait_limit_us(20000)
    try:
        lib.gt_debug_tc_withhold_arrive()
        t0 = time.time()
        run()
        with pytest.raises(GTError, match=r"pipeline wait timed out \(site \d\)"):
            be.Sync()
        assert time.time() - t0 < 10
        be.Sync()
    finally:
        lib.gt_debug_set_tc_wait_limit_us(0)
    run()
    assert np.array_equal(be.ToHost(dx), want)
