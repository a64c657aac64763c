"""The fused entry points of gt_cuda.h against the chains of reference ops
they replace, computed by the oracle on identical inputs."""
import ctypes

import numpy as np
import pytest

from gotensor import _lib
from gotensor._lib import AdamCfg, SgdCfg, check
from gpu_common import assert_bits, assert_close, cuda_backend
from oracle import gotensor_ref as T
from oracle import nn_ref as nn

pytestmark = pytest.mark.gpu

ACTS = {0: None, 1: "ReLU", 2: "Tanh", 3: "Sigmoid"}
DT = [(T.Float32, np.float32, 1e-4), (T.Float64, np.float64, 1e-10)]


def lib():
    return cuda_backend().lib


def ctx():
    return cuda_backend().ctx.ptr


_keep = []  # device storages must outlive the asynchronous calls that use them


@pytest.fixture(autouse=True)
def _keep_alive():
    yield
    cuda_backend().Sync()
    _keep.clear()


def dev(a):
    s = cuda_backend().FromHost(np.ascontiguousarray(a))
    _keep.append(s)
    return s


def host(s):
    return cuda_backend().ToHost(s)


def new(n, dt):
    s = cuda_backend().Zeros(dt, n)
    _keep.append(s)
    return s


def ref(a, *shape):
    return T.FromFloat64(np.asarray(a, dtype=np.float64).reshape(-1), *shape).ToDType(
        T.Float32 if np.asarray(a).dtype == np.float32 else T.Float64)


def apply_act(t, act):
    return t if act == 0 else getattr(t, ACTS[act])()


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("act", [0, 1, 2, 3])
# the last four: classifiers (N <= 32 runs the thin kernel: a warp per row)
@pytest.mark.parametrize("mkn", [(64, 784, 128), (257, 129, 65), (1024, 512, 1000), (5, 3, 7), (4096, 1024, 10),
                                 (256, 128, 10), (1000, 2048, 10), (100, 64, 20)])
def test_linear_fwd(dt, npdt, tol, act, mkn):
    M, K, N = mkn
    rng = np.random.default_rng(M + K + N)
    x = rng.standard_normal((M, K)).astype(npdt)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(npdt)
    b = rng.standard_normal(N).astype(npdt)
    y = new(M * N, dt)
    check(lib().gt_linear_fwd(ctx(), dt, dev(x).ptr, dev(w).ptr, dev(b).ptr, y.ptr, M, K, N, act))
    with T.no_grad():
        want = apply_act(ref(x, M, K).MatMul(ref(w, N, K).T()).Add(ref(b, N)), act).Float64s()
    assert_close(host(y), want, tol, f"linear fwd act={act}")


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("act_prev", [0, 1, 2, 3])
# the last three: classifiers (dW with 10 or 20 rows runs the thin kernel: a
# thread per column, K split, partials added in order)
@pytest.mark.parametrize("mkn", [(64, 784, 128), (257, 129, 65), (512, 1024, 1000), (4096, 1024, 10), (64, 128, 10),
                                 (300, 96, 20)])
def test_linear_bwd(dt, npdt, tol, act_prev, mkn):
    M, K, N = mkn
    rng = np.random.default_rng(M * 3 + K + N)
    x = rng.standard_normal((M, K)).astype(npdt)
    yprev = apply_act(ref(x, M, K), act_prev).Float64s().astype(npdt).reshape(M, K)  # an activation output
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(npdt)
    # gradients of a mean loss scale like 1/batch
    dy = (rng.standard_normal((M, N)) / np.sqrt(M)).astype(npdt)
    dx, dw, db = new(M * K, dt), new(N * K, dt), new(N, dt)
    check(lib().gt_linear_bwd_data(ctx(), dt, dev(dy).ptr, dev(w).ptr, dev(yprev).ptr, act_prev, dx.ptr, M, K, N))
    check(lib().gt_linear_bwd_weight(ctx(), dt, dev(yprev).ptr, dev(dy).ptr, dw.ptr, db.ptr, M, K, N))
    with T.no_grad():
        g = ref(dy, M, N).MatMul(ref(w, N, K))  # dX = dY @ W (tensor/ops.go:321-323)
        y = ref(yprev, M, K)
        if act_prev == 1:
            g = g.Mul(y._raw(T.STEP, 0.0))
        elif act_prev == 2:
            g = g.Mul(y.Mul(y).Neg().AddScalar(1))
        elif act_prev == 3:
            g = g.Mul(y.Mul(y.Neg().AddScalar(1)))
        want_dx = g.Float64s()
        want_dw = ref(yprev, M, K).T().MatMul(ref(dy, M, N)).T().Float64s()  # Permute backward of W.T()
        want_db = ref(dy, M, N).SumDim(0, False).Float64s()
    assert_close(host(dx), want_dx, tol, "dx")
    assert_close(host(dw), want_dw, tol, "dw")
    assert_close(host(db), want_db, tol, "db")


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("mkn_rows", [(1024, 512, 1024, (0, 256, 512, 768, 1024)), (64, 27, 50, (0, 20, 50)),
                                      (300, 130, 257, (0, 256, 257))])
def test_linear_bwd_weight_rows(dt, npdt, tol, mkn_rows):
    """gt_linear_bwd_weight_rows over consecutive row ranges rebuilds the
    weight gradient of gt_linear_bwd_weight (the chunks may take other
    K-split plans, so equal within the device tolerance), and leaves rows
    outside its range untouched."""
    M, K, N, rows = mkn_rows
    rng = np.random.default_rng(M + K + N)
    x = dev(rng.standard_normal((M, K)).astype(npdt))
    dy = dev((rng.standard_normal((M, N)) / np.sqrt(M)).astype(npdt))
    dw_full, dw = new(N * K, dt), new(N * K, dt)
    check(lib().gt_linear_bwd_weight(ctx(), dt, x.ptr, dy.ptr, dw_full.ptr, None, M, K, N))
    for r0, r1 in zip(rows[:-1], rows[1:]):
        check(lib().gt_linear_bwd_weight_rows(ctx(), dt, x.ptr, dy.ptr, dw.ptr, M, K, N, r0, r1))
        got = host(dw).reshape(N, K)
        assert (got[r1:] == 0).all(), "rows past the range were written"
    assert_close(host(dw), host(dw_full), tol, "dw by rows")


def _relu_bits(y, M, N):
    """Word (b, n) holds bit j = (y[32 b + j, n] > 0): ceil(M / 32) rows of N words."""
    nb = (M + 31) // 32
    pos = np.zeros((nb * 32, N), dtype=np.uint64)
    pos[:M] = np.asarray(y).reshape(M, N) > 0
    return (pos.reshape(nb, 32, N) << np.arange(32, dtype=np.uint64)[None, :, None]).sum(axis=1).astype(np.uint32)


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("mkn2", [(2048, 512, 1024, 96), (256, 8192, 256, 4096), (64, 27, 50, 40),
                                  (257, 129, 65, 33), (1, 5, 33, 7)])
def test_relu_bits_forward_and_dx(dt, npdt, tol, mkn2):
    """gt_linear_fwd_bits stores what gt_linear_fwd with ReLU stores, plus the
    bits (y > 0) (NaN gives 0); gt_relu_bits packs the same bits; and the next
    layer's gt_linear_bwd_data_bits equals gt_linear_bwd_data with the ReLU
    output, bit for bit. The shapes take the tensor-core path whole and
    K-split (forward and dX), and the SIMT path (K = 27 or 129), with word
    rows that end mid-word; NaN and infinities come in through the bias."""
    M, K, N, N2 = mkn2
    rng = np.random.default_rng(M + 2 * K + N)
    x = rng.standard_normal((M, K)).astype(npdt)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(npdt)
    b = rng.standard_normal(N).astype(npdt)
    b[1:4] = [np.nan, -np.inf, np.inf]
    ldw = (M + 31) // 32
    y1, y2 = new(M * N, dt), new(M * N, dt)
    bits, bits2 = new(N * ldw, T.Float32), new(N * ldw, T.Float32)  # 4-byte words
    xd, wd, bd = dev(x), dev(w), dev(b)
    check(lib().gt_linear_fwd(ctx(), dt, xd.ptr, wd.ptr, bd.ptr, y1.ptr, M, K, N, 1))
    check(lib().gt_linear_fwd_bits(ctx(), dt, xd.ptr, wd.ptr, bd.ptr, y2.ptr, bits.ptr, M, K, N))
    check(lib().gt_relu_bits(ctx(), dt, y1.ptr, bits2.ptr, M, N))
    y = host(y1)
    assert_bits(host(y2), y, "y")
    want_bits = _relu_bits(y, M, N)
    assert np.array_equal(host(bits).view(np.uint32).reshape(ldw, N), want_bits)
    assert np.array_equal(host(bits2).view(np.uint32).reshape(ldw, N), want_bits)
    # the next layer: dx (M, N) = dy (M, N2) @ w2 (N2, N) * Step(y)
    w2 = (rng.standard_normal((N2, N)) / np.sqrt(N)).astype(npdt)
    dy = (rng.standard_normal((M, N2)) / np.sqrt(M)).astype(npdt)
    dx1, dx2 = new(M * N, dt), new(M * N, dt)
    dyd, w2d = dev(dy), dev(w2)
    check(lib().gt_linear_bwd_data(ctx(), dt, dyd.ptr, w2d.ptr, y1.ptr, 1, dx1.ptr, M, N, N2))
    check(lib().gt_linear_bwd_data_bits(ctx(), dt, dyd.ptr, w2d.ptr, bits.ptr, dx2.ptr, M, N, N2))
    assert_bits(host(dx2), host(dx1), "dx")


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("kind", ["mse", "bce"])
@pytest.mark.parametrize("n", [1, 37, 4096, 1_000_003])
def test_fused_losses(dt, npdt, tol, kind, n):
    """gt_mse_fwd_bwd / gt_bce_fwd_bwd against the oracle's tape for MSELoss /
    BCELoss (nn/loss.go:6-22) and Backward: the gradient bit for bit for MSE
    and within the float64-log tolerance for BCE; the loss within the device
    tolerance (the sums run in different orders; a million float32 terms
    summed in sequence on the CPU carry ~1e-4 of error, so that size uses the
    reference's large-op tolerance 1e-3)."""
    rng = np.random.default_rng(n + 7 * (kind == "bce"))
    if kind == "bce":
        pred = (1 / (1 + np.exp(-rng.standard_normal(n)))).astype(npdt)
        target = rng.random(n).astype(npdt)
    else:
        pred = rng.standard_normal(n).astype(npdt)
        target = rng.standard_normal(n).astype(npdt)
    p = ref(pred, n).SetRequiresGrad(True)
    loss_t = (nn.MSELoss if kind == "mse" else nn.BCELoss)(p, ref(target, n))
    loss_t.Backward()
    loss, g = new(1, dt), new(n, dt)
    fn = lib().gt_mse_fwd_bwd if kind == "mse" else lib().gt_bce_fwd_bwd
    check(fn(ctx(), dt, dev(pred).ptr, dev(target).ptr, n, loss.ptr, g.ptr))
    want_g = p.Grad().Float64s().astype(npdt)
    if kind == "mse":
        assert_bits(host(g), want_g, "mse dpred")
    else:
        assert_close(host(g), want_g, 1e-6 if dt == T.Float32 else 1e-15, "bce dpred")
    lt = 1e-3 if (dt == T.Float32 and n > 4096) else tol
    assert_close(host(loss), loss_t.Float64s(), lt, f"{kind} loss")
    # the forward alone (dpred NULL) gives the same loss
    loss2 = new(1, dt)
    check(fn(ctx(), dt, dev(pred).ptr, dev(target).ptr, n, loss2.ptr, None))
    assert_bits(host(loss2), host(loss), "loss without gradient")


@pytest.mark.parametrize("fn", ["gt_mse_fwd_bwd", "gt_bce_fwd_bwd"])
def test_fused_losses_empty(fn):
    """Mean over no elements is 0 * (1/0) = NaN in the reference."""
    loss = new(1, T.Float32)
    check(getattr(lib(), fn)(ctx(), T.Float32, None, None, 0, loss.ptr, None))
    assert np.isnan(host(loss)[0])


# (N, C, H, W, O, k, stride, pad). The float32 implicit-GEMM paths (stride 1,
# position tiles that are rectangles of the output) cover tile widths 64 /
# 128 / 256 and two column tiles (O = 512), weights whose C*k*k is not a
# multiple of 4 (padded copies) and a 1x1 window; the other shapes (stride
# 2, 5x5 with 144 positions, 28 x 28 and 14 x 14 planes, ragged O) take the
# explicit im2col path.
CONVS = [(2, 3, 5, 5, 4, 3, 1, 0), (2, 2, 5, 4, 3, 3, 2, 1), (8, 1, 28, 28, 32, 3, 1, 1), (4, 32, 14, 14, 64, 3, 1, 1),
         (2, 3, 32, 32, 64, 3, 1, 1), (16, 64, 16, 16, 128, 3, 1, 1), (8, 128, 8, 8, 256, 3, 1, 1),
         (8, 256, 4, 4, 512, 3, 1, 1), (2, 5, 8, 6, 70, 3, 1, 1), (2, 4, 12, 12, 20, 5, 1, 2), (4, 16, 8, 8, 32, 1, 1, 0)]


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("cs", CONVS[:6])
def test_conv_cols_entry_points(dt, npdt, tol, cs):
    """gt_conv_fwd_cols keeps the columns gt_im2col builds (bit for bit) and
    stores the convolution; gt_conv_bwd from those columns gives the weight,
    bias and input gradients, the same bits with and without dx. These are the
    explicit-column algorithm (im2col, GEMM, col2im), so they are held to the
    oracle like the implicit-GEMM entry points, not to those bit for bit."""
    N, C, H, W, O, k, s, p = cs
    rng = np.random.default_rng(3 * sum(cs))
    x = rng.standard_normal((N, C, H, W)).astype(npdt)
    w = (rng.standard_normal((O, C, k, k)) / np.sqrt(C * k * k)).astype(npdt)
    b = rng.standard_normal(O).astype(npdt)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, s, p)
    gg = ctypes.byref(_lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_]))
    L, CKK = g.OH * g.OW, C * k * k
    xd, wd, bd = dev(x), dev(w), dev(b)
    y2, cols, cols_ref = new(N * O * L, dt), new(N * L * CKK, dt), new(N * L * CKK, dt)
    check(lib().gt_conv_fwd_cols(ctx(), dt, xd.ptr, wd.ptr, bd.ptr, y2.ptr, cols.ptr, gg, O, 1))
    check(lib().gt_im2col(ctx(), dt, xd.ptr, cols_ref.ptr, gg))
    assert_bits(host(cols), host(cols_ref), "cols")
    with T.no_grad():
        want = T.Conv2d(ref(x, N, C, H, W), ref(w, O, C, k, k), ref(b, O), s, p).ReLU().Float64s()
    assert_close(host(y2), want, tol, "conv fwd from columns")
    # dy at the scale a mean loss gives it (1/N per image): unscaled N(0,1)
    # gradients summed over N*OH*OW positions reach partial sums where the
    # oracle's own sequential rounding is ~1e-4 by itself
    dy = (rng.standard_normal((N, O, g.OH, g.OW)) / N).astype(npdt)
    dyd = dev(dy)
    dx2, dw2, db2, dw3 = new(N * C * H * W, dt), new(O * CKK, dt), new(O, dt), new(O * CKK, dt)
    check(lib().gt_conv_bwd(ctx(), dt, cols.ptr, dyd.ptr, wd.ptr, dx2.ptr, dw2.ptr, db2.ptr, gg, O))
    check(lib().gt_conv_bwd(ctx(), dt, cols.ptr, dyd.ptr, wd.ptr, None, dw3.ptr, None, gg, O))
    assert_bits(host(dw3), host(dw2), "dw without dx")
    xs, ws, bs = ref(x, N, C, H, W).SetRequiresGrad(True), ref(w, O, C, k, k).SetRequiresGrad(True), \
        ref(b, O).SetRequiresGrad(True)
    T.Conv2d(xs, ws, bs, s, p).Backward(ref(dy, N, O, g.OH, g.OW))
    assert_close(host(dx2), xs.Grad().Float64s(), tol, "conv dx from columns")
    assert_close(host(dw2), ws.Grad().Float64s(), tol, "conv dw from columns")
    assert_close(host(db2), bs.Grad().Float64s(), tol, "conv db from columns")


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("cs", CONVS)
def test_conv_fwd_bwd(dt, npdt, tol, cs):
    N, C, H, W, O, k, s, p = cs
    rng = np.random.default_rng(sum(cs))
    x = rng.standard_normal((N, C, H, W)).astype(npdt)
    w = (rng.standard_normal((O, C, k, k)) / np.sqrt(C * k * k)).astype(npdt)
    b = rng.standard_normal(O).astype(npdt)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, s, p)
    gg = _lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_])
    L = g.OH * g.OW
    for act in (0, 1):
        y = new(N * O * L, dt)
        check(lib().gt_conv_fwd(ctx(), dt, dev(x).ptr, dev(w).ptr, dev(b).ptr, y.ptr, ctypes.byref(gg), O, act))
        with T.no_grad():
            want = apply_act(T.Conv2d(ref(x, N, C, H, W), ref(w, O, C, k, k), ref(b, O), s, p), act).Float64s()
        assert_close(host(y), want, tol, f"conv fwd act={act}")
    dy = (rng.standard_normal((N, O, g.OH, g.OW)) / N).astype(npdt)  # the mean loss's scale, as above
    dx, dw, db = new(N * C * H * W, dt), new(O * C * k * k, dt), new(O, dt)
    check(lib().gt_conv_bwd_data(ctx(), dt, dev(dy).ptr, dev(w).ptr, dx.ptr, ctypes.byref(gg), O))
    check(lib().gt_conv_bwd_weight(ctx(), dt, dev(x).ptr, dev(dy).ptr, dw.ptr, db.ptr, ctypes.byref(gg), O))
    xs, ws, bs = ref(x, N, C, H, W).SetRequiresGrad(True), ref(w, O, C, k, k).SetRequiresGrad(True), \
        ref(b, O).SetRequiresGrad(True)
    T.Conv2d(xs, ws, bs, s, p).Backward(ref(dy, N, O, g.OH, g.OW))
    assert_close(host(dx), xs.Grad().Float64s(), tol, "conv dx")
    assert_close(host(dw), ws.Grad().Float64s(), tol, "conv dw")
    assert_close(host(db), bs.Grad().Float64s(), tol, "conv db")


@pytest.mark.parametrize("cs", [(2, 3, 32, 32, 64, 3, 1, 1), (4, 64, 16, 16, 128, 3, 1, 1), (4, 128, 8, 8, 256, 3, 1, 1),
                                (8, 256, 4, 4, 512, 3, 1, 1), (4, 16, 8, 8, 32, 1, 1, 0), (2, 8, 16, 16, 16, 5, 1, 2)])
def test_conv_implicit_against_float64(cs):
    """The float32 implicit-GEMM convolutions (forward, input and weight
    gradients, bias gradient) at the conv stack's layer shapes and a 1x1 and
    a 5x5 window,
    on unscaled N(0,1) data, against the exact (float64) results: the error,
    relative to the same sums over absolute values, stays at the level of a
    float32 dot product (the oracle's own float32 error is shown beside it)."""
    N, C, H, W, O, k, s, p = cs
    rng = np.random.default_rng(sum(cs) + 1)
    x = rng.standard_normal((N, C, H, W)).astype(np.float32)
    w = rng.standard_normal((O, C, k, k)).astype(np.float32)
    b = rng.standard_normal(O).astype(np.float32)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, s, p)
    gg = ctypes.byref(_lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_]))
    dy = rng.standard_normal((N, O, g.OH, g.OW)).astype(np.float32)
    y, dx, dw, db = new(N * O * g.OH * g.OW, T.Float32), new(N * C * H * W, T.Float32), new(O * C * k * k, T.Float32), \
        new(O, T.Float32)
    check(lib().gt_conv_fwd(ctx(), 0, dev(x).ptr, dev(w).ptr, dev(b).ptr, y.ptr, gg, O, 0))
    assert lib().gt_gemm_path_taken() == 4
    check(lib().gt_conv_bwd_data(ctx(), 0, dev(dy).ptr, dev(w).ptr, dx.ptr, gg, O))
    assert lib().gt_gemm_path_taken() == 4
    check(lib().gt_conv_bwd_weight(ctx(), 0, dev(x).ptr, dev(dy).ptr, dw.ptr, db.ptr, gg, O))
    assert lib().gt_gemm_path_taken() == 4

    def run(dt, absolute=False):
        def t(a, *shape):
            a = np.abs(a) if absolute else a
            return T.FromFloat64(a.astype(np.float64).reshape(-1), *shape).ToDType(dt).SetRequiresGrad(True)
        xs, ws, bs = t(x, N, C, H, W), t(w, O, C, k, k), t(b, O)
        out = T.Conv2d(xs, ws, bs, s, p)
        out.Backward(t(dy, N, O, g.OH, g.OW))
        return [out.Float64s(), xs.Grad().Float64s(), ws.Grad().Float64s(), bs.Grad().Float64s()]

    T.SetDefaultDType(T.Float64)
    try:
        exact, scale = run(T.Float64), run(T.Float64, absolute=True)
    finally:
        T.SetDefaultDType(T.Float32)
    oracle32 = run(T.Float32)
    for name, got, ex, sc, o32 in zip(("y", "dx", "dw", "db"), (host(y), host(dx), host(dw), host(db)), exact, scale,
                                      oracle32):
        err = np.abs(got.astype(np.float64) - ex) / np.maximum(sc, 1e-30)
        err32 = np.abs(o32 - ex) / np.maximum(sc, 1e-30)
        assert err.max() <= max(4 * err32.max(), 2.0 ** -20), (name, cs, float(err.max()), float(err32.max()))


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("ps", [(2, 3, 4, 6, 2), (8, 32, 28, 28, 2), (4, 64, 7, 7, 2), (2, 2, 9, 9, 3)])
def test_pool_idx_with_relu_mask_bit_exact(dt, npdt, tol, ps):
    N, C, H, W, k = ps
    g = T.conv_geom("MaxPool2d", [N, C, H, W], k, k, k, 0)
    gg = _lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_])
    rng = np.random.default_rng(H + C)
    z = rng.integers(-3, 4, (N, C, H, W)).astype(npdt)  # ties and non-positive windows
    relu = np.maximum(z, 0).astype(npdt)
    out, idx = new(N * C * g.OH * g.OW, dt), new(N * C * g.OH * g.OW, T.Float32)
    check(lib().gt_maxpool_fwd_idx(ctx(), dt, dev(relu).ptr, out.ptr, idx.ptr, ctypes.byref(gg)))
    grad = rng.standard_normal(N * C * g.OH * g.OW).astype(npdt)
    dz = new(N * C * H * W, dt)
    check(lib().gt_maxpool_bwd_idx(ctx(), dt, dev(grad).ptr, idx.ptr, out.ptr, 1, dz.ptr, ctypes.byref(gg)))
    # reference: ReLU -> MaxPool2d, backward through both
    zt = ref(z, N, C, H, W).SetRequiresGrad(True)
    y = T.MaxPool2d(zt.ReLU(), k, k)
    assert_bits(host(out), y.Float64s().astype(npdt), "pool fwd")
    y.Backward(ref(grad, N, C, g.OH, g.OW))
    assert_bits(host(dz), zt.Grad().Float64s().astype(npdt), "pool+relu bwd")


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("bc", [(64, 10), (8192, 1000), (3, 4), (256, 10), (1, 1)])
def test_xent_fwd_bwd(dt, npdt, tol, bc):
    B, C = bc
    rng = np.random.default_rng(B + C)
    x = (rng.standard_normal((B, C)) * 3).astype(npdt)
    y = rng.integers(0, C, B).astype(np.int32)
    loss, dl = new(1, dt), new(B * C, dt)
    bad = new(1, T.Float32)
    check(lib().gt_zero(ctx(), bad.ptr, 4))
    labels = cuda_backend().ctx.alloc(4 * B)
    check(lib().gt_upload(ctx(), labels, y.ctypes.data, 4 * B))
    check(lib().gt_xent_fwd_bwd(ctx(), dt, dev(x).ptr, labels, B, C, loss.ptr, dl.ptr, bad.ptr))
    xt = ref(x, B, C).SetRequiresGrad(True)
    lt = xt.LogSoftmax().Pick(list(y)).Mean().Neg()  # CrossEntropyLoss, nn/loss.go:12-14
    lt.Backward()
    assert_close(host(loss), lt.Float64s(), tol, "loss")
    assert_close(host(dl), xt.Grad().Float64s(), tol, "dlogits")
    assert host(bad).view(np.int32)[0] == 0
    cuda_backend().ctx.release(labels)


def _opt_params(npdt, n, rng):
    p = rng.standard_normal(n).astype(npdt)
    gs = [rng.standard_normal(n).astype(npdt) * s for s in (1.0, 1e-3, 10.0)]
    gs[0][:5] = [0.0, -0.0, 1e-30, -1e-30, 1e30]
    return p, gs


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("wd", [0.0, 1e-4])
def test_adam_bit_exact(dt, npdt, tol, wd):
    """Adam.Step (optim/optim.go:110-132) given identical gradients: bit-identical."""
    from oracle import optim_ref as optim
    n = 1001
    rng = np.random.default_rng(11)
    p, gs = _opt_params(npdt, n, rng)
    pt = ref(p, n).SetRequiresGrad(True)
    opt = optim.NewAdam([pt], optim.AdamConfig(LR=1e-3, WeightDecay=wd))
    pd, m, v = dev(p), new(n, dt), new(n, dt)
    cfg = AdamCfg(1e-3, 0, 0, 0, wd)
    for step, g in enumerate(gs, 1):
        pt.grad = ref(g, n)
        opt.Step()
        check(lib().gt_adam_step(ctx(), dt, pd.ptr, dev(g).ptr, m.ptr, v.ptr, n, ctypes.byref(cfg), step))
        assert_bits(host(pd), pt.Float64s().astype(npdt), f"adam step {step}")


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("mom,wd", [(0.9, 1e-4), (0.0, 0.0), (0.9, 0.0), (0.0, 1e-4)])
def test_sgd_bit_exact(dt, npdt, tol, mom, wd):
    """SGD.Step (optim/optim.go:48-70) given identical gradients: bit-identical."""
    from oracle import optim_ref as optim
    n = 1003
    rng = np.random.default_rng(12)
    p, gs = _opt_params(npdt, n, rng)
    pt = ref(p, n).SetRequiresGrad(True)
    opt = optim.NewSGD([pt], optim.SGDConfig(LR=0.01, Momentum=mom, WeightDecay=wd))
    pd, vel = dev(p), new(n, dt)
    cfg = SgdCfg(0.01, mom, wd)
    for step, g in enumerate(gs):
        pt.grad = ref(g, n)
        opt.Step()
        check(lib().gt_sgd_step(ctx(), dt, pd.ptr, dev(g).ptr, vel.ptr, n, ctypes.byref(cfg), int(step == 0)))
        assert_bits(host(pd), pt.Float64s().astype(npdt), f"sgd step {step}")


def test_adam_device_step_counter():
    """gt_adam_step_dev reads and advances the device step: same as host steps."""
    n = 4097
    rng = np.random.default_rng(13)
    p, gs = _opt_params(np.float32, n, rng)
    a, b = dev(p), dev(p)
    ma, va, mb, vb = (new(n, T.Float32) for _ in range(4))
    step = cuda_backend().ctx.alloc(8)
    check(lib().gt_zero(ctx(), step, 8))
    cfg = AdamCfg(1e-3, 0.9, 0.999, 1e-8, 0)
    for s, g in enumerate(gs, 1):
        gd = dev(g)
        check(lib().gt_adam_step(ctx(), T.Float32, a.ptr, gd.ptr, ma.ptr, va.ptr, n, ctypes.byref(cfg), s))
        check(lib().gt_adam_step_dev(ctx(), T.Float32, b.ptr, gd.ptr, mb.ptr, vb.ptr, n, ctypes.byref(cfg), step))
    # bias corrections from the device's pow may differ from the host's in the
    # last float64 bit; after rounding to float32 that is at most one ulp
    assert_close(host(b), host(a), 1e-6, "device-step adam")
    cnt = np.zeros(1, dtype=np.int64)
    check(lib().gt_download(ctx(), cnt.ctypes.data, step, 8))
    assert cnt[0] == 3
    cuda_backend().ctx.release(step)


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("bc", [(8192, 1000), (64, 10), (1000, 33), (300, 1500)])
def test_xent_db_is_the_column_sum_of_dlogits(dt, npdt, tol, bc):
    """gt_xent_fwd_bwd_db: the loss and dlogits of gt_xent_fwd_bwd, bit for
    bit, and db = the column sums of dlogits, the last Linear's bias gradient
    (sumTo over the batch, tensor/ops.go:418-433); rows wider than 1024
    classes take the reduction path."""
    B, C = bc
    rng = np.random.default_rng(B + 3 * C)
    x = (rng.standard_normal((B, C)) * 3).astype(npdt)
    y = rng.integers(0, C, B).astype(np.int32)
    labels = cuda_backend().ctx.alloc(4 * B)
    check(lib().gt_upload(ctx(), labels, y.ctypes.data, 4 * B))
    xd = dev(x)
    loss1, dl1, loss2, dl2, db = new(1, dt), new(B * C, dt), new(1, dt), new(B * C, dt), new(C, dt)
    check(lib().gt_xent_fwd_bwd(ctx(), dt, xd.ptr, labels, B, C, loss1.ptr, dl1.ptr, None))
    check(lib().gt_xent_fwd_bwd_db(ctx(), dt, xd.ptr, labels, B, C, loss2.ptr, dl2.ptr, db.ptr, None))
    assert_bits(host(loss2), host(loss1), "loss")
    dl = host(dl1)
    assert_bits(host(dl2), dl, "dlogits")
    cpu = T.backend_for(T.CPU)
    want = cpu.ToHost(cpu.Reduce(0, cpu.FromHost(dl), 1, B, C))
    assert_close(host(db), want, tol, "db")
    cuda_backend().ctx.release(labels)


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("mkn", [(8192, 4096, 1000), (1024, 4096, 4096), (256, 128, 10), (300, 36, 132)])
@pytest.mark.parametrize("act", [1, 2])
def test_linear_bwd_data_db_is_the_column_sum_of_dx(dt, npdt, tol, mkn, act):
    """gt_linear_bwd_data_db and gt_linear_bwd_data_bits_db: dx of the entry
    points they extend, bit for bit, and db_prev = the column sums of dx (the
    bias gradient of the layer before). The shapes take the tensor-core path
    whole and K-split (the column sums then come from the split reduction)
    and the SIMT path."""
    M, K, N = mkn  # dx (M, K) = dy (M, N) @ w (N, K) * act'(y_prev)
    rng = np.random.default_rng(M + K + N + act)
    y_prev = rng.standard_normal((M, K)).astype(npdt)
    if act == 1:
        y_prev = np.maximum(y_prev, 0)
    else:
        y_prev = np.tanh(y_prev).astype(npdt)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(npdt)
    dy = (rng.standard_normal((M, N)) / M).astype(npdt)
    dyd, wd, yd = dev(dy), dev(w), dev(y_prev)
    dx1, dx2, db = new(M * K, dt), new(M * K, dt), new(K, dt)
    check(lib().gt_linear_bwd_data(ctx(), dt, dyd.ptr, wd.ptr, yd.ptr, act, dx1.ptr, M, K, N))
    check(lib().gt_linear_bwd_data_db(ctx(), dt, dyd.ptr, wd.ptr, yd.ptr, act, dx2.ptr, db.ptr, M, K, N))
    dx = host(dx1)
    assert_bits(host(dx2), dx, "dx")
    cpu = T.backend_for(T.CPU)
    want = cpu.ToHost(cpu.Reduce(0, cpu.FromHost(dx), 1, M, K))
    assert_close(host(db), want, tol, "db_prev")
    if act == 1:  # the same through the ReLU bit mask
        ldw = (M + 31) // 32
        bits = new(K * ldw, T.Float32)
        check(lib().gt_relu_bits(ctx(), dt, yd.ptr, bits.ptr, M, K))
        dx3, db3 = new(M * K, dt), new(K, dt)
        check(lib().gt_linear_bwd_data_bits_db(ctx(), dt, dyd.ptr, wd.ptr, bits.ptr, dx3.ptr, db3.ptr, M, K, N))
        assert_bits(host(dx3), dx, "dx through the bit mask")
        assert_close(host(db3), want, tol, "db_prev through the bit mask")


# (N, C, H, W, O, kernel, stride, pad, pool window): the conv stack's and the
# CNN's first convolutions, a strided one, 3 x 3 windows, and two that take
# the fallback through the full-resolution gradient (C*KH*KW > 32; a pool
# that leaves the last row and column out).
POOL_CONVS = [(4, 3, 32, 32, 64, 3, 1, 1, 2), (4, 1, 28, 28, 32, 3, 1, 1, 2), (2, 2, 11, 11, 8, 3, 2, 1, 2),
              (2, 3, 12, 12, 16, 3, 1, 1, 3), (2, 4, 8, 8, 8, 3, 1, 1, 2), (2, 3, 9, 9, 8, 3, 1, 1, 2)]


def _pool_wgrad_case(dt, npdt, cs, relu, rng, x=None):
    """Forward conv [+ ReLU] -> MaxPool2d on the device, then the fused
    weight gradient and the two-call chain on the same pooled gradient."""
    N, C, H, W, O, k, s, p, kp = cs
    if x is None:
        x = rng.standard_normal((N, C, H, W)).astype(npdt)
    w = (rng.standard_normal((O, C, k, k)) / np.sqrt(C * k * k)).astype(npdt)
    b = (0.1 * rng.standard_normal(O)).astype(npdt)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, s, p)
    pg = T.conv_geom("MaxPool2d", [N, O, g.OH, g.OW], kp, kp, kp, 0)
    gg = ctypes.byref(_lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_]))
    pgg = ctypes.byref(_lib.GtGeom(*[getattr(pg, f) for f, _ in _lib.GtGeom._fields_]))
    y = new(N * O * g.OH * g.OW, dt)
    check(lib().gt_conv_fwd(ctx(), dt, dev(x).ptr, dev(w).ptr, dev(b).ptr, y.ptr, gg, O, 1 if relu else 0))
    npool = N * O * pg.OH * pg.OW
    pooled, idx = new(npool, dt), new(npool, T.Float32)
    check(lib().gt_maxpool_fwd_idx(ctx(), dt, y.ptr, pooled.ptr, idx.ptr, pgg))
    grad = (rng.standard_normal(npool) / npool).astype(npdt)
    xd, gd = dev(x), dev(grad)
    dw, db = new(O * C * k * k, dt), new(O, dt)
    check(lib().gt_conv_bwd_weight_pool(ctx(), dt, xd.ptr, gd.ptr, idx.ptr, pooled.ptr, 1 if relu else 0, dw.ptr,
                                        db.ptr, gg, pgg, O))
    dy, dw2, db2 = new(N * O * g.OH * g.OW, dt), new(O * C * k * k, dt), new(O, dt)
    check(lib().gt_maxpool_bwd_idx(ctx(), dt, gd.ptr, idx.ptr, pooled.ptr, 1 if relu else 0, dy.ptr, pgg))
    check(lib().gt_conv_bwd_weight(ctx(), dt, xd.ptr, dy.ptr, dw2.ptr, db2.ptr, gg, O))
    return x, w, b, grad, host(dw), host(db), host(dw2), host(db2)


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("cs", POOL_CONVS)
@pytest.mark.parametrize("relu", [True, False])
def test_conv_bwd_weight_pool(dt, npdt, tol, cs, relu):
    """The fused pool-backward weight gradient against the oracle's Conv2d
    [-> ReLU] -> MaxPool2d backward (tensor/conv.go:40-70) and against the
    two device calls it replaces."""
    N, C, H, W, O, k, s, p, kp = cs
    rng = np.random.default_rng(sum(cs) + relu)
    x, w, b, grad, dw, db, dw2, db2 = _pool_wgrad_case(dt, npdt, cs, relu, rng)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, s, p)
    ws, bs = ref(w, O, C, k, k).SetRequiresGrad(True), ref(b, O).SetRequiresGrad(True)
    out = T.Conv2d(ref(x, N, C, H, W), ws, bs, s, p)
    if relu:
        out = out.ReLU()
    pooled = T.MaxPool2d(out, kp, kp)
    pooled.Backward(ref(grad, N, O, g.OH // kp, g.OW // kp))
    want_w, want_b = ws.Grad().Float64s(), bs.Grad().Float64s()
    assert_close(dw, want_w, tol, "dw vs oracle")
    assert_close(db, want_b, tol, "db vs oracle")
    assert_close(dw, dw2, tol, "dw vs the two calls")
    assert_close(db, db2, tol, "db vs the two calls")


@pytest.mark.parametrize("dt,npdt,tol", DT)
def test_conv_bwd_weight_pool_non_finite_input(dt, npdt, tol):
    """An infinite input value meets zero entries of the output gradient
    (positions that are not window maxima): 0 * inf = NaN in the dense sum, so
    the fused kernel must leave the same weight-gradient entries non-finite
    as the two calls (whose 3xTF32 GEMM turns every product with an infinity
    into NaN, where the fused kernel keeps g * inf = inf at a window maximum)."""
    cs = (3, 3, 16, 16, 8, 3, 1, 1, 2)
    N, C, H, W = cs[:4]
    rng = np.random.default_rng(5)
    x = rng.standard_normal((N, C, H, W)).astype(npdt)
    x[1, 2, 5, 7] = np.inf
    x[2, 0, 0, 3] = -np.inf
    *_, dw, db, dw2, db2 = _pool_wgrad_case(dt, npdt, cs, True, rng, x=x)
    assert np.isnan(dw2).any() and np.isnan(dw).any()
    np.testing.assert_array_equal(np.isfinite(dw), np.isfinite(dw2))
    fin = np.isfinite(dw2)
    assert_close(dw[fin], dw2[fin], tol, "finite dw entries")
    assert_close(db, db2, tol, "db")


@pytest.mark.parametrize("cs", [(4, 32, 14, 14, 64, 3, 1, 1), (3, 16, 10, 10, 32, 3, 1, 1), (2, 64, 14, 14, 32, 3, 1, 1)])
def test_conv_implicit_whole_image_halo_against_float64(cs):
    """Images whose positions do not split into whole-row 128-position tiles
    (14 x 14, 10 x 10): the implicit forward and input gradient take halo
    boxes of whole image planes (two or three images per tile) with the
    padding masked in the gather, checked against float64 results. The bound
    is that of a float32 dot product: 8x the oracle's own float32 error or
    2^-19 of the sum of absolute products (3xTF32 drops lo * lo and the tensor
    core's accumulation truncates; a wrong or missing tap would be ~1e-3)."""
    N, C, H, W, O, k, s, p = cs
    rng = np.random.default_rng(sum(cs) + 7)
    x = rng.standard_normal((N, C, H, W)).astype(np.float32)
    w = rng.standard_normal((O, C, k, k)).astype(np.float32)
    b = rng.standard_normal(O).astype(np.float32)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, s, p)
    gg = ctypes.byref(_lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_]))
    dy = rng.standard_normal((N, O, g.OH, g.OW)).astype(np.float32)
    y, dx = new(N * O * g.OH * g.OW, T.Float32), new(N * C * H * W, T.Float32)
    check(lib().gt_conv_fwd(ctx(), 0, dev(x).ptr, dev(w).ptr, dev(b).ptr, y.ptr, gg, O, 0))
    assert lib().gt_gemm_path_taken() == 4
    check(lib().gt_conv_bwd_data(ctx(), 0, dev(dy).ptr, dev(w).ptr, dx.ptr, gg, O))
    assert lib().gt_gemm_path_taken() == 4

    def run(dt, absolute=False):
        def t(a, *shape):
            a = np.abs(a) if absolute else a
            return T.FromFloat64(a.astype(np.float64).reshape(-1), *shape).ToDType(dt).SetRequiresGrad(True)
        xs, ws, bs = t(x, N, C, H, W), t(w, O, C, k, k), t(b, O)
        out = T.Conv2d(xs, ws, bs, s, p)
        out.Backward(t(dy, N, O, g.OH, g.OW))
        return [out.Float64s(), xs.Grad().Float64s()]

    T.SetDefaultDType(T.Float64)
    try:
        exact, scale = run(T.Float64), run(T.Float64, absolute=True)
    finally:
        T.SetDefaultDType(T.Float32)
    oracle32 = run(T.Float32)
    for name, got, ex, sc, o32 in zip(("y", "dx"), (host(y), host(dx)), exact, scale, oracle32):
        err = np.abs(got.astype(np.float64) - ex) / np.maximum(sc, 1e-30)
        err32 = np.abs(o32 - ex) / np.maximum(sc, 1e-30)
        assert err.max() <= max(8 * err32.max(), 2.0 ** -19), (name, cs, float(err.max()), float(err32.max()))


# (N, C, H, W, O, kernel, pad, pool window): the conv stack's four layers
# (whole-row and whole-image position tiles, an odd image count that leaves
# half of the last tile empty), a 64-wide image, and geometries that take the
# unfused path (a 128-wide image, 3 x 3 windows); the first conv of each
# benchmark config, a two-channel one without padding and a 5 x 5 window take
# the direct kernel or not by their patch size; the CNN's second conv (14 x 14)
# and a 10 x 10 one pool in the epilogue of tiles whose halo holds whole images.
CONV_POOLS = [(2, 3, 32, 32, 64, 3, 1, 2), (3, 64, 16, 16, 128, 3, 1, 2), (3, 128, 8, 8, 256, 3, 1, 2),
              (5, 256, 4, 4, 512, 3, 1, 2), (1, 8, 64, 64, 32, 3, 1, 2), (1, 4, 128, 128, 16, 3, 1, 2),
              (2, 1, 28, 28, 32, 3, 1, 2), (2, 3, 12, 12, 16, 3, 1, 3), (2, 2, 10, 10, 8, 3, 0, 2),
              (2, 3, 12, 12, 8, 5, 2, 2), (4, 32, 14, 14, 64, 3, 1, 2), (3, 16, 10, 10, 32, 3, 1, 2)]


def _direct(cs):
    """Whether gt_conv_fwd_pool computes this geometry with the direct
    first-conv kernel (3 x 3 windows over at most 3 channels, stride 1, 2 x 2
    pooling of an even-sized output)."""
    N, C, H, W, O, k, p, kp = cs
    oh, ow = H + 2 * p - k + 1, W + 2 * p - k + 1
    return k == 3 and C <= 3 and p <= 2 and kp == 2 and oh % 2 == 0 and ow % 2 == 0


@pytest.mark.parametrize("dt,npdt,tol", DT)
@pytest.mark.parametrize("cs", CONV_POOLS)
@pytest.mark.parametrize("act", [0, 1])
def test_conv_fwd_pool_bit_exact(dt, npdt, tol, cs, act):
    """gt_conv_fwd_pool gives the pooled values and first-max indices of
    gt_conv_fwd followed by gt_maxpool_fwd_idx bit for bit where it pools in
    the implicit GEMM's epilogue (which changes only which lane holds which
    position) or falls back to the two calls; the direct first-conv kernel
    sums the same products in another rounding, so there the values agree
    within tolerance and the indices wherever a window's two largest values
    are not within that tolerance. All against the oracle's Conv2d [-> ReLU]
    -> MaxPool2d within tolerance. float64 always takes the direct kernel or
    the two calls."""
    N, C, H, W, O, k, p, kp = cs
    if dt == T.Float64 and C * H * W * N > 2 * 64 * 16 * 16:
        pytest.skip("float64 through the explicit path: the small geometries suffice")
    rng = np.random.default_rng(sum(cs) + act)
    x = rng.standard_normal((N, C, H, W)).astype(npdt)
    w = (rng.standard_normal((O, C, k, k)) / np.sqrt(C * k * k)).astype(npdt)
    b = (0.1 * rng.standard_normal(O)).astype(npdt)
    g = T.conv_geom("Conv2d", [N, C, H, W], k, k, 1, p)
    pg = T.conv_geom("MaxPool2d", [N, O, g.OH, g.OW], kp, kp, kp, 0)
    gg = ctypes.byref(_lib.GtGeom(*[getattr(g, f) for f, _ in _lib.GtGeom._fields_]))
    pgg = ctypes.byref(_lib.GtGeom(*[getattr(pg, f) for f, _ in _lib.GtGeom._fields_]))
    xd, wd, bd = dev(x), dev(w), dev(b)
    npool = N * O * pg.OH * pg.OW
    pooled, idx = new(npool, dt), new((npool + 3) // 4, T.Float32)
    check(lib().gt_conv_fwd_pool(ctx(), dt, xd.ptr, wd.ptr, bd.ptr, pooled.ptr, idx.ptr, gg, pgg, O, act))
    y = new(N * O * g.OH * g.OW, dt)
    pooled2, idx2 = new(npool, dt), new((npool + 3) // 4, T.Float32)
    check(lib().gt_conv_fwd(ctx(), dt, xd.ptr, wd.ptr, bd.ptr, y.ptr, gg, O, act))
    check(lib().gt_maxpool_fwd_idx(ctx(), dt, y.ptr, pooled2.ptr, idx2.ptr, pgg))
    got, want = host(pooled), host(pooled2)
    gi = host(idx).view(np.uint8)[:npool]
    wi = host(idx2).view(np.uint8)[:npool]
    if _direct(cs):
        assert_close(got, want, tol, "pooled values (direct kernel)")
        if kp == 2:
            win = host(y).reshape(N, O, pg.OH, 2, pg.OW, 2).transpose(0, 1, 2, 4, 3, 5).reshape(-1, 4)
            top = np.sort(win.astype(np.float64), axis=1)
            close = top[:, 3] - top[:, 2] <= tol * np.maximum(1.0, np.abs(top[:, 3]))
            assert np.all((gi == wi) | close), int(((gi != wi) & ~close).sum())
    else:
        assert_bits(got, want, "pooled values")
        np.testing.assert_array_equal(gi, wi)
    out = T.Conv2d(ref(x, N, C, H, W), ref(w, O, C, k, k), ref(b, O), 1, p)
    if act:
        out = out.ReLU()
    assert_close(got, T.MaxPool2d(out, kp, kp).Float64s(), tol, "pooled vs oracle")
