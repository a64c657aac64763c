"""Every backend.Backend primitive on the B200 against the oracle (the CPU
restatement of internal/cpu) on identical seeded inputs: bit-exact wherever
the arithmetic is order-independent (element-wise, copies, Max, im2col,
col2im, pooling), within the reference's device tolerance
|a-b| <= tol*max(1,|b|) for sums and products (tol 1e-4 float32, 1e-10
float64)."""
import numpy as np
import pytest

from gpu_common import assert_bits, assert_close, cpu_backend, cuda_backend
from oracle import gotensor_ref as T

pytestmark = pytest.mark.gpu

DTYPES = [(T.Float32, np.float32, 1e-4), (T.Float64, np.float64, 1e-10)]


def both(data):
    return cpu_backend().FromHost(data), cuda_backend().FromHost(data)


def host(s):
    return cuda_backend().ToHost(s) if not hasattr(s, "data") else s.data


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
@pytest.mark.parametrize("op", range(13))
def test_unary(dt, npdt, tol, op):
    rng = np.random.default_rng(op)
    x = rng.standard_normal(1027).astype(npdt) * 3
    if op in (T.LOG, T.SQRT):
        x = np.abs(x) + 0.01
    x[:6] = [0.0, -0.0, np.nan, np.inf, -np.inf, 1e-30] if op not in (T.LOG, T.SQRT) else x[:6]
    c, g = both(x)
    want = cpu_backend().Unary(op, 2.5 if op != T.POW else 3.0, c).data
    got = cuda_backend().ToHost(cuda_backend().Unary(op, 2.5 if op != T.POW else 3.0, g))
    if op in (T.EXP, T.LOG, T.SIGMOID, T.TANH, T.POW):
        # evaluated in float64 on both sides; the float64 math libraries may
        # differ in the last bit, which rounding to float32 almost always hides
        assert_close(got, want, 1e-6 if dt == T.Float32 else 1e-15, f"unary {op}")
    else:
        assert_bits(got, want, f"unary {op}")


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
@pytest.mark.parametrize("op", range(4))
@pytest.mark.parametrize("shapes", [([3, 4], [4]), ([3, 1], [1, 4]), ([2, 3, 4], [3, 1]), ([257, 129], [257, 129]),
                                    ([2, 1, 3, 1, 2, 1, 2, 3], [1, 2, 1, 4, 1, 2, 1, 3])])
def test_binary_broadcast(dt, npdt, tol, op, shapes):
    rng = np.random.default_rng(op)
    sa, sb = shapes
    a = rng.standard_normal(int(np.prod(sa))).astype(npdt)
    b = rng.standard_normal(int(np.prod(sb))).astype(npdt) + (3 if op == T.DIV else 0)
    shape = T._broadcast_shapes(sa, sb)
    av = T.make_view(shape, T._broadcast_strides(sa, shape))
    bv = T.make_view(shape, T._broadcast_strides(sb, shape))
    ca, ga = both(a)
    cb, gb = both(b)
    want = cpu_backend().Binary(op, ca, av, cb, bv).data
    got = cuda_backend().ToHost(cuda_backend().Binary(op, ga, av, gb, bv))
    assert_bits(got, want, f"binary {op} {shapes}")


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
def test_copy_views(dt, npdt, tol):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(2 * 3 * 4 * 5).astype(npdt)
    c, g = both(x)
    views = [
        T.make_view([4, 5], [1, 4], 0),                 # 2-D transpose
        T.make_view([5, 2, 3, 4], [1, 60, 20, 5], 0),   # permute (3, 0, 1, 2)
        T.make_view([3, 4], [4, 1], 7),                 # offset slice
        T.make_view([6, 4], [0, 1], 3),                 # broadcast rows
        T.make_view([1], [1], 119),                     # At()
        T.make_view([0, 3], [3, 1], 0),                 # empty
    ]
    for v in views:
        want = cpu_backend().Copy(c, v).data
        got = cuda_backend().ToHost(cuda_backend().Copy(g, v))
        assert_bits(got, want, "copy")


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
@pytest.mark.parametrize("dims", [(1, 1027, 1), (257, 129, 1), (1, 257, 129), (3, 4, 5), (2, 1, 7),
                                  (1, 3_000_000, 1), (1, 8192, 1000), (4, 0, 3), (5, 2, 1)])
def test_reduce(dt, npdt, tol, dims):
    outer, n, inner = dims
    rng = np.random.default_rng(n)
    x = rng.standard_normal(outer * n * inner).astype(npdt)
    c, g = both(x)
    for op in (T.SUM, T.MAX):
        if op == T.MAX and n == 0:
            continue
        want = cpu_backend().Reduce(op, c, outer, n, inner).data
        got = cuda_backend().ToHost(cuda_backend().Reduce(op, g, outer, n, inner))
        if op == T.MAX:
            assert_bits(got, want, f"max {dims}")
        else:
            # tree order on the GPU, sequential on the CPU; the reference's sum
            # carries ~n*eps error, so compare at the scale of sum |x|
            scale = cpu_backend().Reduce(T.SUM, T.CPUStorage(np.abs(x)), outer, n, inner).data
            assert_close(got / np.maximum(1, scale), want / np.maximum(1, scale), tol, f"sum {dims}")


def test_reduce_max_nan_and_signed_zero():
    x = np.array([-0.0, np.nan, 0.0, 1.0, 0.0, -0.0], dtype=np.float32)
    c, g = both(x)
    want = cpu_backend().Reduce(T.MAX, c, 1, 3, 2).data
    got = cuda_backend().ToHost(cuda_backend().Reduce(T.MAX, g, 1, 3, 2))
    assert_bits(got, want, "max nan/zero")


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
@pytest.mark.parametrize("mkn", [(2, 3, 2), (70, 50, 40), (257, 129, 65), (64, 784, 128), (33, 17, 9), (1, 1, 1),
                                 (300, 1000, 10), (512, 256, 384), (10, 4096, 200), (16, 70, 129)])
def test_matmul_trans(dt, npdt, tol, mkn):
    """Activations N(0,1) against weight-scaled operands U(+-1/sqrt(k)) (the
    scales a training step multiplies) at the device tolerance; unscaled
    N(0,1) x N(0,1) operands (sums ~sqrt(k) with heavy cancellation) at the
    reference's large-op tolerance 1e-3 (tensor/device_mps_test.go:68-93)."""
    m, k, n = mkn
    rng = np.random.default_rng(m * k + n)
    for weight_like, t in ((True, tol), (False, 1e-3 if dt == T.Float32 else tol)):
        for ta in (False, True):
            for tb in (False, True):
                a = rng.standard_normal(m * k).astype(npdt)
                b = rng.standard_normal(k * n)
                b = (b / np.sqrt(k) if weight_like else b).astype(npdt)
                ca, ga = both(a)
                cb, gb = both(b)
                want = cpu_backend().MatMul(ca, cb, m, k, n, ta, tb).data
                got = cuda_backend().ToHost(cuda_backend().MatMul(ga, gb, m, k, n, ta, tb))
                assert_close(got, want, t, f"matmul {mkn} ta={ta} tb={tb} weight_like={weight_like}")


@pytest.mark.parametrize("mkn", [(130, 33, 129), (1100, 64, 1500), (384, 1000, 256), (512, 2048, 512)])
def test_matmul_f64_main_kernel(mkn):
    """The float64 kernel for outputs of at least 128 x 128: ragged tiles in
    both directions, K not a multiple of its 16-deep slices, and K-splits
    (3 ways for 384 x 256 over K = 1000, 8 ways for 512 x 512 over K = 2048),
    in all four transpose layouts, against the oracle at the float64 device
    tolerance, and the same bits on a second run."""
    m, k, n = mkn
    rng = np.random.default_rng(m + 7 * k + n)
    be = cuda_backend()
    for ta in (False, True):
        for tb in (False, True):
            a = rng.standard_normal(m * k)
            b = rng.standard_normal(k * n) / np.sqrt(k)
            ca, ga = both(a)
            cb, gb = both(b)
            want = cpu_backend().MatMul(ca, cb, m, k, n, ta, tb).data
            got = be.ToHost(be.MatMul(ga, gb, m, k, n, ta, tb))
            assert_close(got, want, 1e-10, f"f64 matmul {mkn} ta={ta} tb={tb}")
            assert np.array_equal(be.ToHost(be.MatMul(ga, gb, m, k, n, ta, tb)), got)


def test_matmul_known_values():
    """tensor/tensor_test.go:208-218 on the device: exact."""
    _, ga = both(np.array([1, 2, 3, 4, 5, 6], dtype=np.float32))
    _, gb = both(np.array([7, 8, 9, 10, 11, 12], dtype=np.float32))
    got = cuda_backend().ToHost(cuda_backend().MatMul(ga, gb, 2, 3, 2, False, False))
    assert list(got) == [58, 64, 139, 154]


GEOMS = [  # (N, C, H, W, KH, KW, stride, pad)
    (2, 3, 5, 5, 3, 3, 1, 0), (2, 2, 5, 4, 3, 2, 2, 1), (1, 1, 3, 3, 2, 2, 1, 0), (4, 3, 32, 32, 3, 3, 1, 1),
    (3, 5, 7, 9, 4, 2, 3, 2), (1, 2, 4, 4, 1, 1, 1, 0),
    # stride 1 through the tiled col2im: several channel groups, ragged
    # column tiles (W > 32) with an odd channel count, a 5 x 5 kernel
    (8, 64, 16, 16, 3, 3, 1, 1), (2, 37, 9, 40, 3, 3, 1, 1), (2, 5, 33, 7, 5, 5, 1, 2),
]


def geom(N, C, H, W, KH, KW, stride, pad):
    return T.conv_geom("test", [N, C, H, W], KH, KW, stride, pad)


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
@pytest.mark.parametrize("gs", GEOMS)
def test_im2col_col2im(dt, npdt, tol, gs):
    g = geom(*gs)
    rng = np.random.default_rng(sum(gs))
    x = rng.standard_normal(g.N * g.C * g.H * g.W).astype(npdt)
    c, gx = both(x)
    assert_bits(cuda_backend().ToHost(cuda_backend().Im2col(gx, g)), cpu_backend().Im2col(c, g).data, "im2col")
    cols = rng.standard_normal(g.N * g.OH * g.OW * g.C * g.KH * g.KW).astype(npdt)
    cc, gc = both(cols)
    assert_bits(cuda_backend().ToHost(cuda_backend().Col2im(gc, g)), cpu_backend().Col2im(cc, g).data, "col2im")


POOLS = [(2, 3, 4, 6, 2, 2), (1, 2, 5, 5, 3, 1), (1, 1, 3, 3, 2, 1), (8, 16, 28, 28, 2, 2), (2, 3, 7, 7, 2, 2),
         (1, 1, 9, 9, 3, 2)]


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
@pytest.mark.parametrize("ps", POOLS)
def test_maxpool_fwd_bwd_bit_exact(dt, npdt, tol, ps):
    N, C, H, W, k, s = ps
    g = T.conv_geom("MaxPool2d", [N, C, H, W], k, k, s, 0)
    rng = np.random.default_rng(H * W + k)
    # integers in a small range make ties common: the first-max rule must hold
    x = rng.integers(-3, 4, N * C * H * W).astype(npdt)
    c, gx = both(x)
    assert_bits(cuda_backend().ToHost(cuda_backend().MaxPool2d(gx, g)), cpu_backend().MaxPool2d(c, g).data, "pool")
    grad = rng.standard_normal(N * C * g.OH * g.OW).astype(npdt)
    cg, gg = both(grad)
    assert_bits(cuda_backend().ToHost(cuda_backend().MaxPool2dBackward(gx, gg, g)),
                cpu_backend().MaxPool2dBackward(c, cg, g).data, "pool backward")


@pytest.mark.parametrize("dt,npdt,tol", DTYPES)
def test_memory_primitives(dt, npdt, tol):
    be = cuda_backend()
    z = be.Zeros(dt, 10)
    assert (be.ToHost(z) == 0).all() and be.ToHost(z).dtype == npdt
    src = be.FromHost(np.arange(4, dtype=npdt))
    be.Write(z, 3, src)
    assert list(be.ToHost(z)) == [0, 0, 0, 0, 1, 2, 3, 0, 0, 0]
    other = T.Float64 if dt == T.Float32 else T.Float32
    x = np.array([0.1, -2.5, 1e-40, 3.4e38], dtype=npdt)
    want = cpu_backend().Cast(cpu_backend().FromHost(x), other).data
    got = be.ToHost(be.Cast(be.FromHost(x), other))
    assert_bits(got, want, "cast")
    assert be.ToHost(be.Zeros(dt, 0)).size == 0
    with pytest.raises(IndexError):
        be.Write(z, 8, src)
    with pytest.raises(TypeError):
        be.Unary(T.NEG, 0, cpu_backend().FromHost(x))


@pytest.mark.parametrize("dt,npdt,bound", [(T.Float32, np.float32, 2.0 ** -20), (T.Float64, np.float64, 1e-14)])
def test_simt_split_k_long_k(dt, npdt, bound):
    """A convolution's first-layer weight gradient: 64 x 27 outputs over K =
    200,000 (the SIMT path, as 27-wide rows are not 16-byte aligned). It runs
    as many K-splits summed in order: error at the dtype's level against the
    float64 product, and the same bits on every run."""
    be = cuda_backend()
    rng = np.random.default_rng(12)
    m, k, n = 64, 200_000, 27
    a = rng.standard_normal(k * m).astype(npdt)  # stored (k, m): dY of the layer
    b = rng.standard_normal(k * n).astype(npdt)  # stored (k, n): the im2col rows
    ga, gb = be.FromHost(a), be.FromHost(b)
    got = be.ToHost(be.MatMul(ga, gb, m, k, n, True, False))
    A = a.reshape(k, m).T.astype(np.float64)
    B = b.reshape(k, n).astype(np.float64)
    exact = A @ B
    scale = np.abs(A) @ np.abs(B)
    assert (np.abs(got.reshape(m, n) - exact) / scale).max() <= bound
    assert np.array_equal(be.ToHost(be.MatMul(ga, gb, m, k, n, True, False)), got)
