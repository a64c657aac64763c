"""Evaluation on the device: gt_argmax_rows against the oracle's
Tensor.Argmax (tensor/ops.go:176-192), index for index, including the
reference's comparison rule on ties, NaNs, signed zeros and infinities; and
the runtime's gth_predict / gth_count_correct against the oracle's
model.Forward(x).Argmax() and the accuracy count of examples/mnist/main.go."""
import ctypes

import numpy as np
import pytest

from gotensor import _lib
from gotensor import model as gm
from gotensor._lib import FLOAT32, FLOAT64, GTError, check
from gpu_common import cuda_backend
from oracle import gotensor_ref as T
from oracle import nn_ref as nn

pytestmark = pytest.mark.gpu


def device_argmax(x, dt):
    be = cuda_backend()
    rows, n = x.shape
    xs = be.FromHost(np.ascontiguousarray(x).reshape(-1))
    out = be.ctx.alloc(max(rows, 1) * 4)
    try:
        check(_lib.cuda_lib().gt_argmax_rows(be.ctx.ptr, dt, xs.ptr, rows, n, out))
        got = np.empty(rows, dtype=np.int32)
        if rows:
            check(_lib.cuda_lib().gt_download(be.ctx.ptr, got.ctypes.data, out, rows * 4))
        return got
    finally:
        be.Sync()
        be.ctx.release(out)


def oracle_argmax(x, tdt):
    T.SetDefaultDType(tdt)
    try:
        return np.array(T.New(x.astype(np.float64).reshape(-1), *x.shape).Argmax(), dtype=np.int64)
    finally:
        T.SetDefaultDType(T.Float32)


def special_rows(n, npdt, rng):
    """Rows that exercise the comparison rule."""
    rows = []
    r = rng.standard_normal(n).astype(npdt)
    r[[1, n - 1]] = r.max() + 1  # tie between two maxima: the first wins
    rows.append(r)
    r = rng.standard_normal(n).astype(npdt)
    r[0] = np.nan  # NaN at index 0: never replaced
    rows.append(r)
    r = rng.standard_normal(n).astype(npdt)
    r[n // 2] = np.nan  # NaN elsewhere: never chosen
    rows.append(r)
    r = np.full(n, -np.inf, dtype=npdt)  # all -inf: index 0
    rows.append(r)
    r = np.zeros(n, dtype=npdt)
    r[0] = -0.0  # -0 == +0: the first one stays
    rows.append(r)
    r = rng.standard_normal(n).astype(npdt)
    r[n - 1] = np.inf
    rows.append(r)
    r = np.full(n, np.nan, dtype=npdt)  # all NaN: index 0
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("dt,npdt,tdt", [(FLOAT32, np.float32, T.Float32), (FLOAT64, np.float64, T.Float64)])
@pytest.mark.parametrize("shape", [(1, 1), (3, 7), (64, 10), (513, 1000), (5, 4099)])
def test_argmax_matches_oracle(dt, npdt, tdt, shape):
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    x = rng.standard_normal(shape).astype(npdt)
    if shape[1] >= 4:
        x = np.concatenate([x, special_rows(shape[1], npdt, rng)])
    x[0, :] = np.round(x[0, :])  # many ties
    assert np.array_equal(device_argmax(x, dt), oracle_argmax(x, tdt))


def test_argmax_wide_rows_against_vectorised_rule():
    """8192 x 1000 (the wide MLP's logits) against a vectorised statement of
    the same rule: the first maximum, NaNs after index 0 ignored."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((8192, 1000)).astype(np.float32)
    x[::97, 3] = np.nan
    x[::101, 500] = x[::101].max(axis=1) + 1
    x[::101, 700] = x[::101, 500]  # ties at 500 and 700
    want = np.argmax(np.where(np.isnan(x), -np.inf, x), axis=1)
    want[np.isnan(x[:, 0])] = 0
    assert np.array_equal(device_argmax(x, FLOAT32), want)


def test_argmax_and_count_reject_bad_sizes():
    be = cuda_backend()
    lib = _lib.cuda_lib()
    with pytest.raises(GTError):
        check(lib.gt_argmax_rows(be.ctx.ptr, FLOAT32, None, 4, 0, None))
    with pytest.raises(GTError):
        check(lib.gt_count_equal(be.ctx.ptr, None, None, -1, None))


def test_count_equal():
    be = cuda_backend()
    lib = _lib.cuda_lib()
    rng = np.random.default_rng(2)
    for n in (0, 1, 1000, 1 << 20):
        a = rng.integers(0, 10, n).astype(np.int32)
        b = np.where(rng.random(n) < 0.3, a, rng.integers(0, 10, n)).astype(np.int32)
        da, db, cnt = be.ctx.alloc(max(4 * n, 4)), be.ctx.alloc(max(4 * n, 4)), be.ctx.alloc(8)
        try:
            if n:
                check(lib.gt_upload(be.ctx.ptr, da, a.ctypes.data, 4 * n))
                check(lib.gt_upload(be.ctx.ptr, db, b.ctypes.data, 4 * n))
            check(lib.gt_count_equal(be.ctx.ptr, da, db, n, cnt))
            got = ctypes.c_int64()
            check(lib.gt_download(be.ctx.ptr, ctypes.byref(got), cnt, 8))
            assert got.value == int(np.sum(a == b))
        finally:
            be.Sync()
            for p in (da, db, cnt):
                be.ctx.release(p)


def test_model_predict_and_count_match_oracle():
    """A small MLP after a few training steps (so its logits have structure):
    the device's per-row Argmax equals the oracle forward's, and the count of
    correct rows equals the reference loop's. With two batches staged, each
    evaluation reads its own batch and labels."""
    cuda_backend()
    T.SetDefaultDType(T.Float32)
    T.ManualSeed(3)
    ref = nn.NewSequential(nn.NewLinear(64, 48), nn.NewReLU(), nn.NewLinear(48, 10))
    model = gm.Model([gm.Linear(64, 48), gm.ReLU(), gm.Linear(48, 10)], [256, 64])
    model.load_state_dict({k: v.Float64s().reshape(v.Shape()) for k, v in nn.StateDict(ref).items()})
    model.adam(lr=1e-2)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((256, 64)).astype(np.float32)
    y = (x[:, :10].argmax(axis=1)).astype(np.int32)  # a learnable rule
    model.set_batch(x, y)
    for _ in range(30):
        model.train_step()
    sd = model.state_dict()
    nn.LoadStateDict(ref, {k: T.New(v.astype(np.float64).reshape(-1), *v.shape) for k, v in sd.items()}, True)
    for seed in (10, 11):
        xb = np.random.default_rng(seed).standard_normal((256, 64)).astype(np.float32)
        yb = (xb[:, :10].argmax(axis=1)).astype(np.int32)
        want = np.array(ref.Forward(T.New(xb.astype(np.float64).reshape(-1), 256, 64)).Argmax())
        model.set_batch(xb, yb)
        assert np.array_equal(model.predict(), want)
        assert model.count_correct() == int(np.sum(want == yb))
    # two staged batches: each count reads its own batch's labels
    pinned = []
    lib = _lib.cuda_lib()
    try:
        wants = []
        for seed in (20, 21):
            xb = np.random.default_rng(seed).standard_normal((256, 64)).astype(np.float32)
            yb = (xb[:, :10].argmax(axis=1) if seed == 20 else np.zeros(256)).astype(np.int32)
            want = np.array(ref.Forward(T.New(xb.astype(np.float64).reshape(-1), 256, 64)).Argmax())
            wants.append(int(np.sum(want == yb)))
            px, py = ctypes.c_void_p(), ctypes.c_void_p()
            check(lib.gt_host_alloc(xb.nbytes, ctypes.byref(px)))
            check(lib.gt_host_alloc(yb.nbytes, ctypes.byref(py)))
            ctypes.memmove(px, xb.ctypes.data, xb.nbytes)
            ctypes.memmove(py, yb.ctypes.data, yb.nbytes)
            pinned.append((px, py))
            model.stage_batch(px.value, py.value)
        assert [model.count_correct(), model.count_correct()] == wants
    finally:
        model.ctx.sync()
        for px, py in pinned:
            lib.gt_host_free(px)
            lib.gt_host_free(py)
