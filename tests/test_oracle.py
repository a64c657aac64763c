"""Pins the oracle (the CPU restatement of go-tensor) to the reference's own
known answers, gradient checks, training tests and PyTorch golden vectors.
CPU only."""
import io
import json
import math
import os

import numpy as np
import pytest

from gradcases import grad_cases, sample_inputs
from oracle import gotensor_ref as T
from oracle import nn_ref as nn
from oracle import optim_ref as optim

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(autouse=True)
def _defaults():
    T.SetDefaultDType(T.Float32)
    yield
    T.SetDefaultDType(T.Float32)


def test_matmul_values():
    """tensor/tensor_test.go:208-218"""
    a = T.New([1, 2, 3, 4, 5, 6], 2, 3)
    b = T.New([7, 8, 9, 10, 11, 12], 3, 2)
    assert list(a.MatMul(b).Float64s()) == [58, 64, 139, 154]


def test_large_matmul_against_naive_loop():
    """tensor/tensor_test.go:220-237: the parallel row-split path."""
    rng = np.random.default_rng(7)
    av, bv = sample_inputs([[70, 50], [50, 40]], False, rng)
    a, b = T.FromFloat64(av, 70, 50), T.FromFloat64(bv, 50, 40)
    got = a.MatMul(b).Float64s().reshape(70, 40)
    want = av.reshape(70, 50) @ bv.reshape(50, 40)
    assert np.max(np.abs(got - want)) <= 1e-9


def test_matmul_transposes_materialized():
    """internal/cpu/linalg.go:15-28: trans flags read the stored transpose."""
    rng = np.random.default_rng(3)
    be = T.CPUBackend()
    for ta in (False, True):
        for tb in (False, True):
            m, k, n = 33, 17, 9
            a = rng.standard_normal((k, m) if ta else (m, k))
            b = rng.standard_normal((n, k) if tb else (k, n))
            c = be.MatMul(be.FromHost(a.reshape(-1)), be.FromHost(b.reshape(-1)), m, k, n, ta, tb)
            want = (a.T if ta else a) @ (b.T if tb else b)
            assert np.allclose(c.data.reshape(m, n), want, atol=1e-12)


def test_conv2d_and_pool_values():
    """tensor/tensor_test.go:271-292"""
    x = T.New([1, 2, 3, 4, 5, 6, 7, 8, 9], 1, 1, 3, 3)
    w = T.Ones(1, 1, 2, 2)
    got = T.Conv2d(x, w, T.New([10]), 1, 0)
    assert got.Shape() == [1, 1, 2, 2]
    assert list(got.Float64s()) == [22, 26, 34, 38]
    assert list(T.MaxPool2d(x, 2, 1).Float64s()) == [5, 6, 8, 9]


@pytest.mark.parametrize("case", grad_cases(), ids=lambda c: c[0])
def test_gradients_finite_difference(case):
    """tensor/tensor_test.go:75-128: autograd vs central differences in float64."""
    name, f, shapes, pos = case
    vals = sample_inputs(shapes, pos, np.random.default_rng(1))

    def build():
        return [T.FromFloat64(v, *s) for v, s in zip(vals, shapes)]
    xs = build()
    for x in xs:
        x.SetRequiresGrad(True)
    f(xs).Sum().Backward()
    eps = 1e-6

    def evaluate():
        with T.no_grad():
            return f(build()).Sum().Item()
    for n, x in enumerate(xs):
        grad = x.Grad().Float64s() if x.Grad() is not None else None
        for i in range(len(vals[n])):
            orig = vals[n][i]
            vals[n][i] = orig + eps
            fp = evaluate()
            vals[n][i] = orig - eps
            fm = evaluate()
            vals[n][i] = orig
            want = (fp - fm) / (2 * eps)
            got = 0.0 if grad is None else grad[i]
            assert abs(want - got) <= 1e-5 * max(1.0, abs(want)), f"{name}: input {n} element {i}: {got} vs {want}"


def test_grad_accumulates():
    """tensor/tensor_test.go:239-246"""
    x = T.New([2]).SetRequiresGrad(True)
    x.Mul(x).Sum().Backward()
    x.Mul(x).Sum().Backward()
    assert x.Grad().Item() == 8


def test_relu_and_max_follow_go_semantics():
    """Go's builtin max (used by ReLU and Reduce Max, internal/cpu/cpu.go:129-131,
    285-287) propagates NaN and maps -0 to +0."""
    be = T.CPUBackend()
    x = be.FromHost(np.array([np.nan, -0.0, -1.0, 2.0], dtype=np.float32))
    y = be.Unary(T.RELU, 0.0, x).data
    assert np.isnan(y[0]) and y[1] == 0 and not np.signbit(y[1]) and y[2] == 0 and y[3] == 2
    r = be.Reduce(T.MAX, be.FromHost(np.array([1.0, np.nan, 3.0, 0.5, 2.0, 1.0], dtype=np.float32)), 1, 3, 2).data
    assert r[0] == 3.0 and np.isnan(r[1])


def test_maxpool_first_max_tie_rule():
    """internal/cpu/linalg.go:177: the first maximum in a window wins."""
    be = T.CPUBackend()
    x = np.zeros(16, dtype=np.float32)
    g = T.conv_geom("MaxPool2d", [1, 1, 4, 4], 2, 2, 2, 0)
    dx = be.MaxPool2dBackward(be.FromHost(x), be.FromHost(np.ones(4, dtype=np.float32)), g).data.reshape(4, 4)
    assert dx[0, 0] == 1 and dx[0, 2] == 1 and dx[2, 0] == 1 and dx[2, 2] == 1 and dx.sum() == 4


def test_train_xor():
    """nn/nn_test.go:12-35"""
    T.ManualSeed(0)
    x = T.New([0, 0, 0, 1, 1, 0, 1, 1], 4, 2)
    y = [0, 1, 1, 0]
    model = nn.NewSequential(nn.NewLinear(2, 8), nn.NewTanh(), nn.NewLinear(8, 2))
    opt = optim.NewAdam(model.Parameters(), optim.AdamConfig(LR=0.05))
    loss = None
    for _ in range(500):
        loss = nn.CrossEntropyLoss(model.Forward(x), y)
        opt.ZeroGrad()
        loss.Backward()
        opt.Step()
    assert loss.Item() < 0.01
    assert model.Forward(x).Argmax() == y


def test_linear_regression_sgd():
    """nn/nn_test.go:37-55"""
    T.ManualSeed(0)
    x = T.Randn(64, 1)
    y = x.MulScalar(3).AddScalar(-2)
    lin = nn.NewLinear(1, 1)
    opt = optim.NewSGD(lin.Parameters(), optim.SGDConfig(LR=0.1, Momentum=0.9))
    for _ in range(200):
        loss = nn.MSELoss(lin.Forward(x), y)
        opt.ZeroGrad()
        loss.Backward()
        opt.Step()
    assert abs(lin.Weight.Item() - 3) <= 1e-3 and abs(lin.Bias.Item() + 2) <= 1e-3


def test_save_load_round_trip():
    """nn/nn_test.go:64-88"""
    T.ManualSeed(0)
    src = nn.NewSequential(nn.NewLinear(3, 4), nn.NewReLU(), nn.NewLinear(4, 2))
    buf = io.BytesIO()
    nn.Save(buf, src)
    dst = nn.NewSequential(nn.NewLinear(3, 4), nn.NewReLU(), nn.NewLinear(4, 2))
    nn.Load(io.BytesIO(buf.getvalue()), dst)
    x = T.Randn(5, 3)
    assert np.array_equal(src.Forward(x).Float64s(), dst.Forward(x).Float64s())
    wrong = nn.NewSequential(nn.NewLinear(3, 5), nn.NewReLU(), nn.NewLinear(5, 2))
    with pytest.raises(ValueError):
        nn.Load(io.BytesIO(buf.getvalue()), wrong)


def test_dropout_modes():
    """nn/nn_test.go:90-117"""
    T.ManualSeed(0)
    d = nn.NewDropout(0.5)
    model = nn.NewSequential(d)
    x = T.Ones(1000)
    out = model.Forward(x).Float64s()
    zeros = int((out == 0).sum())
    assert set(np.unique(out)) <= {0.0, 2.0}
    assert 400 <= zeros <= 600
    nn.Eval(model)
    assert model.Forward(x) is x
    nn.Train(model)
    assert model.Forward(x) is not x
    assert nn.NewSequential(nn.NewDropout(0.0)).Forward(x) is x


def test_pytorch_cnn_golden_forward():
    """weights/weights_test.go:31-74 with the reference's PyTorch fixture."""
    with open(os.path.join(GOLDEN, "cnn_forward.json")) as f:
        fx = json.load(f)
    model = nn.NewSequential(nn.NewConv2d(1, 2, 3, 1, 1), nn.NewReLU(), nn.NewMaxPool2d(2, 0),
                             nn.NewFlatten(), nn.NewLinear(2 * 4 * 4, 3))
    sd = {k: T.FromFloat32(v["values"], *v["shape"]) for k, v in fx["params"].items()}
    nn.LoadStateDict(model, sd, True)
    x = T.New(fx["input"]["values"], *fx["input"]["shape"])
    with T.no_grad():
        y = model.Forward(x).Float64s()
    assert np.max(np.abs(y - np.array(fx["output"]["values"]))) <= fx["tolerance"]


def test_state_dict_strict_errors():
    """nn/state.go:84-126"""
    m = nn.NewSequential(nn.NewLinear(2, 3))
    with pytest.raises(nn.StateDictError):
        nn.LoadStateDict(m, {"0.weight": T.Zeros(3, 2)}, True)
    with pytest.raises(ValueError):
        nn.LoadStateDict(m, {"0.weight": T.Zeros(2, 3), "0.bias": T.Zeros(3)}, True)


def test_training_step_matches_torch_fp64():
    """Secondary cross-check: one Adam step of an MLP in float64 agrees with
    torch on identical arrays (the Linear/CE/Adam formulas are PyTorch's)."""
    torch = pytest.importorskip("torch")
    T.SetDefaultDType(T.Float64)
    T.ManualSeed(5)
    model = nn.NewSequential(nn.NewLinear(6, 5), nn.NewTanh(), nn.NewLinear(5, 4), nn.NewSigmoid(), nn.NewLinear(4, 3))
    x = T.Uniform(-1, 1, 8, 6)
    y = [0, 1, 2, 0, 1, 2, 2, 1]
    tw = [torch.tensor(p.Float64s().reshape(p.Shape()), requires_grad=True) for p in model.Parameters()]
    opt = optim.NewAdam(model.Parameters(), optim.AdamConfig(LR=1e-3))
    topt = torch.optim.Adam(tw, lr=1e-3)
    for _ in range(3):
        loss = nn.CrossEntropyLoss(model.Forward(x), y)
        opt.ZeroGrad(); loss.Backward(); opt.Step()
        tx = torch.tensor(x.Float64s().reshape(8, 6))
        h = torch.tanh(tx @ tw[0].T + tw[1])
        h = torch.sigmoid(h @ tw[2].T + tw[3])
        tl = torch.nn.functional.cross_entropy(h @ tw[4].T + tw[5], torch.tensor(y))
        topt.zero_grad(); tl.backward(); topt.step()
        assert math.isclose(loss.Item(), tl.item(), rel_tol=1e-12)
    for p, q in zip(model.Parameters(), tw):
        assert np.allclose(p.Float64s(), q.detach().numpy().reshape(-1), rtol=1e-10, atol=1e-12)
