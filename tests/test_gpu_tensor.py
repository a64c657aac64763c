"""tensor/device_mps_test.go for the CUDA device: the same tensor-level ops
(the oracle's restatement of go-tensor's tensor package) run on the CPU
backend and on the B200 backend, outputs and every input gradient compared
with the reference's closeEnough rule."""
import numpy as np
import pytest

from gpu_common import assert_close, cuda_backend
from gradcases import close_enough, grad_cases, sample_inputs
from oracle import gotensor_ref as T
from oracle import nn_ref as nn

pytestmark = pytest.mark.gpu

CUDA0 = T.CUDA(0)


@pytest.fixture(autouse=True)
def _registered():
    cuda_backend()
    T.SetDefaultDType(T.Float32)
    yield


@pytest.mark.parametrize("case", grad_cases(), ids=lambda c: c[0])
def test_cuda_matches_cpu(case):
    """TestMPSMatchesCPU (tensor/device_mps_test.go:35-66), float32."""
    name, f, shapes, pos = case
    vals = sample_inputs(shapes, pos, np.random.default_rng(2))

    def run(dev):
        xs = [T.FromFloat64(v, *s).ToDType(T.Float32).To(dev).SetRequiresGrad(True) for v, s in zip(vals, shapes)]
        y = f(xs)
        assert y.Device() == dev, f"{name}: output on {y.Device()}"
        y.Sum().Backward()
        grads = []
        for x in xs:
            assert x.Grad().Device() == dev
            grads.append(x.Grad().Float64s())
        return y.Float64s(), grads

    cpu_out, cpu_grads = run(T.CPU)
    gpu_out, gpu_grads = run(CUDA0)
    assert close_enough(gpu_out, cpu_out).all(), f"{name}: output"
    for n, (g, c) in enumerate(zip(gpu_grads, cpu_grads)):
        assert close_enough(g, c).all(), f"{name}: grad of input {n}"


@pytest.mark.parametrize("case", grad_cases(), ids=lambda c: c[0])
def test_cuda_matches_cpu_float64(case):
    """The same in float64 (which MPS lacks), at the float64 tolerance 1e-10."""
    name, f, shapes, pos = case
    vals = sample_inputs(shapes, pos, np.random.default_rng(3))

    def run(dev):
        xs = [T.FromFloat64(v, *s).To(dev).SetRequiresGrad(True) for v, s in zip(vals, shapes)]
        y = f(xs)
        y.Sum().Backward()
        return y.Float64s(), [x.Grad().Float64s() for x in xs]

    cpu_out, cpu_grads = run(T.CPU)
    gpu_out, gpu_grads = run(CUDA0)
    assert_close(gpu_out, cpu_out, 1e-10, f"{name} output")
    for g, c in zip(gpu_grads, cpu_grads):
        assert_close(g, c, 1e-10, f"{name} grad")


def test_cuda_large_ops():
    """TestMPSLargeOps (tensor/device_mps_test.go:68-93)."""
    T.ManualSeed(3)
    a, b = T.Randn(257, 129), T.Randn(129, 65)
    cases = {
        "matmul": lambda a, b: a.MatMul(b),
        "matmul^T": lambda a, b: b.T().MatMul(a.T()),
        "sum": lambda a, _: a.Reshape(-1).Sum(),
        "sumdim0": lambda a, _: a.SumDim(0, False),
        "maxdim": lambda a, _: a.MaxDim(1, False),
        "softmax": lambda a, _: a.Softmax(),
        "broadcast": lambda a, b: a.Add(b.SumDim(1, True).T()),
    }
    for name, f in cases.items():
        cpu = f(a, b).Float64s()
        gpu = f(a.To(CUDA0), b.To(CUDA0)).Float64s()
        assert close_enough(gpu, cpu, 1e-3).all(), name


def test_cuda_device_semantics():
    """TestMPSDeviceSemantics (tensor/device_mps_test.go:95-119)."""
    x = T.New([1, 2, 3]).To(CUDA0)
    assert x.Device() == CUDA0 and x.DType() == T.Float32
    back = x.MulScalar(2).To(T.CPU)
    assert back.Device() == T.CPU and back.Float64s()[2] == 6
    p = T.Zeros(3).To(CUDA0)
    p.CopyFrom(T.FromFloat64([4, 5, 6]))
    q = T.Zeros(2, 2)
    q.MoveTo(CUDA0)
    assert p.Float64s()[1] == 5 and q.Device() == CUDA0
    # float64 works on CUDA (unlike MPS)
    d = T.FromFloat64([1.5]).To(CUDA0)
    assert d.DType() == T.Float64 and d.Item() == 1.5
    with pytest.raises(ValueError):
        x.Add(T.New([1, 2, 3]))  # mixed devices


def test_conv_values_on_cuda():
    """TestConv2dValues (tensor/tensor_test.go:271-292) on the device."""
    x = T.New([1, 2, 3, 4, 5, 6, 7, 8, 9], 1, 1, 3, 3).To(CUDA0)
    w = T.Ones(1, 1, 2, 2).To(CUDA0)
    got = T.Conv2d(x, w, T.New([10]).To(CUDA0), 1, 0)
    assert list(got.Float64s()) == [22, 26, 34, 38]
    assert list(T.MaxPool2d(x, 2, 1).Float64s()) == [5, 6, 8, 9]


LOSS_CASES = {
    # nn/loss.go:6-22 and the Softmax module (nn/module.go): prediction, target
    "MSELoss": lambda p, t: nn.MSELoss(p, t),
    "BCELoss": lambda p, t: nn.BCELoss(p.Sigmoid(), t),
    "SoftmaxMSE": lambda p, t: nn.MSELoss(nn.NewSoftmax().Forward(p), t),
}


@pytest.mark.parametrize("name", list(LOSS_CASES))
@pytest.mark.parametrize("dt,tol", [(T.Float32, 1e-4), (T.Float64, 1e-10)])
def test_losses_on_cuda_match_cpu(name, dt, tol):
    """The losses and module the fused step does not cover run through the
    tape on the CUDA device: loss value and prediction gradient as on the CPU."""
    rng = np.random.default_rng(8)
    B, C = 64, 10
    pred = rng.standard_normal(B * C)
    target = rng.random(B * C)  # in [0, 1): valid for BCE and MSE

    def run(dev):
        p = T.FromFloat64(pred, B, C).ToDType(dt).To(dev).SetRequiresGrad(True)
        t = T.FromFloat64(target, B, C).ToDType(dt).To(dev)
        loss = LOSS_CASES[name](p, t)
        loss.Backward()
        return loss.Item(), p.Grad().Float64s()

    cpu_loss, cpu_grad = run(T.CPU)
    gpu_loss, gpu_grad = run(CUDA0)
    assert_close(gpu_loss, cpu_loss, tol, f"{name} loss")
    assert_close(gpu_grad, cpu_grad, tol, f"{name} grad")
