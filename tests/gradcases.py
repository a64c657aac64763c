"""The reference's list of differentiable operations with sample shapes
(tensor/tensor_test.go:15-50) and its sample-input rule (54-73), shared by the
oracle's finite-difference check and the device-parity tests."""
import numpy as np

from oracle import gotensor_ref as T


def grad_cases():
    return [
        ("Add/broadcast", lambda x: x[0].Add(x[1]), [[3, 4], [4]], False),
        ("Sub/broadcast", lambda x: x[0].Sub(x[1]), [[3, 1], [1, 4]], False),
        ("Mul/broadcast", lambda x: x[0].Mul(x[1]), [[2, 3, 4], [3, 1]], False),
        ("Div", lambda x: x[0].Div(x[1]), [[3, 4], [3, 4]], True),
        ("Pow", lambda x: x[0].Pow(3), [[5]], False),
        ("Exp", lambda x: x[0].Exp(), [[5]], False),
        ("Log", lambda x: x[0].Log(), [[5]], True),
        ("Sqrt", lambda x: x[0].Sqrt(), [[5]], True),
        ("Abs", lambda x: x[0].Abs(), [[6]], False),
        ("Sigmoid", lambda x: x[0].Sigmoid(), [[5]], False),
        ("Tanh", lambda x: x[0].Tanh(), [[5]], False),
        ("ReLU", lambda x: x[0].ReLU(), [[6]], False),
        ("MulScalar/AddScalar", lambda x: x[0].MulScalar(3).AddScalar(1), [[4]], False),
        ("MatMul", lambda x: x[0].MatMul(x[1]), [[3, 4], [4, 2]], False),
        ("T", lambda x: x[0].T().Mul(x[1]), [[2, 3, 4], [4, 3]], False),
        ("Permute", lambda x: x[0].Permute(2, 0, 1).Mul(x[1]), [[2, 3, 4], [4, 2, 3]], False),
        ("Reshape", lambda x: x[0].Reshape(-1, 2).Mul(x[1]), [[2, 3], [2]], False),
        ("Sum", lambda x: x[0].Sum().Mul(x[0]), [[2, 3]], False),
        ("SumDim", lambda x: x[0].SumDim(1, False).Pow(2), [[2, 3, 4]], False),
        ("MeanDim/keep", lambda x: x[0].MeanDim(-1, True).Mul(x[0]), [[3, 4]], False),
        ("Mean", lambda x: x[0].Mul(x[0]).Mean(), [[3, 4]], False),
        ("LogSoftmax", lambda x: x[0].LogSoftmax().Mul(x[1]), [[3, 4], [3, 4]], False),
        ("Pick", lambda x: x[0].Pick([2, 0, 1]).Pow(2), [[3, 4]], False),
        ("Index", lambda x: x[0].Index(1).Pow(2), [[3, 2, 2]], False),
        ("Stack", lambda x: T.Stack([x[0], x[1].Exp()]).Mul(x[0]), [[3], [3]], False),
        ("Conv2d", lambda x: T.Conv2d(x[0], x[1], x[2], 1, 0).Pow(2), [[2, 3, 5, 5], [4, 3, 3, 3], [4]], False),
        ("Conv2d/stride+pad", lambda x: T.Conv2d(x[0], x[1], None, 2, 1).Pow(2), [[2, 2, 5, 4], [3, 2, 3, 2]], False),
        ("MaxPool2d", lambda x: T.MaxPool2d(x[0], 2, 2).Pow(2), [[2, 3, 4, 6]], False),
        ("MaxPool2d/overlap", lambda x: T.MaxPool2d(x[0], 3, 1).Pow(2), [[1, 2, 5, 5]], False),
        ("reuse", lambda x: x[0].Mul(x[0]).Add(x[0].Exp()), [[4]], False),
    ]


def sample_inputs(shapes, pos, rng: np.random.Generator):
    """tensor/tensor_test.go:54-73: values away from 0 (or in [0.5, 2) when
    the op needs positive inputs)."""
    vals = []
    for shape in shapes:
        n = int(np.prod(shape))
        if pos:
            v = 0.5 + 1.5 * rng.random(n)
        else:
            v = rng.standard_normal(n)
            v = np.where(np.abs(v) < 0.05, v + 0.1, v)
        vals.append(v)
    return vals


def close_enough(a, b, tol=1e-4):
    """tensor/device_mps_test.go:19-21: |a-b| <= tol*max(1,|b|), NaN == NaN."""
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    ok = np.abs(a - b) <= tol * np.maximum(1.0, np.abs(b))
    return ok | (np.isnan(a) & np.isnan(b))
