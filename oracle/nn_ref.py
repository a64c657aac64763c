"""ORACLE — test infrastructure, not part of the product.

Restates go-tensor's ``nn`` package over ``oracle.gotensor_ref``:
``nn/module.go`` (Linear, Sequential, activations, To/ToDType), ``nn/conv.go``
(Conv2d, MaxPool2d), ``nn/loss.go`` (MSE, CrossEntropy, BCE), ``nn/mode.go``
(Dropout, Train/Eval), ``nn/state.go`` (named parameters, state dicts) and
``nn/serialize.go`` (the positional "GOTN" v1 file format).
"""
from __future__ import annotations

import io
import math
import struct

import numpy as np

from . import gotensor_ref as T


class Module:
    def Forward(self, x):
        raise NotImplementedError

    def Parameters(self):
        return []


def To(m: Module, d) -> None:
    """nn/module.go:17-24"""
    for p in m.Parameters():
        p.MoveTo(d)


def ToDType(m: Module, dt) -> None:
    for p in m.Parameters():
        p.CastTo(dt)


class Linear(Module):
    """nn/module.go:34-55: y = x @ Weightᵀ + Bias, init U(±1/sqrt(in))."""

    def __init__(self, in_features, out_features):
        bound = 1.0 / math.sqrt(float(in_features))
        self.Weight = T.Uniform(-bound, bound, out_features, in_features).SetRequiresGrad(True)
        self.Bias = T.Uniform(-bound, bound, out_features).SetRequiresGrad(True)

    def Forward(self, x):
        return x.MatMul(self.Weight.T()).Add(self.Bias)

    def Parameters(self):
        return [self.Weight, self.Bias]

    def NamedParameters(self):
        return [("weight", self.Weight), ("bias", self.Bias)]


NewLinear = Linear


class Sequential(Module):
    """nn/module.go:57-78"""

    def __init__(self, *layers):
        self.Layers = list(layers)

    def Forward(self, x):
        for l in self.Layers:
            x = l.Forward(x)
        return x

    def Parameters(self):
        ps = []
        for l in self.Layers:
            ps.extend(l.Parameters())
        return ps

    def NamedParameters(self):
        out = []
        for i, l in enumerate(self.Layers):
            for name, p in NamedParameters(l):
                out.append((f"{i}.{name}", p))
        return out

    def SetTraining(self, training):
        for l in self.Layers:
            _set_training(l, training)


def NewSequential(*layers):
    return Sequential(*layers)


class _Activation(Module):
    """nn/module.go:80-99"""

    def __init__(self, name, fn):
        self.name, self.fn = name, fn

    def Forward(self, x):
        return self.fn(x)


def NewReLU():
    return _Activation("ReLU", lambda x: x.ReLU())


def NewSigmoid():
    return _Activation("Sigmoid", lambda x: x.Sigmoid())


def NewTanh():
    return _Activation("Tanh", lambda x: x.Tanh())


def NewSoftmax():
    return _Activation("Softmax", lambda x: x.Softmax())


def NewFlatten():
    return _Activation("Flatten", lambda x: x.Flatten())


class Conv2d(Module):
    """nn/conv.go:9-33, init U(±1/sqrt(in*k*k))."""

    def __init__(self, in_ch, out_ch, kernel, stride, padding):
        bound = 1.0 / math.sqrt(float(in_ch * kernel * kernel))
        self.Weight = T.Uniform(-bound, bound, out_ch, in_ch, kernel, kernel).SetRequiresGrad(True)
        self.Bias = T.Uniform(-bound, bound, out_ch).SetRequiresGrad(True)
        self.Stride, self.Padding = stride, padding

    def Forward(self, x):
        return T.Conv2d(x, self.Weight, self.Bias, self.Stride, self.Padding)

    def Parameters(self):
        return [self.Weight, self.Bias]

    def NamedParameters(self):
        return [("weight", self.Weight), ("bias", self.Bias)]


NewConv2d = Conv2d


class MaxPool2d(Module):
    """nn/conv.go:35-55; stride 0 defaults to the kernel size."""

    def __init__(self, kernel, stride=0):
        self.Kernel, self.Stride = kernel, stride or kernel

    def Forward(self, x):
        return T.MaxPool2d(x, self.Kernel, self.Stride)


NewMaxPool2d = MaxPool2d


class Dropout(Module):
    """nn/mode.go:27-66. p == 0 (or eval mode) returns x untouched; otherwise
    the mask is drawn on the host from the seeded generator."""

    def __init__(self, p):
        if p < 0 or p >= 1:
            raise ValueError("nn: dropout probability must be in [0, 1)")
        self.P, self.eval = p, False

    def SetTraining(self, training):
        self.eval = not training

    def Forward(self, x):
        if self.eval or self.P == 0:
            return x
        m = T.Rand(*x.Shape()).Float64s()
        scale = 1.0 / (1.0 - self.P)
        m = np.where(m < self.P, 0.0, scale)
        mask = T.FromFloat64(m, *x.Shape()).ToDType(x.DType()).To(x.Device())
        return x.Mul(mask)


NewDropout = Dropout


def _set_training(m, training):
    if hasattr(m, "SetTraining"):
        m.SetTraining(training)


def Train(m):
    _set_training(m, True)


def Eval(m):
    _set_training(m, False)


# -- losses (nn/loss.go)

def MSELoss(pred, target):
    return pred.Sub(target).Pow(2).Mean()


def CrossEntropyLoss(logits, targets):
    return logits.LogSoftmax().Pick(targets).Mean().Neg()


def BCELoss(pred, target):
    pos = target.Mul(pred.Log())
    neg = target.Neg().AddScalar(1).Mul(pred.Neg().AddScalar(1).Log())
    return pos.Add(neg).Mean().Neg()


# -- state dicts (nn/state.go)

def NamedParameters(m):
    if hasattr(m, "NamedParameters"):
        return m.NamedParameters()
    return [(str(i), p) for i, p in enumerate(m.Parameters())]


def StateDict(m):
    return dict(NamedParameters(m))


class StateDictError(ValueError):
    def __init__(self, missing, unexpected):
        parts = []
        if missing:
            parts.append("missing keys: " + ", ".join(missing))
        if unexpected:
            parts.append("unexpected keys: " + ", ".join(unexpected))
        super().__init__("nn: state dict does not match model: " + "; ".join(parts))
        self.Missing, self.Unexpected = missing, unexpected


def LoadStateDict(m, sd, strict):
    """nn/state.go:84-126: all-or-nothing."""
    params = NamedParameters(m)
    missing, load, known = [], [], set()
    for name, p in params:
        known.add(name)
        if name not in sd:
            missing.append(name)
            continue
        if sd[name].Shape() != p.Shape():
            raise ValueError(f"nn: {name} has shape {sd[name].Shape()} in the state dict but {p.Shape()} in the model")
        load.append((name, sd[name]))
    if strict:
        unexpected = sorted(k for k in sd if k not in known)
        if missing or unexpected:
            raise StateDictError(missing, unexpected)
    by_name = dict(params)
    for name, src in load:
        by_name[name].CopyFrom(src)


# -- GOTN v1 file format (nn/serialize.go:11-89)

_MAGIC, _VERSION = b"GOTN", 1


def Save(w: io.BufferedIOBase, m: Module) -> None:
    params = m.Parameters()
    w.write(_MAGIC)
    w.write(struct.pack("<II", _VERSION, len(params)))
    for p in params:
        shape = p.Shape()
        w.write(struct.pack("<I", len(shape)))
        w.write(struct.pack(f"<{len(shape)}I", *shape))
        w.write(np.asarray(p.Float64s(), dtype="<f8").tobytes())


def Load(r: io.BufferedIOBase, m: Module) -> None:
    magic = r.read(4)
    if magic != _MAGIC:
        raise ValueError("nn: not a go-tensor model file")
    version, count = struct.unpack("<II", r.read(8))
    if version != _VERSION:
        raise ValueError(f"nn: unsupported model file version {version}")
    params = m.Parameters()
    if count != len(params):
        raise ValueError(f"nn: file has {count} parameters, module has {len(params)}")
    for i, p in enumerate(params):
        (rank,) = struct.unpack("<I", r.read(4))
        dims = list(struct.unpack(f"<{rank}I", r.read(4 * rank)))
        if dims != p.Shape():
            raise ValueError(f"nn: parameter {i} has shape {dims} in file, {p.Shape()} in module")
        vals = np.frombuffer(r.read(8 * p.Numel()), dtype="<f8")
        p.CopyFrom(T.FromFloat64(vals))
