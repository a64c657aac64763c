"""ORACLE — test infrastructure, not part of the product.

Restates go-tensor's ``optim`` package (``optim/optim.go``) over
``oracle.gotensor_ref``: every update is the same chain of tensor ops as the
reference, so each intermediate is rounded to the parameter dtype exactly
where the reference rounds it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

from . import gotensor_ref as T


@dataclass
class SGDConfig:
    LR: float = 0.0
    Momentum: float = 0.0
    WeightDecay: float = 0.0


class SGD:
    """optim/optim.go:29-70"""

    def __init__(self, params, cfg: SGDConfig):
        self.cfg, self.params = cfg, list(params)
        self.velocity = [None] * len(self.params)

    def ZeroGrad(self):
        for p in self.params:
            p.ZeroGrad()

    def Step(self):
        c = self.cfg
        with T.no_grad():
            for i, p in enumerate(self.params):
                g = p.Grad()
                if g is None:
                    continue
                d = g
                if c.WeightDecay != 0:
                    d = d.Add(p.MulScalar(c.WeightDecay))
                if c.Momentum != 0:
                    if self.velocity[i] is None:
                        self.velocity[i] = d.Clone()
                    else:
                        self.velocity[i] = self.velocity[i].MulScalar(c.Momentum).Add(d)
                    d = self.velocity[i]
                p.CopyFrom(p.Sub(d.MulScalar(c.LR)))


def NewSGD(params, cfg):
    return SGD(params, cfg)


@dataclass
class AdamConfig:
    LR: float = 0.0
    Beta1: float = 0.0
    Beta2: float = 0.0
    Eps: float = 0.0
    WeightDecay: float = 0.0


class Adam:
    """optim/optim.go:72-132; zero config fields take PyTorch's defaults."""

    def __init__(self, params, cfg: AdamConfig):
        cfg = AdamConfig(cfg.LR or 1e-3, cfg.Beta1 or 0.9, cfg.Beta2 or 0.999, cfg.Eps or 1e-8, cfg.WeightDecay)
        self.cfg, self.params = cfg, list(params)
        self.m = [None] * len(self.params)
        self.v = [None] * len(self.params)
        self.step = 0

    def ZeroGrad(self):
        for p in self.params:
            p.ZeroGrad()

    def Step(self):
        c = self.cfg
        self.step += 1
        bc1 = 1 - math.pow(c.Beta1, float(self.step))
        bc2 = 1 - math.pow(c.Beta2, float(self.step))
        with T.no_grad():
            for i, p in enumerate(self.params):
                g = p.Grad()
                if g is None:
                    continue
                if c.WeightDecay != 0:
                    g = g.Add(p.MulScalar(c.WeightDecay))
                if self.m[i] is None:
                    self.m[i], self.v[i] = T.ZerosLike(p), T.ZerosLike(p)
                self.m[i] = self.m[i].MulScalar(c.Beta1).Add(g.MulScalar(1 - c.Beta1))
                self.v[i] = self.v[i].MulScalar(c.Beta2).Add(g.Mul(g).MulScalar(1 - c.Beta2))
                denom = self.v[i].MulScalar(1 / bc2).Sqrt().AddScalar(c.Eps)
                p.CopyFrom(p.Sub(self.m[i].MulScalar(c.LR / bc1).Div(denom)))


def NewAdam(params, cfg):
    return Adam(params, cfg)
