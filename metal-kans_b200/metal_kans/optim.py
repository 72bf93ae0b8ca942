"""Optimisers over the layers' ``(param, grad)`` pairs, stepping on the GPU.

Drop-in for the reference's ``metal_kans/optim.py`` classes ``Optimizer``, ``SGD``, ``Adam``,
``AdamW`` and ``Lion`` (``optim.py:70-120, 152-316, 479-535``): same constructors and state
(``velocities`` / ``m`` / ``v`` / ``t``), each step one call of the engine's
``metal_kan_{sgd,adam,adamw,lion}_step`` per parameter (the reference's update formulas, fp32).
The reference updates the parameter arrays in place through its bridge; here too, and the owning
layer is told (``param_updated``) so that its device copy is refreshed before the next forward.
Muon and RMSprop of the reference are not part of this engine.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import _engine as E


def _f32(a: np.ndarray) -> np.ndarray:
    if a.dtype != np.float32 or not a.flags["C_CONTIGUOUS"]:
        raise TypeError("the GPU optimisers update C-contiguous fp32 arrays in place")
    return a


class Optimizer:
    """Base class: ``params`` is a sequence of ``(param, grad)`` pairs (layer.parameters())."""

    def __init__(self, params: Sequence[Tuple[np.ndarray, np.ndarray]], lr: float = 1e-3):
        self.params = list(params)
        self.lr = float(lr)

    def zero_grad(self) -> None:
        for _, grad in self.params:
            if grad is not None:
                grad.fill(0)

    def step(self) -> None:
        raise NotImplementedError


class SGD(Optimizer):
    """SGD with momentum, Nesterov acceleration and (coupled) weight decay."""

    def __init__(self, params, lr: float = 1e-2, momentum: float = 0.0, weight_decay: float = 0.0,
                 nesterov: bool = False):
        super().__init__(params, lr)
        self.momentum = float(momentum)
        self.weight_decay = float(weight_decay)
        self.nesterov = bool(nesterov)
        self.velocities: List[Optional[np.ndarray]] = [
            np.zeros_like(p) if momentum > 0.0 else None for p, _ in self.params]

    def step(self) -> None:
        lib = E.lib()
        for i, (param, grad) in enumerate(self.params):
            if grad is None:
                continue
            v = self.velocities[i]
            if v is None:
                v = self.velocities[i] = np.zeros_like(param)
            lib.metal_kan_sgd_step(_f32(param).ctypes.data, _f32(grad).ctypes.data,
                                   _f32(v).ctypes.data, self.lr, self.momentum, self.weight_decay,
                                   int(self.nesterov), param.size)
            E.param_updated(param)


class _AdamBase(Optimizer):
    _ENTRY = ""

    def __init__(self, params, lr: float = 1e-3, betas: Tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0):
        super().__init__(params, lr)
        self.beta1, self.beta2 = float(betas[0]), float(betas[1])
        self.eps = float(eps)
        self.weight_decay = float(weight_decay)
        self.t = 0
        self.m = [np.zeros_like(p) for p, _ in self.params]
        self.v = [np.zeros_like(p) for p, _ in self.params]

    def step(self) -> None:
        self.t += 1
        lr_t = self.lr * math.sqrt(1.0 - self.beta2 ** self.t) / (1.0 - self.beta1 ** self.t)
        fn = getattr(E.lib(), self._ENTRY)
        for i, (param, grad) in enumerate(self.params):
            if grad is None:
                continue
            fn(_f32(param).ctypes.data, _f32(grad).ctypes.data, _f32(self.m[i]).ctypes.data,
               _f32(self.v[i]).ctypes.data, self.lr, self.beta1, self.beta2, self.eps,
               self.weight_decay, lr_t, param.size)
            E.param_updated(param)


class Adam(_AdamBase):
    """Adam with L2 weight decay added to the gradient (coupled)."""

    _ENTRY = "metal_kan_adam_step"


class AdamW(_AdamBase):
    """AdamW: decoupled weight decay (Loshchilov & Hutter)."""

    _ENTRY = "metal_kan_adamw_step"

    def __init__(self, params, lr: float = 1e-3, betas: Tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01):
        super().__init__(params, lr, betas, eps, weight_decay)


class Lion(Optimizer):
    """Lion: sign of the interpolated momentum (Chen et al. 2023)."""

    def __init__(self, params, lr: float = 1e-4, betas: Tuple[float, float] = (0.9, 0.99),
                 weight_decay: float = 0.0):
        super().__init__(params, lr)
        self.beta1, self.beta2 = float(betas[0]), float(betas[1])
        self.weight_decay = float(weight_decay)
        self.m = [np.zeros_like(p) for p, _ in self.params]

    def step(self) -> None:
        lib = E.lib()
        for i, (param, grad) in enumerate(self.params):
            if grad is None:
                continue
            lib.metal_kan_lion_step(_f32(param).ctypes.data, _f32(grad).ctypes.data,
                                    _f32(self.m[i]).ctypes.data, self.lr, self.beta1, self.beta2,
                                    self.weight_decay, param.size)
            E.param_updated(param)
