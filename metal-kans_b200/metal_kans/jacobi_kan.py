"""JacobiKAN layer on the B200 engine.

Drop-in for the reference's ``metal_kans/jacobi_kan.py:13-143``: ``degree`` terms
``P_0 .. P_{degree-1}`` of the Jacobi polynomials ``P^(alpha, beta)`` on ``clamp(x, -1, 1)`` by the
three-term recurrence (``fused_kan.metal:331-366``; fp16 ``:1578-1613``), weights
``w_jacobi[D_out, D_in*degree]``; alpha = beta = 0 gives Legendre polynomials.  New:
``.bfloat16()``.
"""
from __future__ import annotations

import math

import numpy as np

from . import device as D
from ._layer import KANLayerBase


class JacobiKAN(KANLayerBase):
    """Fused JacobiKAN layer."""

    BASIS = D.KAN_JACOBI
    MAIN = "w_jacobi"
    _WEIGHTS = ("w_jacobi", "w_base", "bias")

    def __init__(self, in_features: int, out_features: int, degree: int = 4, alpha: float = 0.0,
                 beta: float = 0.0, bias: bool = True, use_base: bool = True):
        self.in_features = in_features
        self.out_features = out_features
        self.degree = degree
        self.alpha = float(alpha)
        self.beta = float(beta)
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        # jacobi_kan.py:40-47, same order
        bound = 1.0 / math.sqrt(in_features)
        self.w_jacobi = np.random.uniform(-bound, bound, (out_features, in_features * degree)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    def _terms(self) -> int:
        return int(self.degree)

    def _basis_params(self, L, keep):
        L.alpha = float(self.alpha)
        L.beta = float(self.beta)

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward (jacobi_kan.py:120-143 semantics)."""
        if self.dtype != np.float32:
            return self._benchmark_fallback(x, warmup, iters)
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        return self._bridge.benchmark_metal_jacobi(
            xf.ctypes.data, self.w_jacobi.ctypes.data, self.w_base.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.degree, self.alpha, self.beta, self.has_base, self.has_bias,
            warmup, iters)
