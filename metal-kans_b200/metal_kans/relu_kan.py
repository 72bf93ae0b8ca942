"""ReLUKAN layer (piecewise-linear tent basis) on the B200 engine.

Drop-in for the reference's ``metal_kans/relu_kan.py:13-228``: ``grid = linspace(grid_range,
num_grids)``, ``inv_h = 1 / h``, ``w_relu[D_out, D_in*num_grids]``; basis
``max(0, 1 - |x - g_k| inv_h)`` on the raw input (``fused_kan.metal:278-303``; the fp16 mode in
half arithmetic like ``:1452-1474``, and ``.half()`` halves the grid as the reference does).
fp32 layers train: ``backward`` mirrors ``relu_kan.py:132-202``.  New: ``.bfloat16()``.
"""
from __future__ import annotations

import math
from typing import Tuple

import numpy as np

from . import device as D
from ._layer import KANLayerBase


class ReLUKAN(KANLayerBase):
    """Fused ReLUKAN layer (tent basis)."""

    BASIS = D.KAN_RELU
    MAIN = "w_relu"
    _WEIGHTS = ("w_relu", "w_base", "bias", "grid")
    _HALF_EXTRA = ("grid",)

    def __init__(self, in_features: int, out_features: int, num_grids: int = 8,
                 grid_range: Tuple[float, float] = (-1.0, 1.0), bias: bool = True,
                 use_base: bool = True):
        self.in_features = in_features
        self.out_features = out_features
        self.num_grids = num_grids
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        # relu_kan.py:40-51, same order
        self.grid = np.linspace(grid_range[0], grid_range[1], num_grids, dtype=np.float32)
        h = (grid_range[1] - grid_range[0]) / (num_grids - 1)
        self.inv_h = float(1.0 / h)
        bound = 1.0 / math.sqrt(in_features)
        self.w_relu = np.random.uniform(-bound, bound, (out_features, in_features * num_grids)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    def bfloat16(self):
        # the grid stays fp32 in bf16 mode (the basis math is fp32 there)
        from ._engine import BFLOAT16

        return self._cast(BFLOAT16, ())

    def _terms(self) -> int:
        return int(self.num_grids)

    def _basis_params(self, L, keep):
        g = self._dev_array("grid_f32", np.asarray(self.grid).astype(np.float32), "grid")
        keep.append(g)
        L.grid = g.ptr
        L.inv_h = float(self.inv_h)

    def _backward_call(self, lib, dY, x, dW, dWb, dbias, dX, fused):
        P = lambda a: a.ctypes.data if a is not None else None  # noqa: E731
        grid = np.ascontiguousarray(self.grid, np.float32)
        lib.metal_kan_relu_backward(
            P(dY), P(x), P(self.w_relu), P(self.w_base) if self.has_base else None, P(grid),
            P(dW), P(dWb), P(dbias), P(dX), x.shape[0], self.in_features, self.out_features,
            self.num_grids, self.inv_h, self.has_base, self.has_bias)

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward (relu_kan.py:204-228 semantics)."""
        if self.dtype != np.float32:
            return self._benchmark_fallback(x, warmup, iters)
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        g = np.ascontiguousarray(self.grid, np.float32)
        return self._bridge.benchmark_metal_relu(
            xf.ctypes.data, self.w_relu.ctypes.data, self.w_base.ctypes.data, g.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.num_grids, self.inv_h, self.has_base, self.has_bias, warmup,
            iters)
