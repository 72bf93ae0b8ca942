"""BSplineKAN / KAN layer (uniform cubic B-splines) on the B200 engine.

Drop-in for ``metal_kans/bspline_kan.py:13-342``: ``num_bases = grid_size + 3``,
``grid = [grid_min, inv_h]`` (float32, never halved), ``w_spline[D_out, D_in*(grid_size+3)]``;
closed-form cubic weights at ``span = clamp(floor((x-min)*inv_h), 0, G-1)``,
``u = clamp(frac, 0, 1)`` (``fused_kan.metal:240-276``) -- outside [min, max] the edge polynomial
is evaluated at u in {0, 1}, as in the reference.  ``spline_order`` is stored and ignored, like
the reference.
"""
from __future__ import annotations

import math
from typing import Sequence

import numpy as np

from . import device as D
from ._layer import KANLayerBase


class BSplineKAN(KANLayerBase):
    """Fused B-spline KAN layer (cubic, closed form)."""

    BASIS = D.KAN_BSPLINE
    MAIN = "w_spline"
    _WEIGHTS = ("w_spline", "w_base", "bias")

    def __init__(self, in_features: int, out_features: int, grid_size: int = 5,
                 spline_order: int = 3, grid_range: Sequence[float] = (-1.0, 1.0),
                 bias: bool = True, use_base: bool = True, input_map: str = "none"):
        self.in_features = in_features
        self.out_features = out_features
        self.grid_size = grid_size
        self.spline_order = spline_order
        self.num_bases = grid_size + 3
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        self.input_map = input_map
        # bspline_kan.py:44-55, same order
        self.grid_min = float(grid_range[0])
        self.grid_max = float(grid_range[1])
        self.inv_h = float(grid_size) / (self.grid_max - self.grid_min)
        self.grid_params = np.array([self.grid_min, self.inv_h], dtype=np.float32)
        self.grid = self.grid_params
        bound = 1.0 / math.sqrt(in_features)
        self.w_spline = np.random.uniform(-bound, bound, (out_features, in_features * self.num_bases)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    def _terms(self) -> int:
        return int(self.grid_size) + 3

    def _train_call(self, lib, x, target, W, Wb, bias, st, hyper):
        w, wb, b, mw, vw, mwb, vwb, mb, vb = self._train_ptrs(W, Wb, bias, st, self.has_base,
                                                              self.has_bias)
        lib.metal_kan_bspline_train_step(x.ctypes.data, target.ctypes.data, w, wb, b, mw, vw, mwb,
                                         vwb, mb, vb, x.shape[0], self.in_features,
                                         self.out_features, self.grid_size, self.grid_min,
                                         self.grid_max, self.has_base, self.has_bias, *hyper)

    def _backward_call(self, lib, dY, x, dW, dWb, dbias, dX, fused):
        P = lambda a: a.ctypes.data if a is not None else None  # noqa: E731
        g = np.asarray(self.grid, np.float32)
        lib.metal_kan_bspline_backward(
            P(dY), P(x), P(self.w_spline), P(self.w_base) if self.has_base else None, P(dW),
            P(dWb), P(dbias), P(dX), x.shape[0], self.in_features, self.out_features,
            self.grid_size, float(g[0]), float(g[1]), self.has_base, self.has_bias)

    def _basis_params(self, L, keep):
        g = np.asarray(self.grid, dtype=np.float32)
        L.grid_size = int(self.grid_size)
        L.grid_min = float(g[0])
        L.inv_h = float(g[1])

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward (bspline_kan.py benchmark semantics)."""
        if self.dtype != np.float32:
            return self._benchmark_fallback(x, warmup, iters)
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        g = np.ascontiguousarray(self.grid, np.float32)
        return self._bridge.benchmark_metal_bspline(
            xf.ctypes.data, self.w_spline.ctypes.data, self.w_base.ctypes.data, g.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.grid_size, self.spline_order, self.has_base, self.has_bias,
            warmup, iters)


KAN = BSplineKAN
