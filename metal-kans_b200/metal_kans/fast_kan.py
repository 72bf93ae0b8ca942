"""FastKAN layer (Gaussian radial basis functions) on the B200 engine.

Drop-in for ``metal_kans/fast_kan.py:13-334``: ``grid = linspace(grid_range, num_centers)``,
``inv_denominator = 1 / (2 h^2)`` (overridable attribute, as the reference forwards whatever is
set), ``w_rbf[D_out, D_in*num_centers]``; ``.half()`` also halves the grid (``fast_kan.py:60-68``)
and the fp16 mode evaluates the RBF in half arithmetic like ``fused_kan.metal:1428-1450``.
New: ``input_map="layernorm"`` (row LayerNorm, no affine, eps ``ln_eps``) and ``.bfloat16()``.
"""
from __future__ import annotations

import math
from typing import Tuple

import numpy as np

from . import device as D
from ._layer import KANLayerBase


class FastKAN(KANLayerBase):
    """Fused FastKAN layer.

    Parameters:
        in_features, out_features: layer widths.
        num_centers: Number of Gaussian centres (default 8).
        grid_range: (min, max) of the uniform centre grid (default (-1, 1)).
        bias, use_base: as the reference.
        input_map: "none" or "layernorm" (new pre-op).
    """

    BASIS = D.KAN_RBF
    MAIN = "w_rbf"
    _WEIGHTS = ("w_rbf", "w_base", "bias", "grid")
    _HALF_EXTRA = ("grid",)

    def __init__(self, in_features: int, out_features: int, num_centers: int = 8,
                 grid_range: Tuple[float, float] = (-1.0, 1.0), bias: bool = True,
                 use_base: bool = True, input_map: str = "none", ln_eps: float = 1e-5):
        self.in_features = in_features
        self.out_features = out_features
        self.num_centers = num_centers
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        self.input_map = input_map
        self.ln_eps = ln_eps
        # fast_kan.py:40-49, same order
        self.grid = np.linspace(grid_range[0], grid_range[1], num_centers, dtype=np.float32)
        h = (grid_range[1] - grid_range[0]) / (num_centers - 1)
        self.inv_denominator = float(1.0 / (2.0 * (h ** 2)))
        bound = 1.0 / math.sqrt(in_features)
        self.w_rbf = np.random.uniform(-bound, bound, (out_features, in_features * num_centers)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    def _train_call(self, lib, x, target, W, Wb, bias, st, hyper):
        w, wb, b, mw, vw, mwb, vwb, mb, vb = self._train_ptrs(W, Wb, bias, st, self.has_base,
                                                              self.has_bias)
        g = np.ascontiguousarray(self.grid, np.float32)
        lib.metal_kan_fastkan_train_step(x.ctypes.data, target.ctypes.data, w, wb, g.ctypes.data,
                                         b, mw, vw, mwb, vwb, mb, vb, x.shape[0],
                                         self.in_features, self.out_features, self.num_centers,
                                         self.inv_denominator, self.has_base, self.has_bias,
                                         *hyper)

    def _backward_call(self, lib, dY, x, dW, dWb, dbias, dX, fused):
        P = lambda a: a.ctypes.data if a is not None else None  # noqa: E731
        grid = np.ascontiguousarray(self.grid, np.float32)
        lib.metal_kan_fastkan_backward(
            P(dY), P(x), P(self.w_rbf), P(self.w_base) if self.has_base else None, P(grid), P(dW),
            P(dWb), P(dbias), P(dX), x.shape[0], self.in_features, self.out_features,
            self.num_centers, self.inv_denominator, self.has_base, self.has_bias)

    def bfloat16(self):
        # the grid stays fp32 in bf16 mode (basis math is fp32 there)
        from ._engine import BFLOAT16

        return self._cast(BFLOAT16, ())

    def _terms(self) -> int:
        return int(self.num_centers)

    def _basis_params(self, L, keep):
        g = self._dev_array("grid_f32", np.asarray(self.grid).astype(np.float32), "grid")
        keep.append(g)
        L.grid = g.ptr
        L.inv_den = float(self.inv_denominator)

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward (fast_kan.py:223-247 semantics)."""
        if self.dtype != np.float32:
            return self._benchmark_fallback(x, warmup, iters)
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        return self._bridge.benchmark_metal_fastkan(
            xf.ctypes.data, self.w_rbf.ctypes.data, self.w_base.ctypes.data,
            self.grid.ctypes.data, self.bias.ctypes.data, y.ctypes.data, xf.shape[0],
            self.in_features, self.out_features, self.num_centers, self.inv_denominator,
            self.has_base, self.has_bias, warmup, iters)
