"""FourierKAN layer on the B200 engine.

Drop-in for the reference's ``metal_kans/fourier_kan.py:13-138``: ``num_frequencies`` F gives
2F + 1 bases per feature, ``1, cos(pi x), sin(pi x), ..., cos(F pi x), sin(F pi x)`` on the raw
input (``fused_kan.metal:306-329``; fp16 angles in half like ``:1550-1576``), weights
``w_fourier[D_out, D_in*(2F+1)]``.  New: ``.bfloat16()``.
"""
from __future__ import annotations

import math

import numpy as np

from . import device as D
from ._layer import KANLayerBase


class FourierKAN(KANLayerBase):
    """Fused FourierKAN layer."""

    BASIS = D.KAN_FOURIER
    MAIN = "w_fourier"
    _WEIGHTS = ("w_fourier", "w_base", "bias")

    def __init__(self, in_features: int, out_features: int, num_frequencies: int = 4,
                 bias: bool = True, use_base: bool = True):
        self.in_features = in_features
        self.out_features = out_features
        self.num_frequencies = num_frequencies
        self.num_bases = 2 * num_frequencies + 1
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        # fourier_kan.py:37-44, same order
        bound = 1.0 / math.sqrt(in_features)
        self.w_fourier = np.random.uniform(-bound, bound, (out_features, in_features * self.num_bases)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    def _terms(self) -> int:
        return int(self.num_bases)

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward (fourier_kan.py:115-138 semantics)."""
        if self.dtype != np.float32:
            return self._benchmark_fallback(x, warmup, iters)
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        return self._bridge.benchmark_metal_fourier(
            xf.ctypes.data, self.w_fourier.ctypes.data, self.w_base.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.num_frequencies, self.has_base, self.has_bias, warmup, iters)
