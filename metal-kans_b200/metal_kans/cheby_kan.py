"""ChebyKAN layer (Chebyshev polynomials) on the B200 engine.

Drop-in for the reference's ``metal_kans/cheby_kan.py:13-341``: same constructor arguments,
weight attributes (``w_cheby[D_out, D_in*degree]`` with column ``i*degree + k``, ``w_base``,
``bias``), ``degree`` counting terms T_0..T_{degree-1}, ``.half()`` / ``.float()``, forward
semantics ``y = bias + silu(x) W_base^T + sum_k T_k(clamp(x,-1,1)) W^T``.  New: ``input_map``
("none" = the reference clamp, "tanh") and ``.bfloat16()``.
"""
from __future__ import annotations

import math

import numpy as np

from . import device as D
from ._layer import KANLayerBase


class ChebyKAN(KANLayerBase):
    """Fused ChebyKAN layer.

    Parameters:
        in_features: Number of input features.
        out_features: Number of output features.
        degree: Number of Chebyshev terms (default 4 -> T_0..T_3), as in the reference.
        bias: Whether to add a bias (default True).
        use_base: Whether to include the residual SiLU base branch (default True).
        input_map: "none" (reference clamp to [-1, 1]) or "tanh" (new pre-op).
    """

    BASIS = D.KAN_CHEBY
    MAIN = "w_cheby"
    _WEIGHTS = ("w_cheby", "w_base", "bias")

    def __init__(self, in_features: int, out_features: int, degree: int = 4, bias: bool = True,
                 use_base: bool = True, input_map: str = "none"):
        self.in_features = in_features
        self.out_features = out_features
        self.degree = degree
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        self.input_map = input_map
        # same initialisation order as cheby_kan.py:38-41 (identical weights for one seed)
        bound = 1.0 / math.sqrt(in_features)
        self.w_cheby = np.random.uniform(-bound, bound, (out_features, in_features * degree)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    def _terms(self) -> int:
        return int(self.degree)

    def _train_call(self, lib, x, target, W, Wb, bias, st, hyper):
        w, wb, b, mw, vw, mwb, vwb, mb, vb = self._train_ptrs(W, Wb, bias, st, self.has_base,
                                                              self.has_bias)
        lib.metal_kan_cheby_train_step(x.ctypes.data, target.ctypes.data, w, wb, b, mw, vw, mwb,
                                       vwb, mb, vb, x.shape[0], self.in_features,
                                       self.out_features, self.degree, self.has_base,
                                       self.has_bias, *hyper)

    def _backward_call(self, lib, dY, x, dW, dWb, dbias, dX, fused):
        fn = lib.metal_kan_cheby_backward_fused if fused else lib.metal_kan_cheby_backward
        P = lambda a: a.ctypes.data if a is not None else None  # noqa: E731
        fn(P(dY), P(x), P(self.w_cheby), P(self.w_base) if self.has_base else None, P(dW), P(dWb),
           P(dbias), P(dX), x.shape[0], self.in_features, self.out_features, self.degree,
           self.has_base, self.has_bias)

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean milliseconds of one host-pointer forward (cheby_kan.py:233-256 semantics:
        x cast to fp32, timed through ``benchmark_metal_cheby``)."""
        if self.dtype != np.float32:
            return self._benchmark_fallback(x, warmup, iters)
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        return self._bridge.benchmark_metal_cheby(
            xf.ctypes.data, self.w_cheby.ctypes.data, self.w_base.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.degree, self.has_base, self.has_bias, warmup, iters)
