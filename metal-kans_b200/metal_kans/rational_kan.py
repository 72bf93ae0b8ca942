"""RationalKAN layer (Pade-Chebyshev rational functions) on the B200 engine.

Drop-in for the reference's ``metal_kans/rational_kan.py:13-120``: per input-output pair
``phi(x) = P(xc) / (1 + |Q(xc)|)`` with Chebyshev expansions ``P = sum_d W_p T_d``,
``Q = sum_d W_q T_d`` of ``xc = clamp(x, -1, 1)``, plus ``silu(xc) W_base`` and the bias
(``kan_rational_tiled``, ``fused_kan.metal:996-1125``).  fp32 only, like the reference; the layer
runs in one CUDA-core kernel (``kan_rational_forward``): the division per (row, output, input)
triple is not a contraction the tensor cores could take.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _engine as E
from . import device as D


class RationalKAN(E.DeviceLayerMixin):
    """Fused RationalKAN layer (fp32)."""

    _WEIGHTS = ("w_p", "w_q", "w_base", "bias")

    def __init__(self, in_features: int, out_features: int, p_degree: int = 4,
                 q_degree: int = 2, bias: bool = True, use_base: bool = True):
        self.in_features = in_features
        self.out_features = out_features
        self.p_degree = p_degree
        self.q_degree = q_degree
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        # rational_kan.py:45-49, same order
        bound = 1.0 / math.sqrt(in_features)
        self.w_p = np.random.uniform(-bound, bound, (out_features, in_features * p_degree)).astype(np.float32)
        self.w_q = np.random.uniform(-bound * 0.1, bound * 0.1, (out_features, in_features * q_degree)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    @property
    def dtype(self) -> np.dtype:
        return self.w_p.dtype

    def forward_device(self, x_ptr: int, y_ptr: int, B: int, stream=None) -> None:
        """Enqueue on device buffers: x [B, in] -> y [B, out] (fp32)."""
        wp, wq = self._dev("w_p", np.float32), self._dev("w_q", np.float32)
        wb = self._dev("w_base", np.float32) if self.has_base else None
        bb = self._dev("bias", np.float32) if self.has_bias else None
        E.lib().kan_rational_forward(
            ctypes.c_void_p(x_ptr), ctypes.c_void_p(wp.ptr), ctypes.c_void_p(wq.ptr),
            ctypes.c_void_p(wb.ptr if wb else 0), ctypes.c_void_p(bb.ptr if bb else 0),
            ctypes.c_void_p(y_ptr), int(B), self.in_features, self.out_features, self.p_degree,
            self.q_degree, self.has_base, self.has_bias, stream)
        self._keep = (wp, wq, wb, bb)

    def forward(self, x: np.ndarray) -> np.ndarray:
        """Fused rational forward (rational_kan.py:57-91 semantics): fp32 in, fp32 out."""
        x2, orig = E.as_activation(x, np.float32, self.in_features)
        B = x2.shape[0]
        y = E.pinned_empty((B, self.out_features), np.float32)
        if B:
            s = self._scratch()
            dx = s.get("x", x2.nbytes).upload(x2)
            dy = s.get("y", y.nbytes)
            self.forward_device(dx.ptr, dy.ptr, B)
            E.fetch(dy, y)
        return E.restore_shape(y, orig, self.out_features)

    __call__ = forward

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward through ``benchmark_metal_rational``."""
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        return self._bridge.benchmark_metal_rational(
            xf.ctypes.data, self.w_p.ctypes.data, self.w_q.ctypes.data, self.w_base.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.p_degree, self.q_degree, self.has_base, self.has_bias, warmup,
            iters)
