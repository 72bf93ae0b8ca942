"""MultKAN layer (KAN 2.0 multiplication nodes) on the B200 engine.

Drop-in for the reference's ``metal_kans/mult_kan.py:14-160``: a FastKAN sub-layer to
``num_add + 2 num_mult`` internal outputs (``num_mult`` defaults to ``max(1, out // 2)``), whose
last ``2 num_mult`` outputs are multiplied in pairs, ``u = internal[num_add + m]``,
``v = internal[num_add + num_mult + m]`` (``combine_mult_nodes``, ``fused_kan.metal:368-389``).
The sub-layer runs on the engine's fused kernels, the pair products in one small kernel on the
device (``kan_mult_combine``).  New: ``.bfloat16()``.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _engine as E
from .fast_kan import FastKAN


class MultKAN:
    """Fused MultKAN layer: ``num_add`` additive and ``num_mult`` multiplicative channels."""

    def __init__(self, in_features: int, out_features: int, num_mult: Optional[int] = None,
                 num_grids: int = 8, bias: bool = True, use_base: bool = True):
        self.in_features = in_features
        self.out_features = out_features
        if num_mult is None:
            self.num_mult = max(1, out_features // 2) if out_features > 1 else 0
        else:
            self.num_mult = min(num_mult, out_features)
        self.num_add = out_features - self.num_mult
        self.internal_out = self.num_add + 2 * self.num_mult
        self.sub_layer = FastKAN(in_features, self.internal_out, num_centers=num_grids, bias=bias,
                                 use_base=use_base)
        self.num_grids = num_grids
        self.has_base, self.has_bias = self.sub_layer.has_base, self.sub_layer.has_bias
        self._bridge = self.sub_layer._bridge

    def _sync_attrs(self):
        pass  # the weight attributes read and write the sub-layer's (properties below)

    # the reference mirrors the sub-layer's arrays as attributes of its own (mult_kan.py:57-63);
    # here they are the sub-layer's, so that an assignment reaches the kernels
    def _sub_attr(name):  # noqa: N805
        return property(lambda self: getattr(self.sub_layer, name),
                        lambda self, v: setattr(self.sub_layer, name, v))

    w_rbf = _sub_attr("w_rbf")
    w_base = _sub_attr("w_base")
    grid = _sub_attr("grid")
    bias = _sub_attr("bias")
    inv_denominator = _sub_attr("inv_denominator")
    del _sub_attr

    @property
    def dtype(self) -> np.dtype:
        return self.sub_layer.dtype

    def half(self) -> "MultKAN":
        """Converts layer parameters to FP16 half precision."""
        self.sub_layer.half()
        self._sync_attrs()
        return self

    def float(self) -> "MultKAN":
        """Converts layer parameters to FP32 single precision."""
        self.sub_layer.float()
        self._sync_attrs()
        return self

    def bfloat16(self) -> "MultKAN":
        """Converts layer parameters to bf16 (new)."""
        self.sub_layer.bfloat16()
        self._sync_attrs()
        return self

    def forward_device(self, x_ptr: int, y_ptr: int, B: int, stream=None) -> None:
        """Enqueue on device buffers: x [B, in] -> y [B, out] (layer dtype)."""
        sl = self.sub_layer
        es = np.dtype(self.dtype).itemsize
        if self.num_mult == 0:
            sl.forward_device(x_ptr, y_ptr, B, stream)
            return
        mid = sl._scratch().get("mult_internal", B * self.internal_out * es)
        sl.forward_device(x_ptr, mid.ptr, B, stream)
        E.lib().kan_mult_combine(ctypes.c_void_p(mid.ptr), ctypes.c_void_p(y_ptr), int(B),
                                 self.num_add, self.num_mult, E.kan_dtype(self.dtype), stream)

    def forward(self, x: np.ndarray) -> np.ndarray:
        """Sub-layer forward and the pair products on the GPU (mult_kan.py:89-136 semantics)."""
        act = self.dtype
        x2, orig = E.as_activation(x, act, self.in_features)
        B = x2.shape[0]
        y = E.pinned_empty((B, self.out_features), act)
        if B:
            s = self.sub_layer._scratch()
            dx = s.get("mult_x", x2.nbytes).upload(x2)
            dy = s.get("mult_y", y.nbytes)
            self.forward_device(dx.ptr, dy.ptr, B)
            E.fetch(dy, y)
        return E.restore_shape(y, orig, self.out_features)

    __call__ = forward

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward through ``benchmark_metal_mult`` (fp32 layers;
        mult_kan.py:138-160)."""
        if self.dtype != np.float32:
            import time

            for _ in range(warmup):
                self.forward(x)
            t0 = time.perf_counter()
            for _ in range(iters):
                self.forward(x)
            return (time.perf_counter() - t0) * 1e3 / iters
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        g = np.ascontiguousarray(self.grid, np.float32)
        return self._bridge.benchmark_metal_mult(
            xf.ctypes.data, self.w_rbf.ctypes.data, self.w_base.ctypes.data, g.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.num_add, self.num_mult, self.num_grids, self.inv_denominator,
            self.has_base, self.has_bias, warmup, iters)
