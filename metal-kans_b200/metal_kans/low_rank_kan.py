"""LowRankKAN layer (rank-factorised bottleneck) on the B200 engine.

Drop-in for the reference's ``metal_kans/low_rank_kan.py:14-170``: a FastKAN down layer to
``rank = min(rank, out, in * num_grids)`` bottleneck outputs (no base, no bias), then
``Y = bias + Z W_up^T + silu(x) W_base^T`` (``metal_kan_bridge.mm:1535-1698``).  The down layer
runs on the engine's fused kernels (Z in the layer dtype, like the reference's MPS output), the
up projection and base branch in one CUDA-core kernel (``kan_lowrank_up``).  New: ``.bfloat16()``.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _engine as E
from .fast_kan import FastKAN


class LowRankKAN(E.DeviceLayerMixin):
    """Fused LowRankKAN layer: W_spline = W_up @ W_down of rank r."""

    _WEIGHTS = ("w_up", "w_base", "bias")

    def __init__(self, in_features: int, out_features: int, rank: int = 8, num_grids: int = 8,
                 bias: bool = True, use_base: bool = True):
        self.in_features = in_features
        self.out_features = out_features
        self.rank = min(rank, out_features, in_features * num_grids)
        self.num_grids = num_grids
        self.has_bias = 1 if bias else 0
        self.has_base = 1 if use_base else 0
        self.use_base = use_base
        # low_rank_kan.py:47-66, same order
        self.down_layer = FastKAN(in_features, self.rank, num_centers=num_grids, bias=False,
                                  use_base=False)
        bound = 1.0 / math.sqrt(self.rank)
        self.w_up = np.random.uniform(-bound, bound, (out_features, self.rank)).astype(np.float32)
        bound_base = 1.0 / math.sqrt(in_features)
        self.w_base = (np.random.uniform(-bound_base, bound_base, (out_features, in_features))
                       .astype(np.float32) if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = self.down_layer._bridge

    # the down layer's arrays, readable and assignable here (low_rank_kan.py:56-58)
    def _down_attr(name):  # noqa: N805
        return property(lambda self: getattr(self.down_layer, name),
                        lambda self, v: setattr(self.down_layer, name, v))

    w_down = _down_attr("w_rbf")
    grid = _down_attr("grid")
    inv_denominator = _down_attr("inv_denominator")
    del _down_attr

    @property
    def dtype(self) -> np.dtype:
        return self.w_up.dtype

    def _cast(self, dt):
        self.w_up = self.w_up.astype(dt)
        if self.has_base:
            self.w_base = self.w_base.astype(dt)
        if self.has_bias:
            self.bias = self.bias.astype(dt)
        return self

    def half(self) -> "LowRankKAN":
        """Converts layer parameters to FP16 half precision."""
        self.down_layer.half()
        return self._cast(np.float16)

    def float(self) -> "LowRankKAN":
        """Converts layer parameters to FP32 single precision."""
        self.down_layer.float()
        return self._cast(np.float32)

    def bfloat16(self) -> "LowRankKAN":
        """Converts layer parameters to bf16 (new)."""
        self.down_layer.bfloat16()
        return self._cast(E.BFLOAT16)

    def forward_device(self, x_ptr: int, y_ptr: int, B: int, stream=None) -> None:
        """Enqueue on device buffers: x [B, in] -> y [B, out] (layer dtype)."""
        es = np.dtype(self.dtype).itemsize
        z = self._scratch().get("z", max(1, B) * self.rank * es)
        self.down_layer.forward_device(x_ptr, z.ptr, B, stream)
        wu = self._dev("w_up")
        wb = self._dev("w_base") if self.has_base else None
        bb = self._dev("bias") if self.has_bias else None
        E.lib().kan_lowrank_up(ctypes.c_void_p(z.ptr), ctypes.c_void_p(x_ptr),
                               ctypes.c_void_p(wu.ptr), ctypes.c_void_p(wb.ptr if wb else 0),
                               ctypes.c_void_p(bb.ptr if bb else 0), ctypes.c_void_p(y_ptr),
                               int(B), self.in_features, self.out_features, self.rank,
                               self.has_base, self.has_bias, E.kan_dtype(self.dtype), stream)
        self._keep = (z, wu, wb, bb)

    def forward(self, x: np.ndarray) -> np.ndarray:
        """Down projection then up projection + base branch on the GPU."""
        act = self.dtype
        x2, orig = E.as_activation(x, act, self.in_features)
        B = x2.shape[0]
        y = E.pinned_empty((B, self.out_features), act)
        if B:
            s = self._scratch()
            dx = s.get("x", x2.nbytes).upload(x2)
            dy = s.get("y", y.nbytes)
            self.forward_device(dx.ptr, dy.ptr, B)
            E.fetch(dy, y)
        return E.restore_shape(y, orig, self.out_features)

    __call__ = forward

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward through ``benchmark_metal_lowrank`` (fp32)."""
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
        return self._bridge.benchmark_metal_lowrank(
            xf.ctypes.data, np.ascontiguousarray(self.w_down).ctypes.data,
            self.w_up.ctypes.data, self.w_base.ctypes.data, g.ctypes.data,
            self.bias.ctypes.data, y.ctypes.data, xf.shape[0], self.in_features,
            self.out_features, self.rank, self.num_grids, self.inv_denominator, self.has_base,
            self.has_bias, warmup, iters)
