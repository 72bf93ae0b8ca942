"""PyTorch interop: ``nn.Module`` wrappers running the CUDA engine on torch tensors.

Replaces the reference's ``metal_kans/torch_module.py:19-137``, whose autograd function copies
every input to host NumPy and back (``:27-31``).  Here tensors stay on the GPU: the module hands
``data_ptr()`` of its CUDA parameters and of the input to ``kan_forward`` on torch's current
stream.  Inputs on the CPU are moved to the current CUDA device and the result is moved back
(the reference returns on the input's device).  Forward only: backward raises, training is
outside this engine.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch
import torch.nn as nn

from . import device as D
from .bspline_kan import BSplineKAN
from .cheby_kan import ChebyKAN
from .fast_kan import FastKAN

_TORCH_KAN = {torch.float32: D.KAN_F32, torch.float16: D.KAN_F16, torch.bfloat16: D.KAN_BF16}


class _KANForward(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, module):
        return module._run(x)

    @staticmethod
    def backward(ctx, grad_output):
        raise NotImplementedError("training (backward) is outside this inference engine")


class TorchMetalKANLinear(nn.Module):
    """KAN layer as an ``nn.Module`` (bases: cheby, fastkan/rbf, bspline/kan)."""

    def __init__(self, in_features: int, out_features: int, basis: str = "cheby",
                 degree: int = 4, bias: bool = True, use_base: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.basis = basis.lower()
        self.degree = degree
        self.use_bias = bias
        if self.basis == "cheby":
            layer = ChebyKAN(in_features, out_features, degree=degree, bias=bias, use_base=use_base)
            w_main = layer.w_cheby
        elif self.basis in ("fastkan", "rbf"):
            layer = FastKAN(in_features, out_features, num_centers=degree, bias=bias,
                            use_base=use_base)
            w_main = layer.w_rbf
        elif self.basis in ("bspline", "kan"):
            layer = BSplineKAN(in_features, out_features, grid_size=degree, bias=bias)
            w_main = layer.w_spline
        else:
            raise ValueError(f"Unsupported basis type: {basis}")
        self.metal_layer = layer
        self.weight = nn.Parameter(torch.from_numpy(np.array(w_main, np.float32)))
        self.base_weight = (nn.Parameter(torch.from_numpy(np.array(layer.w_base, np.float32)))
                            if layer.has_base else None)
        self.bias_param = (nn.Parameter(torch.from_numpy(np.array(layer.bias, np.float32)))
                           if layer.has_bias else None)
        if self.basis in ("fastkan", "rbf"):
            self.register_buffer("grid", torch.from_numpy(np.array(layer.grid, np.float32)))
        self._cast_cache = {}

    def _as(self, t: torch.Tensor, dtype, device, key: str) -> torch.Tensor:
        """Parameter ``t`` as a contiguous ``dtype`` tensor on ``device`` (cached per version)."""
        ver = (t._version, t.data_ptr(), dtype, device)
        hit = self._cast_cache.get(key)
        if hit is not None and hit[0] == ver:
            return hit[1]
        c = t.detach().to(device=device, dtype=dtype).contiguous()
        self._cast_cache[key] = (ver, c)
        return c

    def _run(self, x: torch.Tensor) -> torch.Tensor:
        orig_device = x.device
        dev = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
        dtype = x.dtype if x.dtype in _TORCH_KAN else torch.float32
        x2 = x.detach().to(device=dev, dtype=dtype).reshape(-1, self.in_features).contiguous()
        B = x2.shape[0]
        y = torch.empty((B, self.out_features), device=dev, dtype=dtype)
        lay = self.metal_layer
        L = D.KanLayer()
        L.basis = lay.BASIS
        L.act_dtype = _TORCH_KAN[dtype]
        L.D_in, L.D_out, L.K = self.in_features, self.out_features, lay._terms()
        L.has_base = int(self.base_weight is not None)
        L.has_bias = int(self.bias_param is not None)
        L.ln_eps = 1e-5
        keep = []
        w = self._as(self.weight, dtype, dev, "w")
        keep.append(w)
        L.w.format, L.w.data = D.KAN_W_DENSE, w.data_ptr()
        if self.base_weight is not None:
            wb = self._as(self.base_weight, dtype, dev, "wb")
            keep.append(wb)
            L.wb.format, L.wb.data = D.KAN_W_DENSE, wb.data_ptr()
        if self.bias_param is not None:
            b = self._as(self.bias_param, dtype, dev, "b")
            keep.append(b)
            L.bias = b.data_ptr()
        if lay.BASIS == D.KAN_RBF:
            g = self._as(self.grid, torch.float32, dev, "grid")
            keep.append(g)
            L.grid, L.inv_den = g.data_ptr(), float(lay.inv_denominator)
        elif lay.BASIS == D.KAN_BSPLINE:
            L.grid_size, L.grid_min, L.inv_h = int(lay.grid_size), float(lay.grid[0]), float(lay.grid[1])
        if B:
            with torch.cuda.device(dev):
                stream = torch.cuda.current_stream(dev).cuda_stream
                D.get_metal_bridge().kan_forward(ctypes.byref(L), ctypes.c_void_p(x2.data_ptr()),
                                                 ctypes.c_void_p(y.data_ptr()), B,
                                                 ctypes.c_void_p(stream))
        y = y.reshape(*x.shape[:-1], self.out_features)
        return y if orig_device == dev else y.to(orig_device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _KANForward.apply(x, self)


class TorchMetalKAN(nn.Module):
    """Stack of :class:`TorchMetalKANLinear` layers."""

    def __init__(self, layers_hidden: Sequence[int], basis: str = "cheby", degree: int = 4,
                 bias: bool = True):
        super().__init__()
        self.layers = nn.ModuleList([
            TorchMetalKANLinear(i, o, basis=basis, degree=degree, bias=bias)
            for i, o in zip(layers_hidden, layers_hidden[1:])])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x)
        return x
