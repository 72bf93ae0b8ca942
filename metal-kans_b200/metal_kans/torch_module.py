"""PyTorch interop: ``nn.Module`` wrappers running the CUDA engine on torch tensors.

Replaces the reference's ``metal_kans/torch_module.py:19-137``, whose autograd function copies
every input to host NumPy and back (``:27-31``).  Here tensors stay on the GPU: the layer is the
custom operator ``metal_kans::kan_linear`` (forward through ``kan_forward`` on torch's current
stream, the parameters' ``data_ptr()`` handed to the engine) with its gradient registered as a
second operator, ``metal_kans::kan_linear_backward`` (``kan_backward``: dX, dW, dW_base, dbias in
fp32).  Both have fake (shape-only) implementations, so ``torch.compile`` traces through them
without a graph break.  Inputs on the CPU are moved to the current CUDA device and the result is
moved back (the reference returns on the input's device).  Gradients are computed in fp32 for the
raw-input Chebyshev / RBF / B-spline layers these modules build.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn as nn

from . import device as D
from .bspline_kan import BSplineKAN
from .cheby_kan import ChebyKAN
from .fast_kan import FastKAN
from .relu_kan import ReLUKAN

_TORCH_KAN = {torch.float32: D.KAN_F32, torch.float16: D.KAN_F16, torch.bfloat16: D.KAN_BF16}


def _descriptor(basis: int, dtype, D_in: int, D_out: int, K: int, weight, base_weight, bias,
                grid, grid_size: int, grid_min: float, inv_h: float, inv_den: float):
    L = D.KanLayer()
    L.basis = basis
    L.act_dtype = _TORCH_KAN[dtype]
    L.D_in, L.D_out, L.K = D_in, D_out, K
    L.has_base = int(base_weight is not None)
    L.has_bias = int(bias is not None)
    L.ln_eps = 1e-5
    L.w.format, L.w.data = D.KAN_W_DENSE, weight.data_ptr()
    if base_weight is not None:
        L.wb.format, L.wb.data = D.KAN_W_DENSE, base_weight.data_ptr()
    if bias is not None:
        L.bias = bias.data_ptr()
    if basis == D.KAN_RBF:
        L.grid, L.inv_den = grid.data_ptr(), float(inv_den)
    elif basis == D.KAN_BSPLINE:
        L.grid_size, L.grid_min, L.inv_h = int(grid_size), float(grid_min), float(inv_h)
    elif basis == D.KAN_RELU:
        L.grid, L.inv_h = grid.data_ptr(), float(inv_h)
    return L


def _on(t: Optional[torch.Tensor], dev, dtype):
    return None if t is None else t.detach().to(device=dev, dtype=dtype).contiguous()


@torch.library.custom_op("metal_kans::kan_linear", mutates_args=())
def kan_linear(x: torch.Tensor, weight: torch.Tensor, base_weight: Optional[torch.Tensor],
               bias: Optional[torch.Tensor], grid: Optional[torch.Tensor], basis: int, K: int,
               grid_size: int, grid_min: float, inv_h: float, inv_den: float) -> torch.Tensor:
    """One fused KAN layer: x [..., D_in] -> [..., D_out] (weight [D_out, D_in*K])."""
    D_out, D_in = weight.shape[0], x.shape[-1]
    dev = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
    dtype = x.dtype if x.dtype in _TORCH_KAN else torch.float32
    x2 = x.detach().to(device=dev, dtype=dtype).reshape(-1, D_in).contiguous()
    B = x2.shape[0]
    y = torch.empty((B, D_out), device=dev, dtype=dtype)
    w, wb, b = _on(weight, dev, dtype), _on(base_weight, dev, dtype), _on(bias, dev, dtype)
    g = _on(grid, dev, torch.float32)
    L = _descriptor(basis, dtype, D_in, D_out, K, w, wb, b, g, grid_size, grid_min, inv_h, inv_den)
    if B:
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
            D.get_metal_bridge().kan_forward(ctypes.byref(L), ctypes.c_void_p(x2.data_ptr()),
                                             ctypes.c_void_p(y.data_ptr()), B,
                                             ctypes.c_void_p(stream))
    y = y.reshape(*x.shape[:-1], D_out)
    return y if x.device == dev else y.to(x.device)


@kan_linear.register_fake
def _(x, weight, base_weight, bias, grid, basis, K, grid_size, grid_min, inv_h, inv_den):
    dtype = x.dtype if x.dtype in _TORCH_KAN else torch.float32
    return x.new_empty((*x.shape[:-1], weight.shape[0]), dtype=dtype)


@torch.library.custom_op("metal_kans::kan_linear_backward", mutates_args=())
def kan_linear_backward(grad_y: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                        base_weight: Optional[torch.Tensor], has_bias: bool,
                        grid: Optional[torch.Tensor], basis: int, K: int, grid_size: int,
                        grid_min: float, inv_h: float, inv_den: float
                        ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """fp32 gradients (dX, dW, dW_base, dbias); dW_base / dbias are empty without a base branch
    / bias."""
    D_out, D_in = weight.shape[0], x.shape[-1]
    dev = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
    f32 = torch.float32
    x2 = x.detach().to(device=dev, dtype=f32).reshape(-1, D_in).contiguous()
    gy = grad_y.detach().to(device=dev, dtype=f32).reshape(-1, D_out).contiguous()
    B = x2.shape[0]
    w, wb, g = _on(weight, dev, f32), _on(base_weight, dev, f32), _on(grid, dev, f32)
    dX = torch.empty((B, D_in), device=dev, dtype=f32)
    dW = torch.empty((D_out, D_in * K), device=dev, dtype=f32)
    dWb = torch.empty((D_out, D_in) if wb is not None else (0,), device=dev, dtype=f32)
    db = torch.empty((D_out,) if has_bias else (0,), device=dev, dtype=f32)
    L = _descriptor(basis, f32, D_in, D_out, K, w, wb, None, g, grid_size, grid_min, inv_h, inv_den)
    L.has_bias = int(has_bias)
    if B:
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
            D.get_metal_bridge().kan_backward(
                ctypes.byref(L), ctypes.c_void_p(x2.data_ptr()), ctypes.c_void_p(gy.data_ptr()),
                ctypes.c_void_p(dX.data_ptr()), ctypes.c_void_p(dW.data_ptr()),
                ctypes.c_void_p(dWb.data_ptr() if wb is not None else 0),
                ctypes.c_void_p(db.data_ptr() if has_bias else 0), B, ctypes.c_void_p(stream))
    else:
        dW.zero_(), dWb.zero_(), db.zero_()
    return dX.reshape(x.shape), dW, dWb, db


@kan_linear_backward.register_fake
def _(grad_y, x, weight, base_weight, has_bias, grid, basis, K, grid_size, grid_min, inv_h,
      inv_den):
    f32 = torch.float32
    D_out, D_in = weight.shape[0], x.shape[-1]
    return (x.new_empty(x.shape, dtype=f32), x.new_empty((D_out, D_in * K), dtype=f32),
            x.new_empty((D_out, D_in) if base_weight is not None else (0,), dtype=f32),
            x.new_empty((D_out,) if has_bias else (0,), dtype=f32))


def _setup_context(ctx, inputs, output):
    x, weight, base_weight, bias, grid, basis, K, grid_size, grid_min, inv_h, inv_den = inputs
    ctx.save_for_backward(x, weight, base_weight, grid)
    ctx.has_bias = bias is not None
    ctx.meta = (basis, K, grid_size, grid_min, inv_h, inv_den)
    ctx.dtypes = (x.dtype, weight.dtype, None if base_weight is None else base_weight.dtype,
                  None if bias is None else bias.dtype)


def _backward(ctx, grad_y):
    x, weight, base_weight, grid = ctx.saved_tensors
    dX, dW, dWb, db = kan_linear_backward(grad_y, x, weight, base_weight, ctx.has_bias, grid,
                                          *ctx.meta)
    xd, wd, wbd, bd = ctx.dtypes
    return (dX.to(xd), dW.to(wd), None if wbd is None else dWb.to(wbd),
            None if bd is None else db.to(bd), None, None, None, None, None, None, None)


kan_linear.register_autograd(_backward, setup_context=_setup_context)


class TorchMetalKANLinear(nn.Module):
    """KAN layer as an ``nn.Module`` (bases: cheby, fastkan/rbf, bspline/kan, relu/relukan)."""

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
        elif self.basis in ("relu", "relukan"):
            layer = ReLUKAN(in_features, out_features, num_grids=degree, bias=bias,
                            use_base=use_base)
            w_main = layer.w_relu
        else:
            raise ValueError(f"Unsupported basis type: {basis}")
        self.metal_layer = layer
        self.weight = nn.Parameter(torch.from_numpy(np.array(w_main, np.float32)))
        self.base_weight = (nn.Parameter(torch.from_numpy(np.array(layer.w_base, np.float32)))
                            if layer.has_base else None)
        self.bias_param = (nn.Parameter(torch.from_numpy(np.array(layer.bias, np.float32)))
                           if layer.has_bias else None)
        if self.basis in ("fastkan", "rbf", "relu", "relukan"):
            self.register_buffer("grid", torch.from_numpy(np.array(layer.grid, np.float32)))
        else:
            self.grid = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lay = self.metal_layer
        g = lay.grid if lay.BASIS == D.KAN_BSPLINE else None
        return kan_linear(x, self.weight, self.base_weight, self.bias_param, self.grid,
                          int(lay.BASIS), int(lay._terms()),
                          int(getattr(lay, "grid_size", 0)),
                          float(g[0]) if g is not None else 0.0,
                          float(g[1]) if g is not None else float(getattr(lay, "inv_h", 0.0)),
                          float(getattr(lay, "inv_denominator", 0.0)))


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


class TorchGatedKAN(nn.Module):
    """GatedKAN FFN block as an ``nn.Module`` (new: the reference has no torch GatedKAN):
    hidden = silu(gate(x)) * up(x) with the SiLU argument clamped to +-20 inside the sigmoid, then
    down(hidden) -- three Chebyshev layers of ``degree`` terms, differentiable end to end."""

    def __init__(self, d_model: int, d_ffn: Optional[int] = None, degree: int = 4,
                 has_base: bool = True, has_bias: bool = False):
        super().__init__()
        d_ffn = int(d_ffn if d_ffn is not None else 2 * d_model)
        self.d_model, self.d_ffn = int(d_model), d_ffn
        self.gate = TorchMetalKANLinear(d_model, d_ffn, "cheby", degree, has_bias, has_base)
        self.up = TorchMetalKANLinear(d_model, d_ffn, "cheby", degree, has_bias, has_base)
        self.down = TorchMetalKANLinear(d_ffn, d_model, "cheby", degree, has_bias, has_base)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        g = self.gate(x)
        hidden = g * torch.sigmoid(g.clamp(-20.0, 20.0)) * self.up(x)
        return self.down(hidden)
