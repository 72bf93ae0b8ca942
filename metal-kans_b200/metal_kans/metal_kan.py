"""Sequential multi-layer KAN network on the B200 engine.

Drop-in for ``metal_kans/metal_kan.py:28-288`` (forward side): ``MetalKAN(layers_hidden,
basis_type, degree, bias, use_base, pipeline)``, ``.half()``, ``.float()``, ``async_stream``.
Activations stay on the device between layers (ping-pong buffers); only the input and the final
output cross PCIe.  ``pipeline=True`` on an fp32 Cheby net runs the reference's single-call chain
entry point ``metal_kan_chain_pipeline_cheby``, which here honours each layer's degree (the
reference hard-codes 4 terms, ``metal_kan_bridge.mm:1210``).
Bases served by this engine: every basis_type of the reference -- cheby, fastkan/rbf,
bspline/spline/kan, wav/wavkan/wavelet, relu, fourier, jacobi, rational, mult, lowrank.
"""
from __future__ import annotations

import ctypes
from typing import List, Sequence

import numpy as np

from . import _engine as E
from .bspline_kan import BSplineKAN
from .cheby_kan import ChebyKAN
from .fourier_kan import FourierKAN
from .jacobi_kan import JacobiKAN
from .low_rank_kan import LowRankKAN
from .mult_kan import MultKAN
from .rational_kan import RationalKAN
from .relu_kan import ReLUKAN
from .fast_kan import FastKAN
from .wav_kan import WavKAN

MetalChebyKAN = ChebyKAN
MetalFastKAN = FastKAN


class MetalKAN:
    """Multi-layer KAN network executed layer by layer on the GPU."""

    def __init__(self, layers_hidden: Sequence[int], basis_type: str = "cheby", degree: int = 4,
                 bias: bool = True, use_base: bool = True, pipeline: bool = False):
        self.layers_hidden = list(layers_hidden)
        self.basis_type = basis_type.lower()
        self.degree = degree
        self.bias = bias
        self.use_base = use_base
        self.pipeline = pipeline and (self.basis_type in ("cheby", "chebyshev"))
        self.layers = []
        for i in range(len(layers_hidden) - 1):
            in_f, out_f = layers_hidden[i], layers_hidden[i + 1]
            b = self.basis_type
            if b in ("cheby", "chebyshev"):
                layer = ChebyKAN(in_f, out_f, degree=degree, bias=bias, use_base=use_base)
            elif b in ("fastkan", "rbf"):
                layer = FastKAN(in_f, out_f, num_centers=degree, bias=bias, use_base=use_base)
            elif b in ("wav", "wavkan", "wavelet"):
                layer = WavKAN(in_f, out_f, num_wavelets=degree, bias=bias, use_base=use_base)
            elif b in ("bspline", "spline", "kan"):
                layer = BSplineKAN(in_f, out_f, grid_size=degree, bias=bias, use_base=use_base)
            elif b in ("relukan", "relu", "tent"):
                layer = ReLUKAN(in_f, out_f, num_grids=degree, bias=bias, use_base=use_base)
            elif b in ("fourier", "fourierkan"):
                layer = FourierKAN(in_f, out_f, num_frequencies=degree, bias=bias,
                                   use_base=use_base)
            elif b in ("jacobi", "jacobikan"):
                layer = JacobiKAN(in_f, out_f, degree=degree, bias=bias, use_base=use_base)
            elif b in ("rational", "rationalkan"):
                layer = RationalKAN(in_f, out_f, p_degree=degree, q_degree=max(2, degree // 2),
                                    bias=bias, use_base=use_base)
            elif b in ("mult", "multkan"):
                layer = MultKAN(in_f, out_f, num_grids=degree, bias=bias, use_base=use_base)
            elif b in ("lowrank", "lowrankkan"):
                layer = LowRankKAN(in_f, out_f, rank=degree, num_grids=degree, bias=bias,
                                   use_base=use_base)
            else:
                raise ValueError(f"Unknown or unsupported basis_type for this engine: {basis_type}")
            self.layers.append(layer)
        self._scratch = E._Scratch()

    @property
    def dtype(self) -> np.dtype:
        return self.layers[0].dtype if self.layers else np.dtype(np.float32)

    def half(self) -> "MetalKAN":
        for l in self.layers:
            l.half()
        return self

    def float(self) -> "MetalKAN":
        for l in self.layers:
            l.float()
        return self

    def bfloat16(self) -> "MetalKAN":
        for l in self.layers:
            l.bfloat16()
        return self

    def async_stream(self, batches) -> List[np.ndarray]:
        """Runs several batches back to back and synchronises once (metal_kan.py:105-119)."""
        from .device import set_async, sync

        results = []
        set_async(True)
        try:
            for b in batches:
                results.append(self.forward(b))
        finally:
            sync()
            set_async(False)
        return results

    def forward_device(self, x_ptr: int, y_ptr: int, B: int, stream=None) -> None:
        """Enqueue the whole stack on device buffers (every layer must share one dtype)."""
        esz = self.dtype.itemsize
        width = max(self.layers_hidden)
        bufs = [self._scratch.get("a0", B * width * esz), self._scratch.get("a1", B * width * esz)]
        cur = x_ptr
        for li, layer in enumerate(self.layers):
            nxt = y_ptr if li == len(self.layers) - 1 else bufs[li % 2].ptr
            layer.forward_device(cur, nxt, B, stream)
            cur = nxt

    def forward(self, x: np.ndarray) -> np.ndarray:
        act = self.dtype
        if any(l.dtype != act for l in self.layers):
            for l in self.layers:  # mixed dtypes: each layer casts, like the reference
                x = l(x)
            return x
        x2, orig = E.as_activation(x, act, self.layers_hidden[0])
        self.__dict__["_saved_x"] = x2  # the layers' own inputs are recomputed by backward()
        B = x2.shape[0]
        out_dim = self.layers_hidden[-1]
        if self.pipeline and len(self.layers) > 1 and act == np.float32:
            return E.restore_shape(self._forward_pipelined_cheby(x2), orig, out_dim)
        y = E.pinned_empty((B, out_dim), act)
        if B:
            dx = self._scratch.get("x", x2.nbytes).upload(x2)
            dy = self._scratch.get("y", y.nbytes)
            self.forward_device(dx.ptr, dy.ptr, B)
            E.fetch(dy, y)
        return E.restore_shape(y, orig, out_dim)

    def _forward_pipelined_cheby(self, x2: np.ndarray) -> np.ndarray:
        B = x2.shape[0]
        n = len(self.layers)
        y = np.empty((B, self.layers_hidden[-1]), np.float32)
        dims = (ctypes.c_int * (n + 1))(*self.layers_hidden)
        degs = (ctypes.c_int * n)(*[l.degree for l in self.layers])
        ws = (ctypes.c_void_p * n)(*[l.w_cheby.ctypes.data for l in self.layers])
        wbs = (ctypes.c_void_p * n)(*[l.w_base.ctypes.data if l.has_base else None for l in self.layers])
        bs = (ctypes.c_void_p * n)(*[l.bias.ctypes.data if l.has_bias else None for l in self.layers])
        E.lib().metal_kan_chain_pipeline_cheby(x2.ctypes.data, y.ctypes.data, B, n, dims, degs,
                                               ws, wbs, bs)
        return y

    def __call__(self, x: np.ndarray) -> np.ndarray:
        return self.forward(x)

    def backward(self, dY: np.ndarray) -> np.ndarray:
        """Backward in reverse layer order (metal_kan.py:175-186), returning dX.  The forward
        keeps only the net's input on the host; each layer's input is recomputed here, layer by
        layer, before the reverse sweep fills every layer's gradients."""
        x = self.__dict__.get("_saved_x")
        if x is None:
            raise RuntimeError("Cannot run backward before forward() has been called.")
        h = x
        for layer in self.layers:
            h = layer.forward(h)  # sets the layer's saved input
        grad = dY
        for layer in reversed(self.layers):
            grad = layer.backward(grad)
        return grad

    def train_step(self, x: np.ndarray, target: np.ndarray, optimizer=None, lr: float = 1e-3,
                   beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                   weight_decay: float = 0.01, opt_state=None) -> float:
        """One training step (metal_kan.py:227-283): a one-layer net takes the layer's fused
        step; deeper nets run forward, the MSE gradient 2/B (y - target) on the GPU, backward,
        and ``optimizer.step()`` + ``zero_grad()`` when an optimiser is given."""
        if len(self.layers) == 1 and hasattr(self.layers[0], "train_step"):
            return self.layers[0].train_step(x, target, lr=lr, beta1=beta1, beta2=beta2, eps=eps,
                                             weight_decay=weight_decay, opt_state=opt_state)
        pred = np.ascontiguousarray(self.forward(x), np.float32)
        t = np.ascontiguousarray(np.asarray(target, np.float32).reshape(pred.shape))
        B = pred.shape[0] if pred.ndim == 2 else int(np.prod(pred.shape[:-1]))
        diff = np.empty_like(pred)
        E.lib().metal_kan_calc_mse_loss_backward(pred.ctypes.data, t.ctypes.data,
                                                 diff.ctypes.data, pred.size, 2.0 / float(B))
        self.backward(diff)
        if optimizer is not None:
            optimizer.step()
            self.zero_grad()
        return 0.0

    def zero_grad(self) -> None:
        """Zeros gradients across all layers."""
        for layer in self.layers:
            layer.zero_grad()

    def parameters(self):
        """(param, grad) pairs of every layer (metal_kan.py:194-225)."""
        out = []
        for layer in self.layers:
            out.extend((p, g) for p, g in layer.parameters() if g is not None)
        return out

    def __repr__(self) -> str:
        return f"MetalKAN(layers={self.layers_hidden}, basis={self.basis_type!r})"
