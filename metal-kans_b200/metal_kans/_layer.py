"""Common machinery of the KAN layer classes: descriptor building and the device forward.

A layer holds NumPy weights (the reference's API surface) mirrored on the device, builds a
``kan_layer`` descriptor (include/kan_cuda.h) and runs ``kan_forward``.  Quantised layers (after
``to_int8/to_int4/to_ternary/to_int2``) run their packed weights: decoded in the kernel (exact
fp32 dequantised values), or, for the tensor-core path, from a dense act-dtype copy of the same
values.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _engine as E
from . import device as D

_MAPS = {None: D.KAN_MAP_NONE, "none": D.KAN_MAP_NONE, "clamp": D.KAN_MAP_NONE,
         "tanh": D.KAN_MAP_TANH, "layernorm": D.KAN_MAP_LAYERNORM}

PACKED_SUFFIXES = ("_quantized", "_ternary", "_int2")


class KANLayerBase(E.DeviceLayerMixin):
    """Base of ChebyKAN / FastKAN / BSplineKAN / WavKAN."""

    BASIS = D.KAN_CHEBY
    MAIN = "w_cheby"
    _WEIGHTS = ("w_base", "bias")

    # ---- dtype handling (reference: .half() / .float(); new: .bfloat16()) ------------------
    @property
    def dtype(self) -> np.dtype:
        return getattr(self, self.MAIN).dtype

    def _cast(self, dt, extra=()):
        def cast_weight(name):
            # a packed weight stays authoritative through a dtype cast: the cast array is its
            # dequantised values rounded to `dt`, exactly what the kernels decode and round to
            q = self._packed(name)
            setattr(self, name, getattr(self, name).astype(dt))
            if q is not None:
                q._source_version = self._version(name)

        cast_weight(self.MAIN)
        if self.has_base:
            cast_weight("w_base")
        if self.has_bias:
            self.bias = self.bias.astype(dt)
        for name in extra:
            setattr(self, name, getattr(self, name).astype(dt))
        return self

    def half(self):
        """Converts layer parameters to FP16 half precision."""
        return self._cast(np.float16, self._HALF_EXTRA)

    def float(self):
        """Converts layer parameters to FP32 single precision."""
        return self._cast(np.float32, self._HALF_EXTRA)

    def bfloat16(self):
        """Converts layer parameters to bf16 (new: the reference has no bf16 mode)."""
        if E.BFLOAT16 is None:
            raise RuntimeError("bf16 needs the ml_dtypes package")
        return self._cast(E.BFLOAT16, ())

    _HALF_EXTRA = ()

    # ---- descriptor --------------------------------------------------------------------------
    def _basis_params(self, L: D.KanLayer, keep: list) -> None:
        """Fill the basis-specific fields of the descriptor (subclasses)."""

    def _packed(self, name: str):
        """The packed weight made by to_int*/quantize for ``name``, if still current."""
        for suf in PACKED_SUFFIXES:
            q = self.__dict__.get(f"_{name}{suf}")
            if q is not None and getattr(q, "_source_version", None) == self._version(name):
                return q
        return None

    def _weight_struct(self, name: str, act_np, keep: list) -> D.KanWeight:
        w = D.KanWeight()
        q = self._packed(name)
        if q is None:
            buf = self._dev(name, act_np)
            keep.append(buf)
            w.format = D.KAN_W_DENSE
            w.data = buf.ptr
            return w
        q._fill_struct(w, keep)
        return w

    def _tc_weights(self, L: D.KanLayer, keep: list) -> None:
        """Attach the tensor-core weight layout (packed once per weight version)."""
        if L.act_dtype == D.KAN_F32:
            return
        key = (self._version(self.MAIN), self._version("w_base"), L.act_dtype,
               id(self._packed(self.MAIN)), id(self._packed("w_base")))
        hit = self.__dict__.get("_tc_cache")
        if hit is None or hit[0] != key:
            n = ctypes.c_size_t(0)
            lib = E.lib()
            lib.kan_tc_packed_bytes(ctypes.byref(L), ctypes.byref(n))
            buf = E.DeviceBuffer(n.value)
            lib.kan_tc_pack(ctypes.byref(L), ctypes.c_void_p(buf.ptr), None)
            hit = (key, buf)
            object.__setattr__(self, "_tc_cache", hit)
        keep.append(hit[1])
        L.tc_weights = hit[1].ptr

    def _desc_key(self):
        """What the descriptor depends on: the public-attribute assignment counter (weights,
        basis parameters such as inv_denominator, the input map and flags are all assigned
        through __setattr__; to_int*/half() reassign the weights) and the dtype."""
        return (self.__dict__.get("_pver", 0), self.dtype.str)

    def _descriptor(self, keep: list) -> D.KanLayer:
        """The ``kan_layer`` descriptor, built once per weight/parameter state and cached (the
        device buffers it points at are kept alive with it)."""
        key = self._desc_key()
        hit = self.__dict__.get("_desc_cache")
        if hit is not None and hit[0] == key:
            keep.extend(hit[2])
            return hit[1]
        own: list = []
        L = self._build_descriptor(own)
        object.__setattr__(self, "_desc_cache", (key, L, own))
        keep.extend(own)
        return L

    def _build_descriptor(self, keep: list) -> D.KanLayer:
        act = self.dtype
        L = D.KanLayer()
        L.basis = self.BASIS
        L.act_dtype = E.kan_dtype(act)
        L.D_in = self.in_features
        L.D_out = self.out_features
        L.K = self._terms()
        L.has_base = int(bool(self.has_base))
        L.has_bias = int(bool(self.has_bias))
        L.input_map = _MAPS[getattr(self, "input_map", "none")]
        L.ln_eps = float(getattr(self, "ln_eps", 1e-5))
        L.w = self._weight_struct(self.MAIN, act, keep)
        if self.has_base:
            L.wb = self._weight_struct("w_base", act, keep)
        if self.has_bias:
            b = self._dev("bias", act)
            keep.append(b)
            L.bias = b.ptr
        self._basis_params(L, keep)
        self._tc_weights(L, keep)
        return L

    # ---- forward -----------------------------------------------------------------------------
    def forward_device(self, x_ptr: int, y_ptr: int, B: int, stream=None, path: int = 0) -> None:
        """Enqueue this layer on device buffers (act dtype, [B, in] -> [B, out])."""
        keep: list = []
        L = self._descriptor(keep)
        lib = E.lib()
        if path:
            lib.kan_forward_path(ctypes.byref(L), ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr),
                                 int(B), int(path), stream)
        else:
            lib.kan_forward(ctypes.byref(L), ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr),
                            int(B), stream)
        self._keepalive = keep  # buffers must outlive the queued kernel

    def forward(self, x: np.ndarray, path: int = 0) -> np.ndarray:
        """Fused CUDA forward: x [..., in_features] -> [..., out_features] in the layer dtype."""
        act = self.dtype
        x2, orig = E.as_activation(x, act, self.in_features)
        # kept for backward(), as the reference's layers do (cheby_kan.py:109)
        self.__dict__["_saved_x"] = x2
        self.__dict__["_saved_shape"] = orig
        B = x2.shape[0]
        y = E.pinned_empty((B, self.out_features), act)
        if B and not path and not D.async_enabled():
            # one call: host copies and kernels on the engine's copy and compute streams
            keep: list = []
            L = self._descriptor(keep)
            E.lib().kan_forward_host(ctypes.byref(L), ctypes.c_void_p(x2.ctypes.data),
                                     ctypes.c_void_p(y.ctypes.data), int(B))
            self._keepalive = keep
        elif B:
            s = self._scratch()
            dx = s.get("x", x2.nbytes).upload(x2)
            dy = s.get("y", y.nbytes)
            self.forward_device(dx.ptr, dy.ptr, B, None, path)
            E.fetch(dy, y)
        return E.restore_shape(y, orig, self.out_features)

    __call__ = forward

    # ---- training: fp32 backward like the reference's layers (cheby_kan.py:145-231) --------
    def _backward_call(self, lib, dY, x, dW, dWb, dbias, dX, fused):
        """The bridge's host-pointer backward for this basis (subclasses)."""
        raise NotImplementedError(f"{type(self).__name__} has no backward in the reference")

    def backward(self, dY: np.ndarray, fused: bool = True) -> np.ndarray:
        """GPU backward of the last forward: fills ``grad_<weight>``, ``grad_w_base`` and
        ``grad_bias`` (fp32, overwritten, not accumulated -- as the reference) and returns dX in
        the shape of the forward's input.  fp32 layers with the raw input only."""
        x = self.__dict__.get("_saved_x")
        if x is None:
            raise RuntimeError("Cannot run backward before forward() has been called.")
        if self.dtype != np.float32:
            raise RuntimeError("backward runs on fp32 layers (the reference trains in fp32); "
                               "call .float() first")
        if getattr(self, "input_map", "none") not in (None, "none", "clamp"):
            raise NotImplementedError("backward takes the raw input (no tanh / LayerNorm map)")
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0]
        dY = np.ascontiguousarray(np.asarray(dY, np.float32).reshape(B, self.out_features))
        d = self.__dict__
        main = getattr(self, self.MAIN)

        def grad_array(name, shape):
            # reused (zeroed) when it exists, as the reference does (cheby_kan.py:165-178): an
            # optimiser holding the (param, grad) pairs of parameters() sees every new gradient
            g = d.get(name)
            if g is None or g.shape != shape or g.dtype != np.float32:
                g = d[name] = np.zeros(shape, np.float32)
            else:
                g.fill(0)
            return g

        grad_array("grad_" + self.MAIN, main.shape)
        grad_array("grad_w_base", self.w_base.shape if self.has_base else (1,))
        grad_array("grad_bias", self.bias.shape if self.has_bias else (1,))
        dX = np.empty((B, self.in_features), np.float32)
        self._backward_call(E.lib(), dY, x, d["grad_" + self.MAIN],
                            d["grad_w_base"] if self.has_base else None,
                            d["grad_bias"] if self.has_bias else None, dX, fused)
        shape = d.get("_saved_shape")
        return dX.reshape(shape) if shape is not None and len(shape) > 2 else dX

    def zero_grad(self) -> None:
        """Zeros the stored parameter gradients."""
        for name in ("grad_" + self.MAIN, "grad_w_base", "grad_bias"):
            g = self.__dict__.get(name)
            if g is not None:
                g.fill(0)

    def parameters(self):
        """(param, grad) pairs of the trainable arrays (fast_kan.py:80-87)."""
        d = self.__dict__
        params = [(self._register_param(self.MAIN), d.get("grad_" + self.MAIN))]
        if self.has_base and d.get("grad_w_base") is not None:
            params.append((self._register_param("w_base"), d["grad_w_base"]))
        if self.has_bias and d.get("grad_bias") is not None:
            params.append((self._register_param("bias"), d["grad_bias"]))
        return params

    def _train_call(self, lib, x, target, W, Wb, bias, st, hyper):
        """The bridge's fused training step for this basis (subclasses)."""
        raise NotImplementedError(f"{type(self).__name__} has no fused training step in the "
                                  "reference")

    def train_step(self, x: np.ndarray, target: np.ndarray, lr: float = 1e-3, beta1: float = 0.9,
                   beta2: float = 0.999, eps: float = 1e-8, weight_decay: float = 0.01,
                   opt_state: Optional[dict] = None, optimizer=None, **kwargs) -> float:
        """Fused training step on the GPU (cheby_kan.py:258-343): forward, MSE gradient
        (2/B (y - target)), weight / base / bias gradients and an AdamW update, in one call.
        The AdamW moments live in ``opt_state`` (or the layer's ``_fused_opt_state``) as the
        reference keeps them; returns 0.0 like the reference."""
        import math

        if optimizer is not None:
            lr = getattr(optimizer, "lr", lr)
            beta1 = getattr(optimizer, "beta1", beta1)
            beta2 = getattr(optimizer, "beta2", beta2)
            eps = getattr(optimizer, "eps", eps)
            weight_decay = getattr(optimizer, "weight_decay", weight_decay)
        if self.dtype != np.float32:
            raise RuntimeError("train_step runs on fp32 layers (the reference trains in fp32)")
        if getattr(self, "input_map", "none") not in (None, "none", "clamp"):
            raise NotImplementedError("train_step takes the raw input (no tanh / LayerNorm map)")
        x = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        target = np.ascontiguousarray(np.asarray(target, np.float32).reshape(x.shape[0], -1))
        if target.shape[1] != self.out_features:
            raise ValueError(f"target has {target.shape[1]} columns, expected {self.out_features}")
        main = getattr(self, self.MAIN)
        if opt_state is None:
            st = self.__dict__.get("_fused_opt_state")
            if st is None:
                z = lambda a, on: np.zeros_like(a, np.float32) if on else np.zeros((1,), np.float32)  # noqa: E731
                st = {"m_w": np.zeros_like(main, np.float32), "v_w": np.zeros_like(main, np.float32),
                      "m_wb": z(self.w_base, self.has_base), "v_wb": z(self.w_base, self.has_base),
                      "m_b": z(self.bias, self.has_bias), "v_b": z(self.bias, self.has_bias),
                      "step": 0}
                self.__dict__["_fused_opt_state"] = st
        else:
            st = opt_state
        st["step"] += 1
        t = st["step"]
        lr_t = lr * math.sqrt(1.0 - beta2 ** t) / (1.0 - beta1 ** t)
        # writable copies, updated in place by the step and assigned back (a new weight version:
        # the device copies are refreshed on the next forward)
        W = np.array(main, np.float32)
        Wb = np.array(self.w_base, np.float32) if self.has_base else None
        bias = np.array(self.bias, np.float32) if self.has_bias else None
        self._train_call(E.lib(), x, target, W, Wb, bias, st,
                         (lr, beta1, beta2, eps, weight_decay, lr_t))
        setattr(self, self.MAIN, W)
        if self.has_base:
            self.w_base = Wb
        if self.has_bias:
            self.bias = bias
        return 0.0

    @staticmethod
    def _train_ptrs(W, Wb, bias, st, has_base, has_bias):
        P = lambda a, on=True: a.ctypes.data if (a is not None and on) else None  # noqa: E731
        return (P(W), P(Wb, has_base), P(bias, has_bias), P(st["m_w"]), P(st["v_w"]),
                P(st["m_wb"], has_base), P(st["v_wb"], has_base), P(st["m_b"], has_bias),
                P(st["v_b"], has_bias))

    def _benchmark_fallback(self, x, warmup, iters):
        import time

        for _ in range(warmup):
            self.forward(x)
        t0 = time.perf_counter()
        for _ in range(iters):
            self.forward(x)
        return (time.perf_counter() - t0) * 1e3 / iters
