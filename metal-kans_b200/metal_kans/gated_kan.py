"""GatedKAN FFN block on the B200 engine.

Drop-in for ``metal_kans/gated_kan.py:24-282``: three ChebyKAN layers (gate, up: d_model ->
d_ffn; down: d_ffn -> d_model), ``hidden = SiLU(gate) * up`` with the SiLU argument clamped to
+-20 (``gated_kan.py:112-131``, ``fused_kan.metal:2284-2296``), (B, Seq, d) inputs flattened.
The whole block runs on the device through ``kan_gated_forward``: activations never return to
the host between the three layers (the reference syncs four times).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _engine as E
from . import device as D
from .cheby_kan import ChebyKAN
from .quantization import to_int2, to_int4, to_int8, to_ternary


class GatedKAN:
    """Gated KAN block: gate = G(x), up = U(x), hidden = SiLU(gate) * up, out = Down(hidden)."""

    def __init__(self, d_model: int, d_ffn: Optional[int] = None, degree: int = 4,
                 has_base: bool = True, has_bias: bool = False, dtype=np.float32):
        self.d_model = int(d_model)
        self.d_ffn = int(d_ffn if d_ffn is not None else 2 * d_model)
        self.degree = int(degree)
        self.has_base = bool(has_base)
        self.has_bias = bool(has_bias)
        self.dtype = np.dtype(dtype)
        self.gate_kan = ChebyKAN(self.d_model, self.d_ffn, degree=self.degree,
                                 bias=self.has_bias, use_base=self.has_base)
        self.up_kan = ChebyKAN(self.d_model, self.d_ffn, degree=self.degree,
                               bias=self.has_bias, use_base=self.has_base)
        self.down_kan = ChebyKAN(self.d_ffn, self.d_model, degree=self.degree,
                                 bias=self.has_bias, use_base=self.has_base)
        if self.dtype == np.float16:
            self.half()
        elif E.BFLOAT16 is not None and self.dtype == E.BFLOAT16:
            self.bfloat16()
        self._scratch = E._Scratch()

    def _layers(self):
        return (self.gate_kan, self.up_kan, self.down_kan)

    def half(self) -> "GatedKAN":
        for l in self._layers():
            l.half()
        self.dtype = np.dtype(np.float16)
        return self

    def float(self) -> "GatedKAN":
        for l in self._layers():
            l.float()
        self.dtype = np.dtype(np.float32)
        return self

    def bfloat16(self) -> "GatedKAN":
        """New: bf16 compute (the reference has no bf16)."""
        for l in self._layers():
            l.bfloat16()
        self.dtype = E.BFLOAT16
        return self

    def _pair(self, gate_desc, up_desc, keep: list) -> int:
        """Gate and up packed as one tensor-core matrix (built once per weight version of either
        layer); 0 when the two layers cannot share a launch (the block then runs them apart)."""
        if gate_desc.act_dtype == D.KAN_F32:
            return 0
        key = (self.gate_kan.__dict__.get("_tc_cache", (None,))[0],
               self.up_kan.__dict__.get("_tc_cache", (None,))[0])
        hit = self.__dict__.get("_pair_cache")
        if hit is None or hit[0] != key:
            lib = E.lib()
            n = ctypes.c_size_t(0)
            try:
                lib.kan_tc_pair_bytes(ctypes.byref(gate_desc), ctypes.byref(up_desc),
                                      ctypes.byref(n))
            except D.KanError:
                self._pair_cache = (key, None)
                return 0
            buf = E.DeviceBuffer(n.value)
            lib.kan_tc_pack_pair(ctypes.byref(gate_desc), ctypes.byref(up_desc),
                                 ctypes.c_void_p(buf.ptr), None)
            hit = (key, buf)
            self._pair_cache = hit
        if hit[1] is None:
            return 0
        keep.append(hit[1])
        return hit[1].ptr

    def forward_device(self, x_ptr: int, h_ptr: int, y_ptr: int, B: int, stream=None) -> None:
        """Enqueue the block on device buffers: x [B, d_model] -> hidden [B, d_ffn] -> y.  Gate and
        up run as one tensor-core launch (shared basis tiles, SwiGLU in the epilogue) when the
        batch fills the GPU; H is the same either way."""
        keep: list = []
        descs = [l._descriptor(keep) for l in self._layers()]
        pair = self._pair(descs[0], descs[1], keep)
        E.lib().kan_gated_forward_pair(*(ctypes.byref(d) for d in descs), ctypes.c_void_p(pair),
                                       ctypes.c_void_p(x_ptr), ctypes.c_void_p(h_ptr),
                                       ctypes.c_void_p(y_ptr), int(B), stream)
        self._keepalive = keep

    def forward(self, x: np.ndarray) -> np.ndarray:
        """Accepts x of shape (B, d_model) or (B, Seq, d_model)."""
        act = self.gate_kan.dtype
        if self.up_kan.dtype != act or self.down_kan.dtype != act:
            raise TypeError("gate/up/down layers must share one dtype")
        x2, orig = E.as_activation(x, act, self.d_model)
        self.__dict__["_saved_x"] = x2
        B = x2.shape[0]
        y = E.pinned_empty((B, self.d_model), act)
        if B:
            esz = np.dtype(act).itemsize
            dx = self._scratch.get("x", x2.nbytes).upload(x2)
            dh = self._scratch.get("h", B * self.d_ffn * esz)
            dy = self._scratch.get("y", y.nbytes)
            self.forward_device(dx.ptr, dh.ptr, dy.ptr, B)
            E.fetch(dy, y)
        return E.restore_shape(y, orig, self.d_model)

    __call__ = forward

    def backward(self, dY: np.ndarray, fused: bool = True) -> np.ndarray:
        """Backward through down, the SwiGLU gating and gate/up (gated_kan.py:145-219): fills
        every layer's gradients, returns dX.  fp32 blocks.  The forward runs on the device and
        keeps only x; gate and up are recomputed here (their saved inputs are x)."""
        x = self.__dict__.get("_saved_x")
        if x is None:
            raise RuntimeError("Cannot run backward before forward() has been called.")
        if self.gate_kan.dtype != np.float32:
            raise RuntimeError("backward runs on fp32 blocks; call .float() first")
        orig = np.shape(dY)
        dY2 = np.asarray(dY, np.float32).reshape(-1, self.d_model)
        lib = E.lib()
        gate = np.ascontiguousarray(self.gate_kan.forward(x), np.float32)
        up = np.ascontiguousarray(self.up_kan.forward(x), np.float32)
        hidden = np.empty_like(gate)
        lib.metal_kan_swiglu_forward(gate.ctypes.data, up.ctypes.data, hidden.ctypes.data,
                                     gate.size)
        self.down_kan.forward(hidden)  # the down layer's saved input
        d_hidden = np.ascontiguousarray(self.down_kan.backward(dY2, fused=fused), np.float32)
        d_gate = np.empty_like(gate)
        d_up = np.empty_like(up)
        lib.metal_kan_swiglu_backward(d_hidden.ctypes.data, gate.ctypes.data, up.ctypes.data,
                                      d_gate.ctypes.data, d_up.ctypes.data, gate.size)
        dX = self.gate_kan.backward(d_gate, fused=fused) + self.up_kan.backward(d_up, fused=fused)
        return dX.reshape(orig[:-1] + (self.d_model,)) if len(orig) > 2 else dX

    def zero_grad(self) -> None:
        """Zeros stored parameter gradients across all KAN layers."""
        for l in self._layers():
            l.zero_grad()

    def get_trainable_params(self):
        """(param, grad) pairs of the three layers (gated_kan.py:226-237)."""
        out = []
        for l in self._layers():
            out.extend(l.parameters())
        return out

    def to_int8(self, group_size: int = 64) -> "GatedKAN":
        for l in self._layers():
            to_int8(l, group_size=group_size)
        self.dtype = self.gate_kan.dtype
        return self

    def to_int4(self, group_size: int = 64) -> "GatedKAN":
        for l in self._layers():
            to_int4(l, group_size=group_size)
        self.dtype = self.gate_kan.dtype
        return self

    def to_ternary(self, group_size: int = 32) -> "GatedKAN":
        for l in self._layers():
            to_ternary(l, group_size=group_size)
        self.dtype = self.gate_kan.dtype
        return self

    def to_int2(self, group_size: int = 32) -> "GatedKAN":
        for l in self._layers():
            to_int2(l, group_size=group_size)
        self.dtype = self.gate_kan.dtype
        return self

    def parameter_count(self) -> int:
        count = 0
        for kan in self._layers():
            count += kan.w_cheby.size
            if kan.has_base and kan.w_base is not None:
                count += kan.w_base.size
            if kan.has_bias and kan.bias is not None:
                count += kan.bias.size
        return count

    def __repr__(self) -> str:
        return (f"GatedKAN(d_model={self.d_model}, d_ffn={self.d_ffn}, degree={self.degree}, "
                f"has_base={self.has_base}, params={self.parameter_count():,})")
