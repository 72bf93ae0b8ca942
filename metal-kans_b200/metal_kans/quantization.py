"""INT8 / INT4 / ternary / INT2 weight quantisation with the reference's packed layouts.

Drop-in for ``metal_kans/quantization.py:13-449``:

* :class:`QuantizedWeight` -- block-affine INT8/INT4 over the row-padded matrix, groups of
  ``group_size`` consecutive elements, ``qweight`` [groups, gs] (INT8) or [groups, gs/2] (INT4,
  byte = q[2i] | q[2i+1] << 4), ``scales``/``biases`` [groups, 1] fp32 (bias = group minimum);
* :class:`TernaryQuantizedWeight` / :class:`Int2QuantizedWeight` -- 2-bit codes, 16 per uint32
  (element k at bits 2*(k%16) of word k/16), per-(row, group) fp32 scales, global codebook[4];
* :func:`quantize` / :func:`to_int8` / :func:`to_int4` / :func:`to_ternary` / :func:`to_int2` --
  in place: the packed object is stored as ``_{attr}_quantized|_ternary|_int2`` and the attribute
  is replaced by the dequantised fp32 array, exactly like the reference.

Quantisation runs in the engine's host C++ (the reference's bridge functions, bit-exact with
their source); 2-bit dequantisation runs on the GPU like the reference's ``dequantize_*_fast``.
Unlike the reference, a layer keeps using its packed weights afterwards: the forward kernels
decode them (same fp32 values as the dequantised array), so memory traffic shrinks with the bits.
"""
from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from . import device as D
from ._engine import DeviceBuffer


class _PackedMixin:
    """Device copies of the packed arrays + filling a ``KanWeight`` descriptor."""

    def _device(self, name: str) -> DeviceBuffer:
        cache = self.__dict__.setdefault("_dev_bufs", {})
        if name not in cache:
            cache[name] = DeviceBuffer.from_array(np.ascontiguousarray(getattr(self, name)))
        return cache[name]


class QuantizedWeight(_PackedMixin):
    """Affine block-quantised weight matrix (INT8, or INT4 with two codes per byte)."""

    def __init__(self, weight: np.ndarray, bits: int = 8, group_size: int = 64):
        if bits not in (8, 4):
            raise ValueError(f"Unsupported bits: {bits}. Choose 8 or 4.")
        if bits == 4 and group_size % 2:
            raise ValueError("INT4 needs an even group_size")
        self.bits = bits
        self.group_size = group_size
        self.shape = weight.shape
        out_features, in_features = weight.shape
        pad_in = (group_size - (in_features % group_size)) % group_size
        padded = np.pad(np.asarray(weight, np.float32), ((0, 0), (0, pad_in))) if pad_in \
            else np.array(weight, np.float32)
        padded = np.ascontiguousarray(padded, np.float32)
        self.padded_in_features = padded.shape[1]
        num_groups = padded.size // group_size
        self.scales = np.empty((num_groups, 1), np.float32)
        self.biases = np.empty((num_groups, 1), np.float32)
        lib = D.get_metal_bridge()
        if bits == 8:
            self.qweight = np.empty((num_groups, group_size), np.uint8)
            fn = lib.metal_kan_quantize_int8
        else:
            self.qweight = np.empty((num_groups, group_size // 2), np.uint8)
            fn = lib.metal_kan_quantize_int4
        fn(padded.ctypes.data, self.qweight.ctypes.data, self.scales.ctypes.data,
           self.biases.ctypes.data, num_groups, group_size)

    def dequantize(self) -> np.ndarray:
        """Dequantises back to the original [out, in] float32 matrix (q*s + b per element)."""
        lib = D.get_metal_bridge()
        num_groups = self.scales.shape[0]
        out = np.empty(num_groups * self.group_size, np.float32)
        fn = lib.metal_kan_dequantize_int8 if self.bits == 8 else lib.metal_kan_dequantize_int4
        fn(np.ascontiguousarray(self.qweight).ctypes.data,
           np.ascontiguousarray(self.scales).ctypes.data,
           np.ascontiguousarray(self.biases).ctypes.data, out.ctypes.data, num_groups,
           self.group_size)
        full = out.reshape(-1, self.padded_in_features)
        return np.ascontiguousarray(full[: self.shape[0], : self.shape[1]])

    def _fill_struct(self, w: D.KanWeight, keep: list) -> None:
        q, s, b = self._device("qweight"), self._device("scales"), self._device("biases")
        keep += [q, s, b]
        w.format = D.KAN_W_INT8 if self.bits == 8 else D.KAN_W_INT4
        w.group_size = self.group_size
        w.padded_cols = self.padded_in_features
        w.data, w.scales, w.biases = q.ptr, s.ptr, b.ptr


class TernaryQuantizedWeight(_PackedMixin):
    """1.58-bit ternary weights {-1, 0, +1} x per-group scale (mean |w|), 16 codes per uint32."""

    def __init__(self, weight: np.ndarray, group_size: int = 32):
        self.group_size = group_size
        self.shape = weight.shape
        D_out, K_dim = weight.shape
        w = np.ascontiguousarray(weight, np.float32)
        self.w_packed = np.zeros((D_out, (K_dim + 15) // 16), np.uint32)
        self.scales = np.zeros((D_out, (K_dim + group_size - 1) // group_size), np.float32)
        D.get_metal_bridge().metal_kan_quantize_ternary(
            w.ctypes.data, self.w_packed.ctypes.data, self.scales.ctypes.data, D_out, K_dim,
            group_size)

    def dequantize(self) -> np.ndarray:
        D_out, K_dim = self.shape
        out = np.empty((D_out, K_dim), np.float32)
        D.get_metal_bridge().metal_kan_dequantize_ternary(
            np.ascontiguousarray(self.w_packed).ctypes.data,
            np.ascontiguousarray(self.scales).ctypes.data, out.ctypes.data, D_out, K_dim,
            self.group_size)
        return out

    def _no_code3(self) -> bool:
        """True when no packed code is 3 (checked once, with the device copy it describes)."""
        cache = self.__dict__.setdefault("_dev_bufs", {})
        if "no_code3" not in cache:
            a = np.ascontiguousarray(self.w_packed).view(np.uint32)
            cache["no_code3"] = not np.any(a & (a >> 1) & np.uint32(0x55555555))
        return cache["no_code3"]

    def _fill_struct(self, w: D.KanWeight, keep: list) -> None:
        p, s = self._device("w_packed"), self._device("scales")
        keep += [p, s]
        w.format = D.KAN_W_TERNARY
        w.group_size = self.group_size
        w.flags = D.KAN_WFLAG_TERNARY_NO3 if self._no_code3() else 0
        w.data, w.scales = p.ptr, s.ptr


class Int2QuantizedWeight(_PackedMixin):
    """2-bit codebook weights: codebook[code] x per-group scale (max |w|), 16 codes per uint32."""

    def __init__(self, weight: np.ndarray, group_size: int = 32, codebook: Any = None):
        self.group_size = group_size
        self.shape = weight.shape
        D_out, K_dim = weight.shape
        if codebook is None:
            codebook = np.array([-1.0, -0.33333, 0.33333, 1.0], dtype=np.float32)
        self.codebook = np.ascontiguousarray(codebook, np.float32)
        w = np.ascontiguousarray(weight, np.float32)
        self.w_packed = np.zeros((D_out, (K_dim + 15) // 16), np.uint32)
        self.scales = np.zeros((D_out, (K_dim + group_size - 1) // group_size), np.float32)
        D.get_metal_bridge().metal_kan_quantize_int2(
            w.ctypes.data, self.w_packed.ctypes.data, self.scales.ctypes.data,
            self.codebook.ctypes.data, D_out, K_dim, group_size)

    def dequantize(self) -> np.ndarray:
        D_out, K_dim = self.shape
        out = np.empty((D_out, K_dim), np.float32)
        D.get_metal_bridge().metal_kan_dequantize_int2(
            np.ascontiguousarray(self.w_packed).ctypes.data,
            np.ascontiguousarray(self.scales).ctypes.data, self.codebook.ctypes.data,
            out.ctypes.data, D_out, K_dim, self.group_size)
        return out

    def _fill_struct(self, w: D.KanWeight, keep: list) -> None:
        p, s, c = self._device("w_packed"), self._device("scales"), self._device("codebook")
        keep += [p, s, c]
        w.format = D.KAN_W_INT2
        w.group_size = self.group_size
        w.data, w.scales, w.codebook = p.ptr, s.ptr, c.ptr


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """2-bit codes [rows, cols] (values 0..3) in the packed layout of the ternary and INT2
    weights: 16 codes per uint32, code k of a row at bits 2*(k % 16) of word k // 16, the row's
    last word zero padded (quantization.py:191-286 of the reference)."""
    c = np.asarray(codes)
    rows, cols = c.shape
    words = (cols + 15) // 16
    padded = np.zeros((rows, words * 16), np.uint32)
    padded[:, :cols] = c.astype(np.uint32) & 3
    lanes = padded.reshape(rows, words, 16)
    out = np.zeros((rows, words), np.uint32)
    for j in range(16):
        out |= lanes[:, :, j] << np.uint32(2 * j)
    return out


def packed_from_codes(kind: str, w_packed: np.ndarray, scales: np.ndarray, shape,
                      group_size: int, codebook=None):
    """Build a Ternary/Int2QuantizedWeight straight from its packed codes and scales (same
    layout as the quantisers produce), e.g. for synthetic or externally quantised weights."""
    cls = TernaryQuantizedWeight if kind == "ternary" else Int2QuantizedWeight
    q = cls.__new__(cls)
    q.group_size = int(group_size)
    q.shape = tuple(shape)
    q.w_packed = np.ascontiguousarray(w_packed, np.uint32)
    q.scales = np.ascontiguousarray(scales, np.float32)
    if kind != "ternary":
        q.codebook = np.ascontiguousarray(
            codebook if codebook is not None else [-1.0, -0.33333, 0.33333, 1.0], np.float32)
    return q


def attach_packed(layer: Any, attr: str, q) -> Any:
    """Install packed weight `q` on `layer.attr` the way to_int*/to_ternary do: the attribute
    becomes the dequantised fp32 array and `q` stays authoritative for the kernels."""
    suffix = {QuantizedWeight: "_quantized", TernaryQuantizedWeight: "_ternary",
              Int2QuantizedWeight: "_int2"}[type(q)]
    setattr(layer, f"_{attr}{suffix}", q)
    setattr(layer, attr, q.dequantize())
    q._source_version = getattr(layer, "_versions", {}).get(attr, 0)
    return layer


WEIGHT_ATTRS = ["w_cheby", "w_rbf", "w_relu", "w_wav", "w_fourier", "w_jacobi", "w_p", "w_q",
                "w_spline", "w_up", "w_base"]


def _apply(model: Any, make, suffix: str) -> Any:
    """Walk a layer / net / block like quantization.py:152-178 and pack every 2-D weight."""
    if hasattr(model, "layers"):
        for layer in model.layers:
            _apply(layer, make, suffix)
        return model
    for attr in WEIGHT_ATTRS:
        if attr == "w_base" and not getattr(model, "has_base", True):
            continue
        w = getattr(model, attr, None)
        if isinstance(w, np.ndarray) and w.ndim == 2:
            qw = make(np.asarray(w, np.float32))
            setattr(model, f"_{attr}{suffix}", qw)
            setattr(model, attr, qw.dequantize())
            # the packed object stays authoritative until the attribute is reassigned
            vers = getattr(model, "_versions", {})
            qw._source_version = vers.get(attr, 0)
            for other in ("_quantized", "_ternary", "_int2"):
                if other != suffix and hasattr(model, f"_{attr}{other}"):
                    object.__setattr__(model, f"_{attr}{other}", None)
    for sub in ("sub_layer", "down_layer"):
        if hasattr(model, sub):
            _apply(getattr(model, sub), make, suffix)
    return model


def quantize(model: Any, bits: int = 8, group_size: int = 64) -> Any:
    """Quantises all weight matrices of a layer or network to INT8/INT4 in place."""
    return _apply(model, lambda w: QuantizedWeight(w, bits=bits, group_size=group_size),
                  "_quantized")


def to_int8(model: Any, group_size: int = 64) -> Any:
    """Quantises all weights to INT8."""
    return quantize(model, bits=8, group_size=group_size)


def to_int4(model: Any, group_size: int = 64) -> Any:
    """Quantises all weights to INT4."""
    return quantize(model, bits=4, group_size=group_size)


def to_ternary(model: Any, group_size: int = 32) -> Any:
    """Quantises all weights to 1.58-bit ternary in place."""
    return _apply(model, lambda w: TernaryQuantizedWeight(w, group_size=group_size), "_ternary")


def to_int2(model: Any, group_size: int = 32, codebook: Any = None) -> Any:
    """Quantises all weights to the 2-bit codebook format in place."""
    return _apply(model, lambda w: Int2QuantizedWeight(w, group_size=group_size,
                                                       codebook=codebook), "_int2")
