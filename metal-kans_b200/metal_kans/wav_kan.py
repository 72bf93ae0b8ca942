"""WavKAN layer (continuous wavelets) on the B200 engine.

Drop-in for ``metal_kans/wav_kan.py:13-171``: wavelet types mexican_hat=0 / morlet=1 / dog=2,
``translation[D_in, W]``, ``scale`` with ``_inv_scale = 1 / (|scale| + 1e-4)``, ``w_wav``.  The
fp16 mode mirrors ``fused_kan.metal:1514-1548`` including its Morlet frequency of 1.75 (the fp32
kernel uses 5).
"""
from __future__ import annotations

import math

import numpy as np

from . import device as D
from ._layer import KANLayerBase


class WavKAN(KANLayerBase):
    """Fused WavKAN layer."""

    BASIS = D.KAN_WAVELET
    MAIN = "w_wav"
    _WEIGHTS = ("w_wav", "w_base", "bias", "translation", "_inv_scale")
    _HALF_EXTRA = ("translation", "_inv_scale")

    def __init__(self, in_features: int, out_features: int, num_wavelets: int = 8,
                 wavelet_type: str = "mexican_hat", bias: bool = True, use_base: bool = True,
                 input_map: str = "none"):
        self.in_features = in_features
        self.out_features = out_features
        self.num_wavelets = num_wavelets
        self.wavelet_type_str = wavelet_type.lower()
        if self.wavelet_type_str == "morlet":
            self.wavelet_type = 1
        elif self.wavelet_type_str in ("dog", "derivative_of_gaussian"):
            self.wavelet_type = 2
        else:
            self.wavelet_type = 0
        self.has_base = 1 if use_base else 0
        self.has_bias = 1 if bias else 0
        self.input_map = input_map
        # wav_kan.py:46-55, same order
        self.translation = np.random.uniform(-1.0, 1.0, (in_features, num_wavelets)).astype(np.float32)
        self._scale = np.random.uniform(0.5, 2.0, (in_features, num_wavelets)).astype(np.float32)
        self._inv_scale = (1.0 / (np.abs(self._scale) + 1e-4)).astype(np.float32)
        bound = 1.0 / math.sqrt(in_features)
        self.w_wav = np.random.uniform(-bound, bound, (out_features, in_features * num_wavelets)).astype(np.float32)
        self.w_base = (np.random.uniform(-bound, bound, (out_features, in_features)).astype(np.float32)
                       if use_base else np.zeros((1,), dtype=np.float32))
        self.bias = (np.zeros((out_features,), dtype=np.float32) if bias
                     else np.zeros((1,), dtype=np.float32))
        self._bridge = D.get_metal_bridge()

    @property
    def scale(self) -> np.ndarray:
        return self._scale

    @scale.setter
    def scale(self, val: np.ndarray):
        target = self.w_wav.dtype
        self._scale = np.asarray(val, dtype=target)
        self._inv_scale = (1.0 / (np.abs(self._scale) + 1e-4)).astype(target)

    def bfloat16(self):
        # translation / inverse scale stay fp32 in bf16 mode (basis math is fp32 there)
        from ._engine import BFLOAT16

        return self._cast(BFLOAT16, ())

    def _terms(self) -> int:
        return int(self.num_wavelets)

    def _basis_params(self, L, keep):
        t = self._dev_array("trans_f32", np.asarray(self.translation).astype(np.float32), "translation")
        s = self._dev_array("isc_f32", np.asarray(self._inv_scale).astype(np.float32), "_inv_scale")
        keep += [t, s]
        L.translation = t.ptr
        L.inv_scale = s.ptr
        L.wavelet_type = int(self.wavelet_type)

    def benchmark(self, x: np.ndarray, warmup: int = 10, iters: int = 50) -> float:
        """Mean ms of one host-pointer forward (wav_kan.py:144-171 semantics)."""
        if self.dtype != np.float32:
            return self._benchmark_fallback(x, warmup, iters)
        xf = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, self.in_features))
        y = np.empty((xf.shape[0], self.out_features), np.float32)
        return self._bridge.benchmark_metal_wavkan(
            xf.ctypes.data, self.w_wav.ctypes.data, self.w_base.ctypes.data,
            self.translation.ctypes.data, self._inv_scale.ctypes.data, self.bias.ctypes.data,
            y.ctypes.data, xf.shape[0], self.in_features, self.out_features, self.num_wavelets,
            self.wavelet_type, self.has_base, self.has_bias, warmup, iters)
