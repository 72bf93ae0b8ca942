"""NumPy stand-in for the reference's Metal bridge -- TEST INFRASTRUCTURE ONLY.

The reference's layer classes call ``metal_kans.device.get_metal_bridge()``, which returns the
module global ``_lib`` when it is set, before its macOS check (``metal_kans/device.py:36-38``).
Installing :class:`FakeBridge` there lets the reference's own Python classes (constructors,
``.half()``, ``to_int*``, ``GatedKAN``, ``MetalKAN``) run unchanged on Linux, with the Metal /
MPS arithmetic replaced by :mod:`kan_oracle`.  Used only by ``tests/golden/make_goldens.py`` in
the development container (the reference source is not present on the GPU boxes).

Every entry point takes raw addresses (ints), exactly as ctypes passes ``x.ctypes.data``, and
mirrors one exported function of ``metal_kans/kernels/metal_kan_bridge.mm``.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import kan_oracle as O


def _arr(ptr, shape, dtype):
    """View ``prod(shape)`` elements of ``dtype`` at address ``ptr`` as a NumPy array."""
    n = int(np.prod(shape))
    if n == 0:
        return np.zeros(shape, dtype)
    buf = (ctypes.c_char * (n * np.dtype(dtype).itemsize)).from_address(int(ptr))
    return np.frombuffer(buf, dtype=dtype, count=n).reshape(shape)


class FakeBridge:
    """Callable attributes named like the bridge's ``extern "C"`` functions."""

    def __init__(self, quant_semantics: str = "bridge"):
        # "bridge" restates the host C++ quantisers; "fallback" returns -1 so that the
        # reference's own NumPy fallback in quantization.py runs instead.
        self.quant_semantics = quant_semantics
        self.calls = []

    # ---- runtime ------------------------------------------------------------------------
    def metal_kan_init(self, path):
        return 0

    def metal_kan_set_async(self, enabled):
        return 0

    def metal_kan_sync(self):
        return 0

    # ---- forwards (metal_kan_bridge.mm:443, :532, :722, :1069, relu / fourier / jacobi and the
    # _fp16 twins) ------------------------------------------------------------------------------
    def _fwd(self, mode, basis, X, W, Wb, bias, Y, B, D_in, D_out, K, has_base, has_bias,
             **kw):
        dt = np.float16 if mode == "f16" else np.float32
        x = _arr(X, (B, D_in), dt)
        w = _arr(W, (D_out, D_in * K), dt)
        wb = _arr(Wb, (D_out, D_in), dt) if has_base else None
        b = _arr(bias, (D_out,), dt) if has_bias else None
        y = _arr(Y, (B, D_out), dt)
        y[...] = O.kan_layer(x, basis, mode, w, wb, b, K=K, **kw)
        self.calls.append((basis, mode))
        return 0

    def metal_kan_cheby_forward(self, X, W, Wb, bias, Y, B, D_in, D_out, K, hb, hbi):
        return self._fwd("f32", "cheby", X, W, Wb, bias, Y, B, D_in, D_out, K, hb, hbi)

    def metal_kan_cheby_forward_fp16(self, X, W, Wb, bias, Y, B, D_in, D_out, K, hb, hbi):
        return self._fwd("f16", "cheby", X, W, Wb, bias, Y, B, D_in, D_out, K, hb, hbi)

    def metal_kan_fastkan_forward(self, X, W, Wb, grid, bias, Y, B, D_in, D_out, K, inv_den,
                                  hb, hbi):
        g = _arr(grid, (K,), np.float32).copy()
        return self._fwd("f32", "rbf", X, W, Wb, bias, Y, B, D_in, D_out, K, hb, hbi, grid=g,
                         inv_den=inv_den)

    def metal_kan_fastkan_forward_fp16(self, X, W, Wb, grid, bias, Y, B, D_in, D_out, K,
                                       inv_den, hb, hbi):
        g = _arr(grid, (K,), np.float16).copy()
        return self._fwd("f16", "rbf", X, W, Wb, bias, Y, B, D_in, D_out, K, hb, hbi, grid=g,
                         inv_den=inv_den)

    def _bspline(self, mode, X, W, Wb, grid, bias, Y, B, D_in, D_out, G, order, hb, hbi):
        gp = _arr(grid, (2,), np.float32)
        return self._fwd(mode, "bspline", X, W, Wb, bias, Y, B, D_in, D_out, G + 3, hb, hbi,
                         grid_size=G, grid_min=float(gp[0]), inv_h=float(gp[1]))

    def metal_kan_bspline_forward(self, *a):
        return self._bspline("f32", *a)

    def metal_kan_bspline_forward_fp16(self, *a):
        return self._bspline("f16", *a)

    def _wav(self, mode, X, W, Wb, trans, inv_sc, bias, Y, B, D_in, D_out, nw, wtype, hb, hbi):
        dt = np.float16 if mode == "f16" else np.float32
        tr = _arr(trans, (D_in, nw), dt).copy()
        sc = _arr(inv_sc, (D_in, nw), dt).copy()
        return self._fwd(mode, "wavelet", X, W, Wb, bias, Y, B, D_in, D_out, nw, hb, hbi,
                         translation=tr, inv_scale=sc, wavelet_type=wtype)

    def metal_kan_wavkan_forward(self, *a):
        return self._wav("f32", *a)

    def metal_kan_wavkan_forward_fp16(self, *a):
        return self._wav("f16", *a)

    def _relu(self, mode, X, W, Wb, grid, bias, Y, B, D_in, D_out, G, inv_h, hb, hbi):
        g = _arr(grid, (G,), np.float16 if mode == "f16" else np.float32).copy()
        return self._fwd(mode, "relu", X, W, Wb, bias, Y, B, D_in, D_out, G, hb, hbi, grid=g,
                         inv_h=inv_h)

    def metal_kan_relu_forward(self, *a):
        return self._relu("f32", *a)

    def metal_kan_relu_forward_fp16(self, *a):
        return self._relu("f16", *a)

    def _fourier(self, mode, X, W, Wb, bias, Y, B, D_in, D_out, F, hb, hbi):
        return self._fwd(mode, "fourier", X, W, Wb, bias, Y, B, D_in, D_out, 2 * F + 1, hb, hbi,
                         num_freqs=F)

    def metal_kan_fourier_forward(self, *a):
        return self._fourier("f32", *a)

    def metal_kan_fourier_forward_fp16(self, *a):
        return self._fourier("f16", *a)

    def _jacobi(self, mode, X, W, Wb, bias, Y, B, D_in, D_out, deg, alpha, beta, hb, hbi):
        return self._fwd(mode, "jacobi", X, W, Wb, bias, Y, B, D_in, D_out, deg, hb, hbi,
                         alpha=alpha, beta=beta)

    def metal_kan_jacobi_forward(self, *a):
        return self._jacobi("f32", *a)

    def metal_kan_jacobi_forward_fp16(self, *a):
        return self._jacobi("f16", *a)

    def _mult(self, mode, X, W, Wb, grid, bias, Y, B, D_in, D_out, na, nm, K, inv_den, hb, hbi):
        dt = np.float16 if mode == "f16" else np.float32
        internal = na + 2 * nm
        x = _arr(X, (B, D_in), dt)
        w = _arr(W, (internal, D_in * K), dt)
        wb = _arr(Wb, (internal, D_in), dt) if hb else None
        b = _arr(bias, (internal,), dt) if hbi else None
        g = _arr(grid, (K,), dt).copy()
        _arr(Y, (B, D_out), dt)[...] = O.mult_layer(x, mode, w, wb, b, grid=g, inv_den=inv_den,
                                                    num_add=na, num_mult=nm)
        return 0

    def metal_kan_mult_forward(self, *a):
        return self._mult("f32", *a)

    def metal_kan_mult_forward_fp16(self, *a):
        return self._mult("f16", *a)

    def _lowrank(self, mode, X, Wd, Wu, Wb, grid, bias, Y, B, D_in, D_out, rank, K, inv_den, hb,
                 hbi):
        dt = np.float16 if mode == "f16" else np.float32
        x = _arr(X, (B, D_in), dt)
        wd = _arr(Wd, (rank, D_in * K), dt)
        wu = _arr(Wu, (D_out, rank), dt)
        wb = _arr(Wb, (D_out, D_in), dt) if hb else None
        b = _arr(bias, (D_out,), dt) if hbi else None
        g = _arr(grid, (K,), dt).copy()
        _arr(Y, (B, D_out), dt)[...] = O.lowrank_layer(x, mode, wd, wu, wb, b, grid=g,
                                                       inv_den=inv_den)
        return 0

    def metal_kan_lowrank_forward(self, *a):
        return self._lowrank("f32", *a)

    def metal_kan_lowrank_forward_fp16(self, *a):
        return self._lowrank("f16", *a)

    def metal_kan_rational_forward(self, X, Wp, Wq, Wb, bias, Y, B, D_in, D_out, p, q, hb, hbi):
        f = np.float32
        _arr(Y, (B, D_out), f)[...] = O.rational_layer(
            _arr(X, (B, D_in), f), _arr(Wp, (D_out, D_in * p), f), _arr(Wq, (D_out, D_in * q), f),
            _arr(Wb, (D_out, D_in), f) if hb else None, _arr(bias, (D_out,), f) if hbi else None,
            p_degree=p, q_degree=q)
        return 0

    def metal_kan_chain_pipeline_cheby(self, X, Y, B, L, dims, degs, Ws, Wbs, biases):
        """``metal_kan_bridge.mm:1168-1248`` -- note the reference hard-codes degree 4 there
        (``:1210``); the stand-in honours ``degs[]`` like the B200 engine does."""
        x = _arr(X, (B, dims[0]), np.float32).copy()
        for l in range(L):
            d_in, d_out, k = dims[l], dims[l + 1], degs[l]
            w = _arr(Ws[l], (d_out, d_in * k), np.float32)
            wb = _arr(Wbs[l], (d_out, d_in), np.float32) if Wbs[l] else None
            b = _arr(biases[l], (d_out,), np.float32) if biases[l] else None
            x = O.kan_layer(x, "cheby", "f32", w, wb, b, K=k)
        _arr(Y, (B, dims[L]), np.float32)[...] = x
        return 0

    def metal_kan_swiglu_forward(self, gate, up, out, n):
        g = _arr(gate, (n,), np.float32)
        u = _arr(up, (n,), np.float32)
        _arr(out, (n,), np.float32)[...] = O.swiglu(g, u).astype(np.float32)
        return 0

    # ---- quantisers ---------------------------------------------------------------------
    def metal_kan_quantize_int8(self, w, q, s, b, groups, gs):
        return self._qaff(8, w, q, s, b, groups, gs)

    def metal_kan_quantize_int4(self, w, q, s, b, groups, gs):
        return self._qaff(4, w, q, s, b, groups, gs)

    def _qaff(self, bits, w, q, s, b, groups, gs):
        if self.quant_semantics != "bridge":
            return -1
        ww = _arr(w, (groups, gs), np.float32)
        qw, sc, bi, _ = O.quantize_affine(ww, bits, gs, "bridge")
        _arr(q, qw.shape, np.uint8)[...] = qw
        _arr(s, (groups,), np.float32)[...] = sc.ravel()
        _arr(b, (groups,), np.float32)[...] = bi.ravel()
        return 0

    def metal_kan_dequantize_int8(self, q, s, b, out, groups, gs):
        return self._dqaff(8, q, s, b, out, groups, gs)

    def metal_kan_dequantize_int4(self, q, s, b, out, groups, gs):
        return self._dqaff(4, q, s, b, out, groups, gs)

    def _dqaff(self, bits, q, s, b, out, groups, gs):
        if self.quant_semantics != "bridge":
            return -1
        qw = _arr(q, (groups, gs if bits == 8 else gs // 2), np.uint8)
        sc = _arr(s, (groups,), np.float32)
        bi = _arr(b, (groups,), np.float32)
        _arr(out, (groups, gs), np.float32)[...] = O.dequantize_affine(qw, sc, bi, bits, gs)
        return 0

    def metal_kan_quantize_ternary(self, W, P, s, D_out, K_dim, gs):
        if self.quant_semantics != "bridge":
            return -1
        p, sc = O.quantize_ternary(_arr(W, (D_out, K_dim), np.float32), gs, "bridge")
        _arr(P, p.shape, np.uint32)[...] = p
        _arr(s, sc.shape, np.float32)[...] = sc
        return 0

    def metal_kan_quantize_int2(self, W, P, s, cb, D_out, K_dim, gs):
        if self.quant_semantics != "bridge":
            return -1
        c = _arr(cb, (4,), np.float32).copy()
        p, sc = O.quantize_int2(_arr(W, (D_out, K_dim), np.float32), gs, c, "bridge")
        _arr(P, p.shape, np.uint32)[...] = p
        _arr(s, sc.shape, np.float32)[...] = sc
        return 0

    def metal_kan_dequantize_ternary(self, P, s, out, D_out, K_dim, gs):
        if self.quant_semantics != "bridge":
            return -1
        words = (K_dim + 15) // 16
        G = (K_dim + gs - 1) // gs
        _arr(out, (D_out, K_dim), np.float32)[...] = O.dequantize_ternary(
            _arr(P, (D_out, words), np.uint32), _arr(s, (D_out, G), np.float32), K_dim, gs)
        return 0

    def metal_kan_dequantize_int2(self, P, s, cb, out, D_out, K_dim, gs):
        if self.quant_semantics != "bridge":
            return -1
        words = (K_dim + 15) // 16
        G = (K_dim + gs - 1) // gs
        _arr(out, (D_out, K_dim), np.float32)[...] = O.dequantize_int2(
            _arr(P, (D_out, words), np.uint32), _arr(s, (D_out, G), np.float32),
            _arr(cb, (4,), np.float32), K_dim, gs)
        return 0


def install(metal_kans_module, quant_semantics: str = "bridge") -> FakeBridge:
    """Install a :class:`FakeBridge` as the reference's loaded bridge and return it."""
    fb = FakeBridge(quant_semantics)
    metal_kans_module.device._lib = fb
    return fb
