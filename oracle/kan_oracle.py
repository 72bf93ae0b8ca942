"""CPU oracle for the fused KAN forward path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import this module, and only as the checker or as the timed CPU
baseline.  The product (``metal_kans`` + ``libkan_cuda.so``) never calls it.

It restates, in NumPy, the arithmetic of the reference (Shuril/metal-kans, ``metal_kans`` v0.6.0):

* basis kernels of ``metal_kans/kernels/fused_kan.metal`` (fp32 kernels and their fp16 twins),
  with the rounding points of each kernel mirrored;
* the projection ``Y = bias + silu(x) W_base^T + Phi W^T`` that the bridge runs as two MPS GEMMs
  (``metal_kans/kernels/metal_kan_bridge.mm:443-530``).  The MPS accumulation order is not
  published, so this oracle accumulates in float64 and rounds once to the output dtype;
* the host C++ quantisers/dequantisers of the bridge (``metal_kan_bridge.mm:4177-4302``,
  ``:4634-4682``, ``:4735-4788``) and the GPU dequantisers (``fused_kan.metal:2392-2441``),
  bit-exactly, plus the NumPy fallbacks of ``metal_kans/quantization.py`` (``semantics="numpy"``).

Pinning: the quantisers are pinned bit-exactly against the reference's own NumPy code paths run
in this container (``tests/golden/make_goldens.py``).  The layer classes of the reference were
driven end to end by a NumPy stand-in for its Metal bridge (``oracle/fake_bridge.py``) to produce
the golden layer outputs; the Metal basis kernels and MPS GEMM themselves cannot run off macOS,
so the basis/projection arithmetic is a restatement, not a re-execution ("parity partially
pinned").

Dtype conventions: ``"f32"`` mirrors the fp32 kernels (basis math evaluated exactly, in float64);
``"f16"`` mirrors the ``*_fp16`` kernels (half arithmetic where the reference uses half,
fp32 math + half store where it stores half); ``"bf16"`` (new, no reference counterpart) rounds x
to bf16, evaluates the basis exactly and rounds it to bf16.
"""
from __future__ import annotations

import numpy as np

try:  # bf16 rounding for the bf16 mode
    import ml_dtypes

    BF16 = np.dtype(ml_dtypes.bfloat16)
except Exception:  # pragma: no cover
    ml_dtypes = None
    BF16 = None

F16 = np.dtype(np.float16)
F32 = np.dtype(np.float32)

ACT_DTYPES = {"f32": F32, "f16": F16}
if BF16 is not None:
    ACT_DTYPES["bf16"] = BF16


def act_dtype(mode: str) -> np.dtype:
    return ACT_DTYPES[mode]


def _h(a):
    """Round to IEEE half (round-to-nearest-even)."""
    return np.asarray(a).astype(np.float16)


def _round_mode(a64: np.ndarray, mode: str) -> np.ndarray:
    """Round exact (float64) basis values to the operand dtype of ``mode``."""
    if mode == "f32":
        return a64
    if mode == "f16":
        return a64.astype(np.float32).astype(np.float16).astype(np.float64)
    return a64.astype(np.float32).astype(BF16).astype(np.float64)


def to_mode(x, mode: str) -> np.ndarray:
    """Round an array to the activation dtype of ``mode`` (x is rounded before any math)."""
    return np.asarray(x, dtype=np.float32).astype(act_dtype(mode))


# --------------------------------------------------------------------------------------------
# Input maps (new pre-ops: tanh for the ChebyKAN config, LayerNorm for the FastKAN config)
# --------------------------------------------------------------------------------------------

def layernorm(x: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """Row LayerNorm without affine parameters, statistics in float64 (population variance).

    No reference counterpart: the FastKAN benchmark config asks for an input LayerNorm that
    the reference lacks.  Returned in float64; callers round to the activation dtype.
    """
    x64 = np.asarray(x, dtype=np.float64)
    mu = x64.mean(axis=-1, keepdims=True)
    var = ((x64 - mu) ** 2).mean(axis=-1, keepdims=True)
    return (x64 - mu) / np.sqrt(var + eps)


def apply_input_map(x_act: np.ndarray, input_map: str, mode: str) -> np.ndarray:
    """Apply the pre-op to the activation-dtype input; result is rounded back to the act dtype
    (the kernel hands the mapped value to the basis in the activation dtype)."""
    if input_map in ("none", "clamp", None):
        return x_act
    if input_map == "tanh":
        y = np.tanh(x_act.astype(np.float64))
    elif input_map == "layernorm":
        y = layernorm(x_act)
    else:
        raise ValueError(input_map)
    return y.astype(np.float32).astype(act_dtype(mode)) if mode != "f32" else y.astype(np.float32)


# --------------------------------------------------------------------------------------------
# Base branch: SiLU on the raw input
# --------------------------------------------------------------------------------------------

def silu(x_act: np.ndarray, mode: str) -> np.ndarray:
    """SiLU column values, float64.

    fp32: ``x / (1 + exp2(-log2e x))`` (``fused_kan.metal:116-138``) -> exact math.
    fp16: ``x / (1.0h + exp(-x))`` in half arithmetic (``fused_kan.metal:1373-1397``):
          three half roundings (exp, add, divide).
    bf16: exact math rounded to bf16.
    """
    if mode == "f16":
        xh = x_act.astype(np.float16)
        e = _h(np.exp(-xh.astype(np.float64)))
        d = _h(np.float64(1.0) + e.astype(np.float64))
        return _h(xh.astype(np.float64) / d.astype(np.float64)).astype(np.float64)
    x64 = x_act.astype(np.float64)
    return _round_mode(x64 / (1.0 + np.exp(-x64)), mode)


# --------------------------------------------------------------------------------------------
# Bases.  Each returns Phi[B, D_in*K] (float64, already rounded to the operand dtype), column
# i*K + k, which is the column order of the reference weight matrices (cheby_kan.py:40).
# --------------------------------------------------------------------------------------------

def cheby_basis(x_act: np.ndarray, K: int, mode: str) -> np.ndarray:
    """Chebyshev T_0..T_{K-1} of clamp(x, -1, 1).

    ``fused_kan.metal:205-238`` (fp32: recurrence 2x T1 - T0) and ``:1399-1426`` (fp16: fp32
    recurrence with fma, result stored as half).  ``K`` counts terms (the reference's
    ``degree``).  fp32 mode evaluates the recurrence exactly in float64.
    """
    xc = np.clip(x_act.astype(np.float64), -1.0, 1.0)
    B, D = xc.shape
    out = np.empty((B, D, K), np.float64)
    if mode == "f16":
        # fp32 recurrence t2 = fma(2x, t1, -t0): the float64 evaluation of a*b+c is exact for
        # fp32 inputs up to the final rounding, which is then done to fp32.
        x32 = xc.astype(np.float32)
        t0 = np.ones_like(x32)
        t1 = x32
        out[..., 0] = 1.0
        if K > 1:
            out[..., 1] = t1
        x2 = (np.float32(2.0) * x32).astype(np.float64)
        for k in range(2, K):
            t2 = (x2 * t1.astype(np.float64) - t0.astype(np.float64)).astype(np.float32)
            out[..., k] = t2
            t0, t1 = t1, t2
        return out.reshape(B, D * K).astype(np.float16).astype(np.float64)
    t0 = np.ones_like(xc)
    t1 = xc
    out[..., 0] = 1.0
    if K > 1:
        out[..., 1] = xc
    for k in range(2, K):
        t2 = 2.0 * xc * t1 - t0
        out[..., k] = t2
        t0, t1 = t1, t2
    return _round_mode(out.reshape(B, D * K), mode)


def rbf_basis(x_act: np.ndarray, grid: np.ndarray, inv_den: float, mode: str) -> np.ndarray:
    """Gaussian RBF exp(-(x - c_k)^2 * inv_den).

    fp32: ``fused_kan.metal:140-166`` (exp2 of -log2e * d^2 * inv_d) -> exact math.
    fp16: ``fused_kan.metal:1428-1450`` -- half arithmetic: diff = x - grid[k] (half),
    -diff*diff (half), * half(inv_den) (half), exp in half (value rounded to half).
    """
    B, D = x_act.shape
    K = grid.shape[0]
    if mode == "f16":
        xh = x_act.astype(np.float16).astype(np.float64)[:, :, None]
        gh = np.asarray(grid).astype(np.float16).astype(np.float64)[None, None, :]
        inv_h = np.float64(np.float16(inv_den))
        diff = _h(xh - gh).astype(np.float64)
        sq = _h(-diff * diff).astype(np.float64)
        t = _h(sq * inv_h).astype(np.float64)
        return _h(np.exp(t)).astype(np.float64).reshape(B, D * K)
    x64 = x_act.astype(np.float64)[:, :, None]
    g64 = np.asarray(grid, dtype=np.float32).astype(np.float64)[None, None, :]
    d = x64 - g64
    inv32 = np.float64(np.float32(inv_den))
    return _round_mode(np.exp(-(d * d) * inv32).reshape(B, D * K), mode)


def bspline_basis(x_act: np.ndarray, grid_size: int, grid_min: float, inv_h: float,
                  mode: str) -> np.ndarray:
    """Closed-form uniform cubic B-spline, ``num_bases = G + 3`` per feature.

    ``fused_kan.metal:240-276`` (fp32) / ``:1476-1512`` (fp16: same fp32 math, half store):
    pos = (x - min) * inv_h (fp32), span = clamp(floor(pos), 0, G-1), u = clamp(pos - span, 0, 1),
    the four cubic weights land on columns span..span+3.  Outside [min, max] the clamp evaluates
    the edge polynomial at u in {0, 1}.
    """
    B, D = x_act.shape
    G = int(grid_size)
    nb = G + 3
    x32 = x_act.astype(np.float32)
    pos = ((x32 - np.float32(grid_min)) * np.float32(inv_h)).astype(np.float32)
    span = np.clip(np.floor(pos), 0, G - 1).astype(np.int64)
    u = np.clip(pos.astype(np.float64) - span, 0.0, 1.0)
    om = 1.0 - u
    b0 = om ** 3 / 6.0
    b1 = (3.0 * u ** 3 - 6.0 * u ** 2 + 4.0) / 6.0
    b2 = (-3.0 * u ** 3 + 3.0 * u ** 2 + 3.0 * u + 1.0) / 6.0
    b3 = u ** 3 / 6.0
    out = np.zeros((B, D, nb), np.float64)
    bi, di = np.meshgrid(np.arange(B), np.arange(D), indexing="ij")
    for j, bj in enumerate((b0, b1, b2, b3)):
        out[bi, di, span + j] = bj
    return _round_mode(out.reshape(B, D * nb), mode)


def wavelet_basis(x_act: np.ndarray, translation: np.ndarray, inv_scale: np.ndarray,
                  wavelet_type: int, mode: str) -> np.ndarray:
    """Continuous wavelets psi((x - t) * inv_s) per (feature, wavelet).

    fp32 (``fused_kan.metal:168-203``): z = (x - t) * inv_s; e = exp(-z^2/2);
    mexican hat (1 - z^2) e, morlet cos(5 z) e, dog -z e.
    fp16 (``fused_kan.metal:1514-1548``): every step in half arithmetic, and the Morlet
    frequency is 1.75 instead of 5 (a quirk of the reference's half kernel, mirrored).
    """
    B, D = x_act.shape
    W = translation.shape[1]
    if mode == "f16":
        xh = x_act.astype(np.float16).astype(np.float64)[:, :, None]
        tr = np.asarray(translation).astype(np.float16).astype(np.float64)[None]
        sc = np.asarray(inv_scale).astype(np.float16).astype(np.float64)[None]
        z = _h(_h(xh - tr).astype(np.float64) * sc).astype(np.float64)
        # exp(-0.5h * z * z): ((-0.5 * z) * z) left to right, then exp, all in half
        a = _h(_h(-0.5 * z).astype(np.float64) * z).astype(np.float64)
        e = _h(np.exp(a)).astype(np.float64)
        if wavelet_type == 0:
            zz = _h(z * z).astype(np.float64)
            psi = _h(_h(1.0 - zz).astype(np.float64) * e)
        elif wavelet_type == 1:
            c = _h(np.cos(_h(1.75 * z).astype(np.float64))).astype(np.float64)
            psi = _h(c * e)
        else:
            psi = _h(_h(-z).astype(np.float64) * e)
        return psi.astype(np.float64).reshape(B, D * W)
    x64 = x_act.astype(np.float64)[:, :, None]
    tr = np.asarray(translation, np.float32).astype(np.float64)[None]
    sc = np.asarray(inv_scale, np.float32).astype(np.float64)[None]
    z = (x64 - tr) * sc
    e = np.exp(-0.5 * z * z)
    if wavelet_type == 0:
        psi = (1.0 - z * z) * e
    elif wavelet_type == 1:
        psi = np.cos(5.0 * z) * e
    else:
        psi = -z * e
    return _round_mode(psi.reshape(B, D * W), mode)


def relu_basis(x_act: np.ndarray, grid: np.ndarray, inv_h: float, mode: str) -> np.ndarray:
    """Tent max(0, 1 - |x - g_k| inv_h) on the raw input (ReLUKAN).

    fp32: ``fused_kan.metal:278-303`` -> |x - g| and the product in fp32 are near-exact; the
    oracle evaluates in float64 with the fp32 grid and fp32 inv_h.
    fp16 (``fused_kan.metal:1452-1474``): half arithmetic -- diff = x - g (half), |diff| * half(inv_h)
    (half), 1 - that (half), max with 0.
    """
    B, D = x_act.shape
    K = np.asarray(grid).shape[0]
    if mode == "f16":
        xh = x_act.astype(np.float16).astype(np.float64)[:, :, None]
        gh = np.asarray(grid).astype(np.float16).astype(np.float64)[None, None, :]
        ih = np.float64(np.float16(inv_h))
        d = np.abs(_h(xh - gh).astype(np.float64))
        t = _h(d * ih).astype(np.float64)
        return np.maximum(0.0, _h(1.0 - t).astype(np.float64)).reshape(B, D * K)
    x64 = x_act.astype(np.float64)[:, :, None]
    g64 = np.asarray(grid, np.float32).astype(np.float64)[None, None, :]
    ih = np.float64(np.float32(inv_h))
    return _round_mode(np.maximum(0.0, 1.0 - np.abs(x64 - g64) * ih).reshape(B, D * K), mode)


def fourier_basis(x_act: np.ndarray, num_freqs: int, mode: str) -> np.ndarray:
    """1, cos(pi x), sin(pi x), ..., cos(F pi x), sin(F pi x) on the raw input (FourierKAN).

    fp32 (``fused_kan.metal:306-329``): angle = fp32(fp32(f * pi) * x), then exact cos/sin.
    fp16 (``fused_kan.metal:1550-1576``): pi_x = half(pi) * x and angle = half(f) * pi_x in half;
    cos/sin of that half angle, stored as half.
    """
    B, D = x_act.shape
    nb = 2 * num_freqs + 1
    out = np.empty((B, D, nb), np.float64)
    out[..., 0] = 1.0
    if mode == "f16":
        xh = x_act.astype(np.float16).astype(np.float64)
        pix = _h(np.float64(np.float16(np.pi)) * xh).astype(np.float64)
        for f in range(1, num_freqs + 1):
            ang = _h(np.float64(f) * pix).astype(np.float64)
            out[..., 2 * f - 1] = _h(np.cos(ang)).astype(np.float64)
            out[..., 2 * f] = _h(np.sin(ang)).astype(np.float64)
        return out.reshape(B, D * nb)
    x32 = x_act.astype(np.float32)
    for f in range(1, num_freqs + 1):
        fr = np.float32(np.float32(f) * np.float32(np.pi))
        ang = (fr * x32).astype(np.float32).astype(np.float64)
        out[..., 2 * f - 1] = np.cos(ang)
        out[..., 2 * f] = np.sin(ang)
    return _round_mode(out.reshape(B, D * nb), mode)


def _jacobi_coeffs(n: int, alpha: float, beta: float):
    """The recurrence coefficients an, bn1, bn2, cn in fp32 arithmetic, in the reference's
    order of operations (``fused_kan.metal:352-356``)."""
    f = np.float32
    fn, a, b = f(n), f(alpha), f(beta)
    ab = f(a + b)
    an = f(f(f(f(2.0) * fn) * f(fn + ab)) * f(f(f(2.0) * fn + ab) - f(2.0)))
    t = f(f(2.0) * fn + ab)
    bn1 = f(f(f(t - f(1.0)) * t) * f(t - f(2.0)))
    bn2 = f(f(t - f(1.0)) * f(f(a * a) - f(b * b)))
    cn = f(f(f(f(2.0) * f(fn + f(a - f(1.0)))) * f(fn + f(b - f(1.0)))) * t)
    return an, bn1, bn2, cn


def jacobi_basis(x_act: np.ndarray, degree: int, alpha: float, beta: float,
                 mode: str) -> np.ndarray:
    """Jacobi P_0..P_{degree-1}^(alpha, beta) of clamp(x, -1, 1) by the three-term recurrence
    ``P_n = ((bn1 x + bn2) P_{n-1} - cn P_{n-2}) / an`` (``fused_kan.metal:331-366``).

    fp32 evaluates the recurrence exactly in float64 with exact coefficients; fp16
    (``:1578-1613``) mirrors the fp32 ``fma(fma(bn1, x, bn2), p1, -cn p0) / an`` recurrence
    (each fma rounded once to fp32) and stores half.
    """
    B, D = x_act.shape
    xc = np.clip(x_act.astype(np.float64), -1.0, 1.0)
    out = np.empty((B, D, degree), np.float64)
    a, b = float(alpha), float(beta)
    if mode == "f16":
        f = np.float32
        x32 = xc.astype(np.float32)
        ab = f(f(a) + f(b))
        p0 = np.ones_like(x32)
        out[..., 0] = 1.0
        if degree > 1:
            p1 = (f(0.5) * (f(f(a) - f(b)) + (ab + f(2.0)) * x32).astype(np.float32)).astype(np.float32)
            out[..., 1] = p1
            for n in range(2, degree):
                an, bn1, bn2, cn = _jacobi_coeffs(n, a, b)
                inner = (np.float64(bn1) * x32.astype(np.float64) + np.float64(bn2)).astype(np.float32)
                m = (-(cn * p0)).astype(np.float32)
                outer = (inner.astype(np.float64) * p1.astype(np.float64) + m.astype(np.float64)).astype(np.float32)
                p = (outer / an).astype(np.float32)
                out[..., n] = p
                p0, p1 = p1, p
        return out.reshape(B, D * degree).astype(np.float16).astype(np.float64)
    ab = a + b
    p0 = np.ones_like(xc)
    out[..., 0] = 1.0
    if degree > 1:
        p1 = 0.5 * (a - b + (ab + 2.0) * xc)
        out[..., 1] = p1
        for n in range(2, degree):
            an = 2.0 * n * (n + ab) * (2.0 * n + ab - 2.0)
            bn1 = (2.0 * n + ab - 1.0) * (2.0 * n + ab) * (2.0 * n + ab - 2.0)
            bn2 = (2.0 * n + ab - 1.0) * (a * a - b * b)
            cn = 2.0 * (n + a - 1.0) * (n + b - 1.0) * (2.0 * n + ab)
            p = ((bn1 * xc + bn2) * p1 - cn * p0) / an
            out[..., n] = p
            p0, p1 = p1, p
    return _round_mode(out.reshape(B, D * degree), mode)


# --------------------------------------------------------------------------------------------
# Projection
# --------------------------------------------------------------------------------------------

def _w64(w, mode):
    """Weights as float64 after rounding to the operand dtype of ``mode``."""
    w = np.asarray(w)
    if mode == "f32":
        return w.astype(np.float32).astype(np.float64)
    return w.astype(np.float32).astype(act_dtype(mode)).astype(np.float64)


def project(phi64: np.ndarray, W, x_base64, W_base, bias, mode: str,
            out_round: bool = True, round_weights: bool = True) -> np.ndarray:
    """Y = bias + silu(x) W_base^T + Phi W^T, accumulated in float64 and rounded once.

    Stand-in for the two MPS GEMMs of ``metal_kan_bridge.mm:489-523`` (accumulation order and
    precision of MPS are not published).  ``round_weights=False`` keeps W and W_base at their
    fp32 values instead of rounding them to the operand dtype (the engine's CUDA-core small-batch
    path multiplies by the exact dequantised INT8/INT4 weight).
    """
    wr = (lambda w: _w64(w, mode)) if round_weights else (
        lambda w: np.asarray(w).astype(np.float32).astype(np.float64))
    y = phi64 @ wr(W).T
    if x_base64 is not None:
        y = y + x_base64 @ wr(W_base).T
    if bias is not None:
        y = y + _w64(bias, mode)[None, :]
    if not out_round:
        return y
    return y.astype(np.float32).astype(act_dtype(mode)) if mode != "f32" else y.astype(np.float32)


def kan_layer(x, basis: str, mode: str, W, W_base=None, bias=None, *, K=None, grid=None,
              inv_den=None, grid_size=None, grid_min=None, inv_h=None, translation=None,
              inv_scale=None, wavelet_type=0, input_map="none", out_round=True,
              round_weights=True, num_freqs=None, alpha=0.0, beta=0.0):
    """One KAN layer forward (reference call stack A of the bridge, any basis).

    ``x`` is rounded to the activation dtype first (the reference casts x to the weight dtype,
    ``cheby_kan.py:97-101``).  The input map (tanh / layernorm) feeds the basis; SiLU of the
    base branch sees the same mapped value.
    """
    xa = to_mode(x, mode) if mode != "f32" else np.asarray(x, np.float32)
    xm = apply_input_map(xa, input_map, mode)
    if basis == "cheby":
        phi = cheby_basis(xm, K, mode)
    elif basis == "rbf":
        phi = rbf_basis(xm, np.asarray(grid), inv_den, mode)
    elif basis == "bspline":
        phi = bspline_basis(xm, grid_size, grid_min, inv_h, mode)
    elif basis == "wavelet":
        phi = wavelet_basis(xm, translation, inv_scale, wavelet_type, mode)
    elif basis == "relu":
        phi = relu_basis(xm, np.asarray(grid), inv_h, mode)
    elif basis == "fourier":
        phi = fourier_basis(xm, num_freqs if num_freqs is not None else (K - 1) // 2, mode)
    elif basis == "jacobi":
        phi = jacobi_basis(xm, K, alpha, beta, mode)
    else:
        raise ValueError(basis)
    xb = silu(xm, mode) if W_base is not None else None
    return project(phi, W, xb, W_base, bias, mode, out_round=out_round,
                   round_weights=round_weights)


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """hidden = g * sigmoid(clamp(g, -20, 20)) * u (``fused_kan.metal:2284-2296``), float64."""
    g = np.asarray(gate, np.float64)
    u = np.asarray(up, np.float64)
    sig = 1.0 / (1.0 + np.exp(-np.clip(g, -20.0, 20.0)))
    return g * sig * u


# --------------------------------------------------------------------------------------------
# Composite layers: MultKAN, LowRankKAN, RationalKAN
# --------------------------------------------------------------------------------------------

def mult_layer(x, mode: str, W_rbf, W_base, bias, *, grid, inv_den, num_add: int,
               num_mult: int):
    """MultKAN (``metal_kan_bridge.mm:1700-1802``): the RBF layer to num_add + 2 num_mult
    internal outputs (rounded to the layer dtype, the MPS output), then the pair products
    ``u v`` of ``combine_mult_nodes`` (``fused_kan.metal:368-389`` / ``:1615-1640``), rounded."""
    internal = kan_layer(x, "rbf", mode, W_rbf, W_base, bias, K=np.asarray(grid).shape[0],
                         grid=grid, inv_den=inv_den)
    if num_mult == 0:
        return internal
    u = internal[:, num_add:num_add + num_mult].astype(np.float64)
    v = internal[:, num_add + num_mult:num_add + 2 * num_mult].astype(np.float64)
    prod = u * v
    prod = (prod.astype(np.float32).astype(act_dtype(mode)) if mode != "f32"
            else prod.astype(np.float32))
    return np.concatenate([internal[:, :num_add], prod], axis=1)


def lowrank_layer(x, mode: str, W_down, W_up, W_base, bias, *, grid, inv_den, out_round=True):
    """LowRankKAN (``metal_kan_bridge.mm:1535-1698``): Z = RBF layer to `rank` outputs, no base
    or bias, rounded to the layer dtype (the MPS output); then
    ``bias + Z W_up^T + silu(x) W_base^T`` in float64, rounded once."""
    z = kan_layer(x, "rbf", mode, W_down, None, None, K=np.asarray(grid).shape[0], grid=grid,
                  inv_den=inv_den)
    xa = to_mode(x, mode) if mode != "f32" else np.asarray(x, np.float32)
    xb = silu(xa, mode) if W_base is not None else None
    return project(np.asarray(z, np.float64), W_up, xb, W_base, bias, mode, out_round=out_round)


def rational_layer(x, W_p, W_q, W_base, bias, *, p_degree: int, q_degree: int):
    """RationalKAN (``kan_rational_tiled``, ``fused_kan.metal:996-1125``), fp32 layer in float64:
    ``y = bias + sum_i silu(xc) W_base[:, i] + P_i / (1 + |Q_i|)``, xc = clamp(x, -1, 1),
    ``P_i = sum_{d<p} T_d(xc) W_p[:, i p + d]``, ``Q_i = sum_{d<q} T_d(xc) W_q[:, i q + d]``."""
    x64 = np.clip(np.asarray(x, np.float32).astype(np.float64), -1.0, 1.0)
    B, D = x64.shape
    md = max(p_degree, q_degree)
    T = cheby_basis(x64, md, "f32").reshape(B, D, md) if md else np.zeros((B, D, 0))
    D_out = np.asarray(W_p if p_degree else W_q).shape[0]
    Wp = np.asarray(W_p, np.float32).astype(np.float64).reshape(D_out, D, p_degree)
    Wq = np.asarray(W_q, np.float32).astype(np.float64).reshape(D_out, D, q_degree)
    P = np.einsum("bik,jik->bji", T[..., :p_degree], Wp)
    Q = np.einsum("bik,jik->bji", T[..., :q_degree], Wq)
    y = (P / (1.0 + np.abs(Q))).sum(-1)
    if W_base is not None:
        y = y + (x64 / (1.0 + np.exp(-x64))) @ np.asarray(W_base, np.float32).astype(np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float32).astype(np.float64)[None, :]
    return y.astype(np.float32)


# --------------------------------------------------------------------------------------------
# Quantisers (reference bridge C++ semantics by default; "numpy" mirrors quantization.py)
# --------------------------------------------------------------------------------------------

def _pad_rows(w: np.ndarray, gs: int) -> np.ndarray:
    """Pad each row with zeros to a multiple of the group size (quantization.py:24-29)."""
    w = np.asarray(w, np.float32)
    pad = (gs - (w.shape[1] % gs)) % gs
    if pad:
        w = np.pad(w, ((0, 0), (0, pad)))
    return np.ascontiguousarray(w, np.float32)


def quantize_affine(w: np.ndarray, bits: int, gs: int, semantics: str = "bridge"):
    """INT8/INT4 block-affine quantiser on a [D_out, K_dim] matrix.

    Returns ``(qweight, scales, biases, padded_in)`` in the reference layout: ``qweight`` is
    [num_groups, gs] (INT8) or [num_groups, gs/2] (INT4, byte = q[2i] | q[2i+1] << 4); scales and
    biases are [num_groups, 1] float32; groups are consecutive ``gs`` elements of the row-padded
    matrix.

    ``semantics="bridge"`` follows ``metal_kan_bridge.mm:4177-4211`` / ``:4234-4275`` evaluated
    with one IEEE fp32 rounding per source operation: s = max(max-min, 1e-7f) / (2^b-1),
    q = (int)((w - min) * (1/s) + 0.5f) clamped.  ``"numpy"`` follows the fallback of
    ``quantization.py:73-97``: q = round_half_even((w - min) / s).
    """
    padded = _pad_rows(w, gs)
    g = padded.reshape(-1, gs)
    mn = g.min(axis=1, keepdims=True)
    mx = g.max(axis=1, keepdims=True)
    rng = np.maximum((mx - mn).astype(np.float32), np.float32(1e-7))
    maxq = (1 << bits) - 1
    s = (rng / np.float32(maxq)).astype(np.float32)
    if semantics == "bridge":
        inv = (np.float32(1.0) / s).astype(np.float32)
        v = (((g - mn).astype(np.float32) * inv).astype(np.float32) + np.float32(0.5)).astype(np.float32)
        q = v.astype(np.int32)
    else:
        q = np.round(((g - mn).astype(np.float32) / s).astype(np.float32)).astype(np.int32)
    q = np.clip(q, 0, maxq)
    if bits == 8:
        qw = q.astype(np.uint8)
    elif bits == 4:
        qw = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    else:
        raise ValueError(bits)
    return qw, s.astype(np.float32), mn.astype(np.float32), padded.shape[1]


def dequantize_affine(qweight: np.ndarray, scales: np.ndarray, biases: np.ndarray, bits: int,
                      gs: int) -> np.ndarray:
    """q * s + b as a separate fp32 multiply and add per element (``metal_kan_bridge.mm:4213``,
    ``:4278``; ``quantization.py:136-146``).  Returns [num_groups, gs] float32."""
    if bits == 8:
        q = qweight.astype(np.float32)
    else:
        q = np.empty((qweight.shape[0], gs), np.float32)
        q[:, 0::2] = qweight & 0x0F
        q[:, 1::2] = (qweight >> 4) & 0x0F
    s = np.asarray(scales, np.float32).reshape(-1, 1)
    b = np.asarray(biases, np.float32).reshape(-1, 1)
    return ((q * s).astype(np.float32) + b).astype(np.float32)


def dequantize_affine_matrix(qweight, scales, biases, bits, gs, shape, padded_in):
    """Dequantise back to the [D_out, K_dim] matrix (padding columns dropped)."""
    full = dequantize_affine(qweight, scales, biases, bits, gs).reshape(-1, padded_in)
    return np.ascontiguousarray(full[: shape[0], : shape[1]])


def _pack2(codes: np.ndarray) -> np.ndarray:
    """Pack 2-bit codes [D_out, K_dim] into uint32 words: element k at bits 2*(k%16) of word k/16."""
    D, Kd = codes.shape
    words = (Kd + 15) // 16
    c = np.zeros((D, words * 16), np.uint32)
    c[:, :Kd] = codes
    c = c.reshape(D, words, 16)
    shifts = (np.arange(16, dtype=np.uint32) * 2)[None, None, :]
    return np.bitwise_or.reduce(c << shifts, axis=2).astype(np.uint32)


def unpack2(packed: np.ndarray, K_dim: int) -> np.ndarray:
    """Inverse of :func:`_pack2`."""
    D, words = packed.shape
    shifts = (np.arange(16, dtype=np.uint32) * 2)[None, None, :]
    c = (packed[:, :, None] >> shifts) & 0x3
    return c.reshape(D, words * 16)[:, :K_dim].astype(np.uint32)


def _group_view(w: np.ndarray, gs: int):
    """Per-row groups with ragged last group: returns (padded [D, G, gs], valid mask, counts)."""
    D, Kd = w.shape
    G = (Kd + gs - 1) // gs
    pad = np.zeros((D, G * gs), np.float32)
    pad[:, :Kd] = w
    mask = np.zeros((G * gs,), bool)
    mask[:Kd] = True
    counts = np.array([min(gs, Kd - gi * gs) for gi in range(G)], np.int64)
    return pad.reshape(D, G, gs), mask.reshape(G, gs), counts


def quantize_ternary(w: np.ndarray, gs: int, semantics: str = "bridge"):
    """Ternary quantiser: codes 0:-1, 1:0, 2:+1 with per-(row, group) scale = mean|w|.

    ``"bridge"``: ``metal_kan_bridge.mm:4634-4682`` -- sum |w| sequentially in double, scale =
    (float)(sum/count) (1e-4f if zero), val = w * (1/scale).  ``"numpy"``:
    ``quantization.py:231-246`` -- float32 ``np.mean``, val = w / scale.
    Returns (w_packed [D_out, ceil(K_dim/16)] uint32, scales [D_out, ceil(K_dim/gs)] float32).
    """
    w = np.ascontiguousarray(w, np.float32)
    D, Kd = w.shape
    gv, mask, counts = _group_view(w, gs)
    if semantics == "bridge":
        a = np.abs(gv.astype(np.float64)) * mask[None]
        ssum = np.add.accumulate(a, axis=2)[:, :, -1]
        sc = np.where(ssum > 0.0, (ssum / counts[None, :]), 1e-4).astype(np.float32)
        sc = np.where(ssum > 0.0, sc, np.float32(1e-4)).astype(np.float32)
        inv = (np.float32(1.0) / sc).astype(np.float32)
        val = (gv * inv[:, :, None]).astype(np.float32)
    else:
        sc = np.empty((D, gv.shape[1]), np.float32)
        for gi in range(gv.shape[1]):
            sl = np.abs(gv[:, gi, : counts[gi]])
            m = np.mean(sl, axis=1)  # float32 pairwise mean, as np.mean(np.abs(slice_w))
            sc[:, gi] = np.where(m > 0, m, np.float32(1e-4))
        val = (gv / sc[:, :, None]).astype(np.float32)
    codes = np.where(val < -0.5, 0, np.where(val > 0.5, 2, 1)).astype(np.uint32)
    codes = codes.reshape(D, -1)[:, :Kd]
    return _pack2(codes), sc.astype(np.float32)


def quantize_int2(w: np.ndarray, gs: int, codebook=None, semantics: str = "bridge"):
    """2-bit codebook quantiser: per-(row, group) scale = max|w|, code = first argmin
    |w/scale - codebook[c]| (``metal_kan_bridge.mm:4735-4788``; numpy fallback
    ``quantization.py:336-352`` divides instead of multiplying by the reciprocal)."""
    if codebook is None:
        codebook = np.array([-1.0, -0.33333, 0.33333, 1.0], np.float32)
    cb = np.asarray(codebook, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    D, Kd = w.shape
    gv, mask, counts = _group_view(w, gs)
    mx = np.max(np.abs(gv) * mask[None], axis=2)
    sc = np.where(mx > 0, mx, np.float32(1e-4)).astype(np.float32)
    if semantics == "bridge":
        inv = (np.float32(1.0) / sc).astype(np.float32)
        val = (gv * inv[:, :, None]).astype(np.float32)
    else:
        val = (gv / sc[:, :, None]).astype(np.float32)
    dist = np.abs(val[..., None] - cb[None, None, None, :]).astype(np.float32)
    codes = np.argmin(dist, axis=-1).astype(np.uint32).reshape(D, -1)[:, :Kd]
    return _pack2(codes), sc.astype(np.float32)


def dequantize_ternary(packed: np.ndarray, scales: np.ndarray, K_dim: int, gs: int) -> np.ndarray:
    """(code - 1) * scale, code 3 -> 0 (``fused_kan.metal:2392-2416``), float32 [D_out, K_dim]."""
    codes = unpack2(packed, K_dim)
    wv = np.where(codes == 3, 0.0, codes.astype(np.float32) - 1.0).astype(np.float32)
    gidx = np.arange(K_dim) // gs
    return (wv * np.asarray(scales, np.float32)[:, gidx]).astype(np.float32)


def dequantize_int2(packed: np.ndarray, scales: np.ndarray, codebook: np.ndarray, K_dim: int,
                    gs: int) -> np.ndarray:
    """codebook[code] * scale (``fused_kan.metal:2418-2441``), float32 [D_out, K_dim]."""
    codes = unpack2(packed, K_dim)
    cb = np.asarray(codebook, np.float32)
    gidx = np.arange(K_dim) // gs
    return (cb[codes] * np.asarray(scales, np.float32)[:, gidx]).astype(np.float32)


# --------------------------------------------------------------------------------------------
# Timed CPU baseline ("the reference's CPU path")
# --------------------------------------------------------------------------------------------

def kan_layer_cpu_f32(x, basis: str, W, W_base=None, bias=None, *, K=None, grid=None,
                      inv_den=None, grid_size=None, grid_min=None, inv_h=None, translation=None,
                      inv_scale=None, wavelet_type=0, input_map="none"):
    """float32 NumPy restatement of the reference's fp32 forward, for timing on host cores.

    The reference has no CPU forward (its only backend is Metal); this is its fp32 pipeline --
    basis kernel (``fused_kan.metal:116-276``) then ``Y = bias + X_silu W_b^T + Phi W^T`` as
    float32 GEMMs standing in for MPS (``metal_kan_bridge.mm:489-523``) -- in float32 NumPy,
    the GEMMs through NumPy's BLAS on all host threads.  Used by bench.py only.
    """
    x = np.asarray(x, np.float32)
    if input_map == "tanh":
        x = np.tanh(x)
    elif input_map == "layernorm":
        mu = x.mean(axis=1, keepdims=True)
        var = ((x - mu) ** 2).mean(axis=1, keepdims=True)
        x = (x - mu) / np.sqrt(var + np.float32(1e-5))
    B, D = x.shape
    if basis == "cheby":
        xc = np.clip(x, -1.0, 1.0)
        phi = np.empty((B, D, K), np.float32)
        phi[..., 0] = 1.0
        if K > 1:
            phi[..., 1] = xc
        for k in range(2, K):
            phi[..., k] = 2.0 * xc * phi[..., k - 1] - phi[..., k - 2]
    elif basis == "rbf":
        d = x[:, :, None] - np.asarray(grid, np.float32)[None, None, :]
        phi = np.exp(-(d * d) * np.float32(inv_den))
    elif basis == "bspline":
        pos = (x - np.float32(grid_min)) * np.float32(inv_h)
        span = np.clip(np.floor(pos), 0, grid_size - 1).astype(np.int64)
        u = np.clip(pos - span, 0.0, 1.0).astype(np.float32)
        om = 1.0 - u
        phi = np.zeros((B, D, grid_size + 3), np.float32)
        bi, di = np.meshgrid(np.arange(B), np.arange(D), indexing="ij")
        for j, bj in enumerate((om ** 3 / 6, (3 * u ** 3 - 6 * u ** 2 + 4) / 6,
                                (-3 * u ** 3 + 3 * u ** 2 + 3 * u + 1) / 6, u ** 3 / 6)):
            phi[bi, di, span + j] = bj
    else:
        z = (x[:, :, None] - translation[None]) * inv_scale[None]
        e = np.exp(-0.5 * z * z)
        phi = ((1 - z * z) * e if wavelet_type == 0 else
               (np.cos(5 * z) * e if wavelet_type == 1 else -z * e)).astype(np.float32)
    y = phi.reshape(B, -1) @ np.asarray(W, np.float32).T
    if W_base is not None:
        y += (x / (1.0 + np.exp(-x))) @ np.asarray(W_base, np.float32).T
    if bias is not None:
        y += np.asarray(bias, np.float32)[None, :]
    return y


# --------------------------------------------------------------------------------------------
# Backward (fp32 training path of the reference)
# --------------------------------------------------------------------------------------------

def _basis_and_grad64(x, basis, K, grid=None, inv_den=None, grid_size=None, grid_min=None,
                      inv_h=None):
    """phi_k(x) and d phi_k / dx in float64, [..., K], with the reference kernels' conventions:
    Chebyshev on clamp(x, -1, 1) with the basis derivative zero outside [-1, 1]
    (fused_kan.metal:1679-1741); Gaussian -2 (x - c) inv_den phi (:1745-1783); cubic B-spline
    pieces differentiated in u and scaled by inv_h on the clamped span/u (:1830-1882)."""
    x = np.asarray(x, np.float64)
    if basis == "cheby":
        xc = np.clip(x, -1.0, 1.0)
        T = np.zeros(x.shape + (K,))
        dT = np.zeros(x.shape + (K,))
        T[..., 0] = 1.0
        if K > 1:
            T[..., 1] = xc
            dT[..., 1] = 1.0
        for k in range(2, K):
            T[..., k] = 2.0 * xc * T[..., k - 1] - T[..., k - 2]
            dT[..., k] = 2.0 * T[..., k - 1] + 2.0 * xc * dT[..., k - 1] - dT[..., k - 2]
        dT[(x < -1.0) | (x > 1.0)] = 0.0
        return T, dT
    if basis == "rbf":
        d = x[..., None] - np.asarray(grid, np.float64)
        phi = np.exp(-(d * d) * float(inv_den))
        return phi, -2.0 * d * float(inv_den) * phi
    if basis == "bspline":
        pos = (x - float(grid_min)) * float(inv_h)
        span = np.clip(np.floor(pos), 0, grid_size - 1).astype(np.int64)
        u = np.clip(pos - span, 0.0, 1.0)
        om = 1.0 - u
        vals = (om ** 3 / 6, (3 * u ** 3 - 6 * u ** 2 + 4) / 6, (-3 * u ** 3 + 3 * u ** 2 + 3 * u + 1) / 6,
                u ** 3 / 6)
        ders = (-0.5 * om ** 2, 1.5 * u ** 2 - 2 * u, -1.5 * u ** 2 + u + 0.5, 0.5 * u ** 2)
        phi = np.zeros(x.shape + (grid_size + 3,))
        dphi = np.zeros_like(phi)
        idx = np.indices(x.shape)
        for j in range(4):
            phi[tuple(idx) + (span + j,)] = vals[j]
            dphi[tuple(idx) + (span + j,)] = ders[j] * float(inv_h)
        return phi, dphi
    if basis == "relu":
        # tent derivative -sign(x - g) inv_h where the tent is positive (fused_kan.metal:1787-1826)
        d = x[..., None] - np.asarray(grid, np.float64)
        v = 1.0 - np.abs(d) * float(inv_h)
        return np.maximum(0.0, v), np.where(v > 0.0, -np.sign(d) * float(inv_h), 0.0)
    raise ValueError(basis)


def kan_layer_backward(x, dY, basis, W, W_base=None, *, K, grid=None, inv_den=None,
                       grid_size=None, grid_min=None, inv_h=None):
    """Gradients of one fp32 layer (raw input) in float64: (dX, dW, dW_base, dbias).

    Restates the reference's backward (metal_kan_bridge.mm:2715-2846 and :2847, :3121): Phi and
    silu(x) re-evaluated, dW = dY^T Phi, dW_base = dY^T silu(x), dbias = sum_b dY,
    dX = sum_k (dY W)[.., i*K + k] phi_k'(x) + (dY W_base) silu'(x) with
    silu'(x) = sigma (1 + x (1 - sigma)) of the raw input."""
    x = np.asarray(x, np.float64)
    dY = np.asarray(dY, np.float64)
    B, D_in = x.shape
    phi, dphi = _basis_and_grad64(x, basis, K, grid, inv_den, grid_size, grid_min, inv_h)
    W = np.asarray(W, np.float64)
    dW = dY.T @ phi.reshape(B, D_in * K)
    dPhi = (dY @ W).reshape(B, D_in, K)
    dX = (dPhi * dphi).sum(-1)
    dWb = None
    if W_base is not None:
        sig = 1.0 / (1.0 + np.exp(-x))
        dWb = dY.T @ (x * sig)
        dX = dX + (dY @ np.asarray(W_base, np.float64)) * (sig * (1.0 + x * (1.0 - sig)))
    return dX, dW, dWb, dY.sum(0)


def swiglu_backward(d_hidden, gate, up):
    """(d_gate, d_up) of hidden = silu(gate) * up, sigma of the clamped gate
    (fused_kan.metal:2298-2316), float64."""
    g = np.asarray(gate, np.float64)
    u = np.asarray(up, np.float64)
    dh = np.asarray(d_hidden, np.float64)
    s = 1.0 / (1.0 + np.exp(-np.clip(g, -20.0, 20.0)))
    return dh * u * (s * (1.0 + g * (1.0 - s))), dh * g * s


# --------------------------------------------------------------------------------------------
# Training: optimiser updates and the fused step (fp32 path of the reference), float64
# --------------------------------------------------------------------------------------------

def optim_update(op: str, p, g, m, v=None, *, lr, beta1=0.9, beta2=0.999, eps=1e-8,
                 weight_decay=0.0, lr_t=None, nesterov=False):
    """One update of the reference's optimiser kernels, returning (p, m, v) in float64:
    ``adamw`` (adamw_step, fused_kan.metal:1896-1921: decoupled decay), ``adam``
    (adam_coupled_step: decay added to the gradient), ``sgd`` (sgd_step :1923-1944: m is the
    velocity, beta1 the momentum), ``lion`` (lion_step :1946-1968)."""
    p = np.asarray(p, np.float64).copy()
    g = np.asarray(g, np.float64).copy()
    m = np.asarray(m, np.float64)
    # the kernels take fp32 hyper-parameters: 1 - beta is then exact in fp32 (Sterbenz) and
    # differs from 1 - beta of the float64 literal by up to ~1e-5 relative (beta2 = 0.999)
    f = lambda a: None if a is None else float(np.float32(a))  # noqa: E731
    lr, beta1, beta2, eps, weight_decay, lr_t = (f(lr), f(beta1), f(beta2), f(eps),
                                                 f(weight_decay), f(lr_t))
    if op in ("adamw", "adam"):
        if op == "adamw" and weight_decay > 0:
            p = p - lr * weight_decay * p
        if op == "adam" and weight_decay > 0:
            g = g + weight_decay * p
        mv = beta1 * m + (1.0 - beta1) * g
        vv = beta2 * np.asarray(v, np.float64) + (1.0 - beta2) * (g * g)
        return p - lr_t * (mv / (np.sqrt(vv) + eps)), mv, vv
    if op == "sgd":
        if weight_decay > 0:
            g = g + weight_decay * p
        vel = beta1 * m + g
        upd = g + beta1 * vel if nesterov else vel
        return p - lr * upd, vel, None
    if op == "lion":
        if weight_decay > 0:
            p = p - lr * weight_decay * p
        u = beta1 * m + (1.0 - beta1) * g
        return p - lr * np.sign(u), beta2 * m + (1.0 - beta2) * g, None
    raise ValueError(op)


def mse_grad(pred, target):
    """dY = (pred - target) * 2 / B (mse_loss_backward, fused_kan.metal:1884-1894)."""
    pred = np.asarray(pred, np.float64)
    return (pred - np.asarray(target, np.float64)) * (2.0 / pred.shape[0])


# --------------------------------------------------------------------------------------------
# Error metric
# --------------------------------------------------------------------------------------------

def max_rel_err(y, y_ref) -> float:
    """max |y - y_ref| / max |y_ref| over the whole output tensor."""
    y = np.asarray(y, np.float64)
    r = np.asarray(y_ref, np.float64)
    den = np.max(np.abs(r))
    if den == 0:
        return float(np.max(np.abs(y)))
    return float(np.max(np.abs(y - r)) / den)


_MANT_BITS = {"f32": 23, "f16": 10, "bf16": 7}


def half_ulp(v, mode: str) -> np.ndarray:
    """Half a unit in the last place of |v| in the output dtype of ``mode`` (normal range)."""
    a = np.abs(np.asarray(v, np.float64))
    e = np.floor(np.log2(np.maximum(a, 1e-30)))
    return 0.5 * np.exp2(e - _MANT_BITS[mode])


def max_rel_err_rounded(y, y_ref64, mode: str) -> float:
    """Error of an output rounded to the dtype of ``mode`` against the UNROUNDED oracle value:
    max over elements of (|y - ref| - half_ulp(ref))_+ / max |ref|.

    The BASELINE tolerance (2e-3 for fp16/bf16 operands with fp32 accumulation, 1e-5 for fp32)
    budgets the computation; the final rounding of the result to its own dtype is allowed on
    top, half an ulp -- which alone can reach 2^-8 relative for bf16 (8 significant bits), so a
    flat 2e-3 on rounded bf16 outputs would be unattainable by any implementation."""
    y = np.asarray(y, np.float64)
    r = np.asarray(y_ref64, np.float64)
    den = np.max(np.abs(r))
    excess = np.maximum(np.abs(y - r) - half_ulp(r, mode), 0.0)
    if den == 0:
        return float(np.max(excess))
    return float(np.max(excess) / den)
