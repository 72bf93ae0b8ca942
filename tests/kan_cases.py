"""Helpers shared by the GPU tests: build engine layers and oracle calls from the same inputs."""
import numpy as np

from oracle import kan_oracle as O

TOL = {"f32": 1e-5, "f16": 2e-3, "bf16": 2e-3}  # max|y - y_ref| / max|y_ref| (BASELINE tolerance)


def np_dtype(mode):
    return O.act_dtype(mode)


def set_mode(layer, mode):
    if mode == "f16":
        layer.half()
    elif mode == "bf16":
        layer.bfloat16()
    return layer


def oracle_for_layer(layer, x, mode, basis, out_round=True, exact_weights=False):
    """Oracle output for an engine layer object (reads its current weights).  exact_weights:
    the packed weights' exact fp32 dequantised values, not rounded to the operand dtype."""
    import metal_kans as mk  # noqa: F401

    W = np.asarray(getattr(layer, layer.MAIN)).astype(np.float32)
    wb = np.asarray(layer.w_base).astype(np.float32) if layer.has_base else None
    if exact_weights:
        W = layer._packed(layer.MAIN).dequantize()
        wb = layer._packed("w_base").dequantize() if layer.has_base else None
    b = np.asarray(layer.bias).astype(np.float32) if layer.has_bias else None
    kw = {}
    if basis == "rbf":
        kw = dict(grid=np.asarray(layer.grid).astype(np.float32), inv_den=layer.inv_denominator)
    elif basis == "bspline":
        kw = dict(grid_size=layer.grid_size, grid_min=float(layer.grid[0]), inv_h=float(layer.grid[1]))
    elif basis == "wavelet":
        kw = dict(translation=np.asarray(layer.translation).astype(np.float32),
                  inv_scale=np.asarray(layer._inv_scale).astype(np.float32),
                  wavelet_type=layer.wavelet_type)
    elif basis == "relu":
        kw = dict(grid=np.asarray(layer.grid), inv_h=layer.inv_h)
    elif basis == "fourier":
        kw = dict(num_freqs=layer.num_frequencies)
    elif basis == "jacobi":
        kw = dict(alpha=layer.alpha, beta=layer.beta)
    return O.kan_layer(x, basis, mode, W, wb, b, K=layer._terms(),
                       input_map=getattr(layer, "input_map", "none"), out_round=out_round,
                       round_weights=not exact_weights, **kw)


def layer_err(y, layer, x, mode, basis, exact_weights=False):
    """Engine output vs the unrounded oracle, final output rounding allowed (half an ulp)."""
    ref = oracle_for_layer(layer, x, mode, basis, out_round=False, exact_weights=exact_weights)
    return O.max_rel_err_rounded(np.asarray(y).astype(np.float64), ref, mode)


def make_layer(basis, d_in, d_out, K, *, bias=True, use_base=True, input_map="none", seed=0,
               wavelet_type="mexican_hat"):
    import metal_kans as mk

    np.random.seed(seed)
    if basis == "cheby":
        return mk.ChebyKAN(d_in, d_out, degree=K, bias=bias, use_base=use_base, input_map=input_map)
    if basis == "rbf":
        return mk.FastKAN(d_in, d_out, num_centers=K, bias=bias, use_base=use_base,
                          grid_range=(-2.0, 2.0), input_map=input_map)
    if basis == "bspline":
        return mk.BSplineKAN(d_in, d_out, grid_size=K - 3, bias=bias, use_base=use_base,
                             input_map=input_map)
    if basis == "relu":
        return mk.ReLUKAN(d_in, d_out, num_grids=K, bias=bias, use_base=use_base,
                          grid_range=(-2.0, 2.0))
    if basis == "fourier":
        return mk.FourierKAN(d_in, d_out, num_frequencies=(K - 1) // 2, bias=bias,
                             use_base=use_base)
    if basis == "jacobi":
        # alpha, beta > 0: values above 1 (the recurrence's general coefficients)
        return mk.JacobiKAN(d_in, d_out, degree=K, alpha=0.5, beta=0.25, bias=bias,
                            use_base=use_base)
    return mk.WavKAN(d_in, d_out, num_wavelets=K, bias=bias, use_base=use_base,
                     wavelet_type=wavelet_type, input_map=input_map)


def randomize_bias(layer, seed=1):
    if layer.has_bias:
        rng = np.random.default_rng(seed)
        layer.bias = rng.normal(0, 0.1, layer.bias.shape).astype(layer.bias.dtype)
