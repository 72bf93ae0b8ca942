"""CPU: the oracle against the golden fixtures made from the reference's own Python code."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from conftest import REPO, group, load_npz
from oracle import kan_oracle as O

LAYERS = load_npz("layers_small.npz")
QUANT = load_npz("quant_reference_numpy.npz")
BLOCKS = load_npz("blocks_small.npz")


def _cases():
    return sorted({k.split("/")[0] for k in LAYERS})


def oracle_layer_from_golden(rec, mode):
    """Call the oracle with the parameters a reference layer golden recorded."""
    hb = int(rec["meta_has_base"])
    hbi = int(rec["meta_has_bias"])
    kw = {}
    wb = rec["w_base"] if hb else None
    b = rec["bias"] if hbi else None
    if "meta_num_mult" in rec:
        return O.mult_layer(rec["x"], mode, rec["w_rbf"], wb, b, grid=rec["grid"],
                            inv_den=float(rec["meta_inv_denominator"]),
                            num_add=int(rec["meta_num_add"]), num_mult=int(rec["meta_num_mult"]))
    if "w_up" in rec:
        return O.lowrank_layer(rec["x"], mode, rec["w_down"], rec["w_up"], wb, b, grid=rec["grid"],
                               inv_den=float(rec["meta_inv_denominator"]))
    if "w_p" in rec:
        return O.rational_layer(rec["x"], rec["w_p"], rec["w_q"], wb, b,
                                p_degree=int(rec["meta_p_degree"]),
                                q_degree=int(rec["meta_q_degree"]))
    if "w_cheby" in rec:
        basis, W, K = "cheby", rec["w_cheby"], int(rec["meta_degree"])
    elif "w_rbf" in rec:
        basis, W, K = "rbf", rec["w_rbf"], int(rec["meta_num_centers"])
        kw = dict(grid=rec["grid"], inv_den=float(rec["meta_inv_denominator"]))
    elif "w_spline" in rec:
        G = int(rec["meta_grid_size"])
        basis, W, K = "bspline", rec["w_spline"], G + 3
        kw = dict(grid_size=G, grid_min=float(rec["grid"][0]), inv_h=float(rec["grid"][1]))
    elif "w_relu" in rec:
        basis, W, K = "relu", rec["w_relu"], int(rec["meta_num_grids"])
        kw = dict(grid=rec["grid"], inv_h=float(rec["meta_inv_h"]))
    elif "w_fourier" in rec:
        F = int(rec["meta_num_frequencies"])
        basis, W, K = "fourier", rec["w_fourier"], 2 * F + 1
        kw = dict(num_freqs=F)
    elif "w_jacobi" in rec:
        basis, W, K = "jacobi", rec["w_jacobi"], int(rec["meta_degree"])
        kw = dict(alpha=float(rec["meta_alpha"]), beta=float(rec["meta_beta"]))
    else:
        basis, W, K = "wavelet", rec["w_wav"], int(rec["meta_num_wavelets"])
        kw = dict(translation=rec["translation"], inv_scale=rec["inv_scale"],
                  wavelet_type=int(rec["meta_wavelet_type"]))
    return O.kan_layer(rec["x"], basis, mode, W, rec["w_base"] if hb else None,
                       rec["bias"] if hbi else None, K=K, **kw)


@pytest.mark.parametrize("case", _cases())
def test_layer_goldens_reproduce(case):
    rec = group(LAYERS, case)
    mode = case.rsplit("_", 1)[1]
    y = oracle_layer_from_golden(rec, mode)
    assert y.dtype == rec["y"].dtype
    np.testing.assert_array_equal(y, rec["y"])


def test_fp16_vs_fp32_reference_tolerance():
    """The reference's own pin: fp16 forward within atol 1e-2 of fp32 (test_metal_kans.py:257)."""
    for case in _cases():
        # Morlet is excluded: the reference's half kernel uses cos(1.75 z), its fp32 kernel
        # cos(5 z) (fused_kan.metal:1541 vs :184), and its own fp16 test only covers Mexican hat.
        # Fourier and Jacobi are outside that test too (it covers Chebyshev, RBF and ReLU): half
        # angles (half(pi) x, rounded) and Jacobi values above 1 (alpha, beta > 0) put their
        # fp16 outputs up to ~1.6e-2 from fp32 on these cases.
        if (not case.endswith("_f32") or "morlet" in case
                or case.startswith(("fourier", "jacobi", "rational"))):
            continue
        r32 = group(LAYERS, case)
        r16 = group(LAYERS, case[:-4] + "_f16")
        np.testing.assert_allclose(r16["y"].astype(np.float32), r32["y"], atol=1e-2)


def test_c1_golden():
    z = load_npz("c1_cheby_f32.npz")
    y = O.kan_layer(z["x"], "cheby", "f32", z["w_cheby"], K=9, input_map="tanh")
    assert O.max_rel_err(y, z["y"]) < 1e-6


def _c_oracle():
    so = os.path.join(REPO, "oracle", "_build", "libquant_oracle.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", os.path.join(REPO, "oracle")], check=True,
                       capture_output=True)
    return ctypes.CDLL(so)


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


@pytest.mark.parametrize("bits", [8, 4])
def test_affine_numpy_semantics_bit_exact(bits):
    for tag in ("n01_32x64_g32", "ragged_12x100_g64", "const_4x64_g64"):
        r = group(QUANT, f"aff{bits}_{tag}")
        gs = int(r["gs"])
        qw, s, b, pin = O.quantize_affine(r["w"], bits, gs, semantics="numpy")
        np.testing.assert_array_equal(qw, r["qweight"])
        np.testing.assert_array_equal(s, r["scales"])
        np.testing.assert_array_equal(b, r["biases"])
        deq = O.dequantize_affine_matrix(r["qweight"], r["scales"], r["biases"], bits, gs,
                                         r["w"].shape, pin)
        np.testing.assert_array_equal(deq, r["deq"])


@pytest.mark.parametrize("bits", [8, 4])
def test_affine_bridge_semantics_vs_c_oracle(bits):
    lib = _c_oracle()
    rng = np.random.default_rng(bits)
    for shape, gs in (((64, 576), 64), ((33, 100), 32), ((5, 128), 128)):
        w = rng.normal(0, 0.02, shape).astype(np.float32)
        qw, s, b, pin = O.quantize_affine(w, bits, gs, "bridge")
        padded = O._pad_rows(w, gs)
        G = padded.size // gs
        cq = np.empty_like(qw)
        cs = np.empty((G,), np.float32)
        cb = np.empty((G,), np.float32)
        assert lib.oracle_quantize_affine(_p(padded), _p(cq), _p(cs), _p(cb), G, gs, bits) == 0
        np.testing.assert_array_equal(cq, qw)
        np.testing.assert_array_equal(cs, s.ravel())
        np.testing.assert_array_equal(cb, b.ravel())
        out = np.empty((G, gs), np.float32)
        assert lib.oracle_dequantize_affine(_p(cq), _p(cs), _p(cb), _p(out), G, gs, bits) == 0
        np.testing.assert_array_equal(out, O.dequantize_affine(qw, s, b, bits, gs))
        # bridge vs numpy rounding differ only where (w-min)/s sits on a rounding boundary
        qn, _, _, _ = O.quantize_affine(w, bits, gs, "numpy")
        assert np.mean(qn != qw) < 1e-3


def test_ternary_int2_numpy_semantics_bit_exact():
    for tag in ("n_8x72_g32", "n_6x100_g64", "zeros_2x40_g16"):
        r = group(QUANT, f"tern_{tag}")
        gs = int(r["gs"])
        p, s = O.quantize_ternary(r["w"], gs, "numpy")
        np.testing.assert_array_equal(p, r["packed"])
        np.testing.assert_array_equal(s, r["scales"])
        np.testing.assert_array_equal(O.dequantize_ternary(r["packed"], r["scales"],
                                                           r["w"].shape[1], gs), r["deq"])
        r = group(QUANT, f"int2_{tag}")
        p, s = O.quantize_int2(r["w"], gs, r["codebook"], "numpy")
        np.testing.assert_array_equal(p, r["packed"])
        np.testing.assert_array_equal(s, r["scales"])
        np.testing.assert_array_equal(O.dequantize_int2(r["packed"], r["scales"], r["codebook"],
                                                        r["w"].shape[1], gs), r["deq"])


def test_ternary_int2_bridge_semantics_vs_c_oracle():
    lib = _c_oracle()
    rng = np.random.default_rng(3)
    cbk = np.array([-1.0, -0.33333, 0.33333, 1.0], np.float32)
    for shape, gs in (((16, 576), 64), ((7, 100), 32), ((3, 37), 16)):
        w = rng.normal(0, 0.03, shape).astype(np.float32)
        D, Kd = shape
        words, G = (Kd + 15) // 16, (Kd + gs - 1) // gs
        p, s = O.quantize_ternary(w, gs, "bridge")
        cp = np.empty((D, words), np.uint32)
        cs = np.empty((D, G), np.float32)
        assert lib.oracle_quantize_ternary(_p(w), _p(cp), _p(cs), D, Kd, gs) == 0
        np.testing.assert_array_equal(cp, p)
        np.testing.assert_array_equal(cs, s)
        out = np.empty((D, Kd), np.float32)
        assert lib.oracle_dequantize_2bit(_p(cp), _p(cs), None, _p(out), D, Kd, gs) == 0
        np.testing.assert_array_equal(out, O.dequantize_ternary(p, s, Kd, gs))
        p, s = O.quantize_int2(w, gs, cbk, "bridge")
        assert lib.oracle_quantize_int2(_p(w), _p(cp), _p(cs), _p(cbk), D, Kd, gs) == 0
        np.testing.assert_array_equal(cp, p)
        np.testing.assert_array_equal(cs, s)
        assert lib.oracle_dequantize_2bit(_p(cp), _p(cs), _p(cbk), _p(out), D, Kd, gs) == 0
        np.testing.assert_array_equal(out, O.dequantize_int2(p, s, cbk, Kd, gs))


def test_pack_roundtrip():
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 4, (5, 53)).astype(np.uint32)
    np.testing.assert_array_equal(O.unpack2(O._pack2(codes), 53), codes)


def test_blocks_gated_int4_dequant_matches_reference():
    """to_int4 in the reference stores dequantised weights; the oracle reproduces them."""
    for nm in ("gate_kan", "up_kan", "down_kan"):
        for attr in ("w_cheby", "w_base"):
            pre = f"gated_int4/{nm}.{attr}"
            deq = BLOCKS[pre + ".deq"]
            pin = BLOCKS[pre + ".qweight"].shape[0] * 64 // deq.shape[0]
            got = O.dequantize_affine_matrix(BLOCKS[pre + ".qweight"], BLOCKS[pre + ".scales"],
                                             BLOCKS[pre + ".biases"], 4, 64, deq.shape, pin)
            np.testing.assert_array_equal(got, deq)


@pytest.mark.parametrize("basis,K", [("cheby", 6), ("rbf", 8), ("bspline", 8), ("relu", 6)])
def test_backward_oracle_matches_finite_differences(basis, K):
    """The backward restatement is the derivative of the forward restatement: central finite
    differences of the float64 forward (f32 mode evaluates the basis exactly) agree with dX, dW,
    dW_base and dbias.  Inputs stay away from the Chebyshev clamp and the B-spline knots, where
    the reference's derivative conventions (zero / one-sided) apply."""
    rng = np.random.default_rng(11)
    B, D_in, D_out = 5, 4, 3
    if basis == "bspline":
        x = (rng.integers(0, 5, (B, D_in)) + rng.uniform(0.2, 0.8, (B, D_in))) * 0.4 - 1.0
        kw = dict(grid_size=5, grid_min=-1.0, inv_h=2.5)
    elif basis == "relu":  # between the tent knots (grid spacing 0.4)
        x = (rng.integers(0, 5, (B, D_in)) + rng.uniform(0.2, 0.8, (B, D_in))) * 0.4 - 1.0
        kw = dict(grid=np.linspace(-1, 1, K), inv_h=2.5)
    else:
        x = rng.uniform(-0.9, 0.9, (B, D_in))
        kw = dict(grid=np.linspace(-2, 2, K), inv_den=1.5) if basis == "rbf" else {}
    W = rng.normal(0, 0.3, (D_out, D_in * K))
    Wb = rng.normal(0, 0.3, (D_out, D_in))
    bias = rng.normal(0, 0.1, D_out)
    dY = rng.normal(0, 1, (B, D_out))

    def loss(x_, W_, Wb_, b_):
        y = O.kan_layer(x_, basis, "f32", W_, Wb_, b_, K=K, out_round=False,
                        round_weights=False, **kw)
        return float((np.asarray(y, np.float64) * dY).sum())

    # the f32 mode rounds x to float32: finite differences are taken in float64 on the
    # restatement evaluated through the same exact-basis path
    def loss64(x_, W_, Wb_, b_):
        phi, _ = O._basis_and_grad64(x_, basis, K, **kw)
        s = 1.0 / (1.0 + np.exp(-x_))
        y = phi.reshape(B, -1) @ W_.T + (x_ * s) @ Wb_.T + b_
        return float((y * dY).sum())

    dX, dW, dWb, db = O.kan_layer_backward(x, dY, basis, W, Wb, K=K, **kw)
    h = 1e-6
    num = np.zeros_like(x)
    for idx in np.ndindex(*x.shape):
        e = np.zeros_like(x)
        e[idx] = h
        num[idx] = (loss64(x + e, W, Wb, bias) - loss64(x - e, W, Wb, bias)) / (2 * h)
    np.testing.assert_allclose(dX, num, rtol=1e-6, atol=1e-8)
    for arr, grad, args in ((W, dW, 1), (Wb, dWb, 2), (bias, db, 3)):
        num = np.zeros_like(arr)
        for idx in np.ndindex(*arr.shape):
            e = np.zeros_like(arr)
            e[idx] = h
            p = [x, W, Wb, bias]
            m = [x, W, Wb, bias]
            p[args] = arr + e
            m[args] = arr - e
            num[idx] = (loss64(*p) - loss64(*m)) / (2 * h)
        np.testing.assert_allclose(grad, num, rtol=1e-6, atol=1e-8)
    # and the float64 restatement of the forward is the f32-mode oracle up to its input rounding
    assert abs(loss(x, W, Wb, bias) - loss64(x.astype(np.float32).astype(np.float64), W, Wb,
                                             bias)) < 1e-6
