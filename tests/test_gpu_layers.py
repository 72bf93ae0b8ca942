"""GPU parity: the CUDA engine against the oracle and the reference-derived golden fixtures."""
import numpy as np
import pytest

from conftest import group, load_npz
from kan_cases import TOL, layer_err, make_layer, oracle_for_layer, randomize_bias, set_mode
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu

PATHS = {"auto": 0, "simt": 1, "tc": 2}


@pytest.fixture(scope="module")
def mk():
    import metal_kans

    assert metal_kans.is_metal_available()
    return metal_kans


def _layer_from_golden(mk, rec):
    hb, hbi = int(rec["meta_has_base"]), int(rec["meta_has_bias"])
    if "meta_num_mult" in rec:
        l = mk.MultKAN(8, 16, num_mult=int(rec["meta_num_mult"]), num_grids=int(rec["meta_num_grids"]),
                       bias=bool(hbi), use_base=bool(hb))
        l.w_rbf, l.grid = rec["w_rbf"], rec["grid"]
        l.inv_denominator = float(rec["meta_inv_denominator"])
        l.w_base, l.bias = rec["w_base"], rec["bias"]
        return l, "mult"
    if "w_up" in rec:
        l = mk.LowRankKAN(8, 16, rank=int(rec["meta_rank"]), num_grids=int(rec["meta_num_grids"]),
                          bias=bool(hbi), use_base=bool(hb))
        l.w_down, l.grid, l.w_up = rec["w_down"], rec["grid"], rec["w_up"]
        l.inv_denominator = float(rec["meta_inv_denominator"])
        l.w_base, l.bias = rec["w_base"], rec["bias"]
        return l, "lowrank"
    if "w_p" in rec:
        l = mk.RationalKAN(8, 16, p_degree=int(rec["meta_p_degree"]),
                           q_degree=int(rec["meta_q_degree"]), bias=bool(hbi), use_base=bool(hb))
        l.w_p, l.w_q, l.w_base, l.bias = rec["w_p"], rec["w_q"], rec["w_base"], rec["bias"]
        return l, "rational"
    if "w_cheby" in rec:
        l = mk.ChebyKAN(8, 16, degree=int(rec["meta_degree"]), bias=bool(hbi), use_base=bool(hb))
        l.w_cheby = rec["w_cheby"]
        basis = "cheby"
    elif "w_rbf" in rec:
        l = mk.FastKAN(8, 16, num_centers=int(rec["meta_num_centers"]), bias=bool(hbi),
                       use_base=bool(hb))
        l.w_rbf = rec["w_rbf"]
        l.grid = rec["grid"]
        l.inv_denominator = float(rec["meta_inv_denominator"])
        basis = "rbf"
    elif "w_spline" in rec:
        l = mk.BSplineKAN(8, 16, grid_size=int(rec["meta_grid_size"]), bias=bool(hbi),
                          use_base=bool(hb))
        l.w_spline = rec["w_spline"]
        l.grid = rec["grid"]
        basis = "bspline"
    elif "w_relu" in rec:
        l = mk.ReLUKAN(8, 16, num_grids=int(rec["meta_num_grids"]), bias=bool(hbi),
                       use_base=bool(hb))
        l.w_relu = rec["w_relu"]
        l.grid = rec["grid"]
        l.inv_h = float(rec["meta_inv_h"])
        basis = "relu"
    elif "w_fourier" in rec:
        l = mk.FourierKAN(8, 16, num_frequencies=int(rec["meta_num_frequencies"]),
                          bias=bool(hbi), use_base=bool(hb))
        l.w_fourier = rec["w_fourier"]
        basis = "fourier"
    elif "w_jacobi" in rec:
        l = mk.JacobiKAN(8, 16, degree=int(rec["meta_degree"]), alpha=float(rec["meta_alpha"]),
                         beta=float(rec["meta_beta"]), bias=bool(hbi), use_base=bool(hb))
        l.w_jacobi = rec["w_jacobi"]
        basis = "jacobi"
    else:
        l = mk.WavKAN(8, 16, num_wavelets=int(rec["meta_num_wavelets"]), bias=bool(hbi),
                      use_base=bool(hb))
        l.wavelet_type = int(rec["meta_wavelet_type"])
        l.w_wav = rec["w_wav"]
        l.translation = rec["translation"]
        l._inv_scale = rec["inv_scale"]
        basis = "wavelet"
    l.w_base = rec["w_base"]
    l.bias = rec["bias"]
    return l, basis


LAYERS = load_npz("layers_small.npz")
CASES = sorted({k.split("/")[0] for k in LAYERS})


@pytest.mark.parametrize("path", ["auto", "simt", "tc"])
@pytest.mark.parametrize("case", CASES)
def test_reference_layer_goldens(mk, case, path):
    """Golden outputs of the reference's own layer classes (8 -> 16, seed 42)."""
    rec = group(LAYERS, case)
    mode = case.rsplit("_", 1)[1]
    if path == "tc" and mode == "f32":
        pytest.skip("the tensor-core path serves f16/bf16 layers")
    layer, kind = _layer_from_golden(mk, rec)
    if kind in ("mult", "lowrank", "rational"):
        if path != "auto":
            pytest.skip("composite layers choose their kernels themselves")
        y = layer.forward(rec["x"])
    else:
        y = layer.forward(rec["x"], path=PATHS[path])
    assert y.dtype == rec["y"].dtype and y.shape == rec["y"].shape
    err = O.max_rel_err(y, rec["y"])
    assert err <= TOL[mode], f"{case}/{path}: max-rel-err {err:.3e}"


def test_c1_golden_fp32_tanh(mk):
    """BASELINE config 1 (ChebyKAN fp32, B=1024, 64->64, T_0..T_8 of tanh(x)) at full size."""
    z = load_npz("c1_cheby_f32.npz")
    l = mk.ChebyKAN(64, 64, degree=9, bias=False, use_base=False, input_map="tanh")
    l.w_cheby = z["w_cheby"]
    y = l(z["x"])
    assert O.max_rel_err(y, z["y"]) <= 1e-5


SHAPES = [  # (basis, d_in, d_out, K, B)
    ("cheby", 64, 64, 9, 1024),
    ("cheby", 48, 200, 5, 300),
    ("rbf", 256, 256, 8, 512),
    ("rbf", 40, 72, 8, 129),
    ("bspline", 784, 128, 8, 257),
    ("bspline", 24, 10, 8, 64),
    ("wavelet", 64, 96, 6, 200),
    ("wavelet", 32, 40, 8, 1),
    # small grids of 256-wide tiles: the column-split cluster kernel (ragged rows and columns)
    ("wavelet", 64, 320, 6, 200),
    ("cheby", 256, 512, 9, 130),
    ("relu", 64, 96, 8, 300),
    ("relu", 200, 256, 5, 1024),
    ("fourier", 64, 128, 9, 257),
    ("fourier", 30, 50, 5, 64),
    ("jacobi", 96, 128, 4, 300),
    ("jacobi", 64, 256, 6, 1024),
]


@pytest.mark.parametrize("mode", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "-".join(map(str, s)))
@pytest.mark.parametrize("path", ["auto", "simt", "tc"])
def test_random_layers_vs_oracle(mk, shape, mode, path):
    basis, d_in, d_out, K, B = shape
    if path == "tc" and mode == "f32":
        pytest.skip("tensor-core path is f16/bf16")
    layer = set_mode(make_layer(basis, d_in, d_out, K, seed=d_in + K), mode)
    randomize_bias(layer)
    rng = np.random.default_rng(B)
    lo, hi = (-2.5, 2.5) if basis in ("rbf", "relu") else (-1.2, 1.2)
    x = rng.uniform(lo, hi, (B, d_in)).astype(np.float32)
    y = layer.forward(x, path=PATHS[path])
    err = layer_err(y, layer, x, mode, basis)
    assert err <= TOL[mode], f"{shape} {mode} {path}: {err:.3e}"


@pytest.mark.parametrize("mode", ["f16", "bf16"])
@pytest.mark.parametrize("path", ["simt", "tc"])
def test_layernorm_fastkan(mk, mode, path):
    """FastKAN with the (new) input LayerNorm, the BASELINE config-2 layer at reduced B."""
    np.random.seed(0)
    l = mk.FastKAN(256, 256, num_centers=8, grid_range=(-2, 2), input_map="layernorm")
    l.inv_denominator = 3.0625
    rng = np.random.default_rng(1)
    l.w_rbf = rng.normal(0, 0.1, (256, 2048)).astype(np.float32)
    l.w_base = rng.normal(0, 1 / 16, (256, 256)).astype(np.float32)
    set_mode(l, mode)
    x = rng.normal(0, 1, (640, 256)).astype(np.float32)
    y = l.forward(x, path=PATHS[path])
    assert layer_err(y, l, x, mode, "rbf") <= TOL[mode]


@pytest.mark.parametrize("wt", ["mexican_hat", "morlet", "dog"])
@pytest.mark.parametrize("mode", ["f32", "f16", "bf16"])
def test_wavelet_types(mk, wt, mode):
    layer = set_mode(make_layer("wavelet", 16, 24, 6, seed=3, wavelet_type=wt), mode)
    x = np.random.default_rng(2).uniform(-1, 1, (96, 16)).astype(np.float32)
    y = layer(x)
    assert layer_err(y, layer, x, mode, "wavelet") <= TOL[mode]


def test_edge_inputs(mk):
    """Empty batch, 3-D input, exact knots/boundaries, large |x| (clamped bases)."""
    l = make_layer("bspline", 8, 16, 8, seed=5)
    assert l(np.zeros((0, 8), np.float32)).shape == (0, 16)
    x3 = np.random.default_rng(0).uniform(-1, 1, (2, 5, 8)).astype(np.float32)
    assert l(x3).shape == (2, 5, 16)
    knots = np.array([-1.0, -0.6, -0.2, 0.2, 0.6, 1.0, -7.0, 9.0], np.float32)
    x = np.tile(knots, (32, 1))
    assert O.max_rel_err(l(x), oracle_for_layer(l, x, "f32", "bspline")) <= 1e-5
    c = make_layer("cheby", 8, 16, 9, seed=6).half()
    xb = np.array([[-1.0, -0.999, 0.0, 0.999, 1.0, -0.5, 0.5, 30.0]] * 4, np.float16)
    y = c(xb)
    assert np.isfinite(y.astype(np.float32)).all()  # tests/test_optimizations.py:16-26
    assert layer_err(y, c, xb, "f16", "cheby") <= TOL["f16"]


def test_bad_arguments_raise(mk):
    import ctypes

    lib = mk.get_metal_bridge()
    with pytest.raises(mk.KanError):
        lib.metal_kan_cheby_forward(None, None, None, None, None, 4, 8, 8, 4, 0, 0)
    l = make_layer("cheby", 8, 16, 4)
    with pytest.raises(ValueError):
        l(np.zeros((3, 7), np.float32))
    L = mk.device.KanLayer()
    with pytest.raises(mk.KanError):
        lib.kan_forward(ctypes.byref(L), None, None, 1, None)


def test_descriptor_cache_follows_parameter_changes(mk):
    """The cached kernel descriptor is rebuilt when a weight, a basis parameter or the dtype
    changes between calls."""
    np.random.seed(5)
    l = mk.FastKAN(64, 96, num_centers=8, grid_range=(-2, 2)).half()
    x = np.random.default_rng(5).uniform(-2, 2, (200, 64)).astype(np.float32)
    y0 = l(x)
    assert layer_err(y0, l, x, "f16", "rbf") <= TOL["f16"]
    l.inv_denominator = 0.5 * float(l.inv_denominator)
    y1 = l(x)
    assert not np.array_equal(y0, y1)
    assert layer_err(y1, l, x, "f16", "rbf") <= TOL["f16"]
    l.w_rbf = (np.asarray(l.w_rbf, np.float32) * 2).astype(np.float16)
    y2 = l(x)
    assert layer_err(y2, l, x, "f16", "rbf") <= TOL["f16"]
    l.float()
    y3 = l(x)
    assert y3.dtype == np.float32 and layer_err(y3, l, x, "f32", "rbf") <= TOL["f32"]


@pytest.mark.parametrize("case", [("rbf", 256, 256, 8, 3000, "f16"), ("cheby", 256, 512, 9, 2500, "bf16"),
                                  ("cheby", 64, 64, 9, 4100, "f32")],
                         ids=lambda c: "-".join(map(str, c)))
def test_host_forward_chunked(mk, case):
    """layer(x) runs kan_forward_host: batches this large go as two chunks whose copies overlap the
    kernels; the result must match the oracle and the one-shot device path."""
    basis, d_in, d_out, K, B, mode = case
    layer = set_mode(make_layer(basis, d_in, d_out, K, seed=7), mode)
    randomize_bias(layer)
    lo, hi = (-2.5, 2.5) if basis in ("rbf", "relu") else (-1.2, 1.2)
    x = np.random.default_rng(B).uniform(lo, hi, (B, d_in)).astype(np.float32)
    y = layer(x)
    assert y.shape == (B, d_out)
    assert layer_err(y, layer, x, mode, basis) <= TOL[mode]
    y1 = layer.forward(x, path=PATHS["simt"])
    assert layer_err(y1, layer, x, mode, basis) <= TOL[mode]


@pytest.mark.parametrize("case", [("cheby", 64, 1024, 9, 7680, "bf16"), ("rbf", 128, 640, 8, 7700, "f16"),
                                  ("cheby", 96, 520, 5, 15400, "f16"),
                                  ("cheby", 400, 512, 9, 8000, "bf16"), ("rbf", 448, 520, 8, 7500, "f16"),
                                  ("cheby", 64, 517, 9, 15400, "bf16")],
                         ids=lambda c: "-".join(map(str, c)))
def test_wide_tiles(mk, case):
    """Grids of >= 120 tiles of 512 outputs run the wide tensor-core variant (two N = 256
    accumulators per basis block); grids of 60-119 such tiles run it with K split in two (the
    cluster reduction in two column rounds).  Ragged rows and ragged output tiles included."""
    basis, d_in, d_out, K, B, mode = case
    layer = set_mode(make_layer(basis, d_in, d_out, K, seed=5), mode)
    randomize_bias(layer)
    lo, hi = (-2.5, 2.5) if basis in ("rbf", "relu") else (-1.2, 1.2)
    x = np.random.default_rng(B).uniform(lo, hi, (B, d_in)).astype(np.float32)
    y = layer.forward(x, path=PATHS["tc"])
    assert layer_err(y, layer, x, mode, basis) <= TOL[mode]
