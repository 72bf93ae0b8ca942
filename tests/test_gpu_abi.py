"""GPU: the reference-compatible host-pointer C ABI, blocks and nets, torch interop, async mode."""
import ctypes

import numpy as np
import pytest

from conftest import group, load_npz
from kan_cases import TOL, layer_err, make_layer, oracle_for_layer
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu
BLOCKS = load_npz("blocks_small.npz")


@pytest.fixture(scope="module")
def mk():
    import metal_kans

    return metal_kans


def P(a):
    return a.ctypes.data


def test_host_abi_all_forwards(mk):
    """Every metal_kan_*_forward{,_fp16} entry point against the oracle (host pointers)."""
    lib = mk.get_metal_bridge()
    rng = np.random.default_rng(0)
    B, Di, Do = 70, 24, 40
    for dt, mode in ((np.float32, "f32"), (np.float16, "f16")):
        sfx = "" if mode == "f32" else "_fp16"
        x = rng.uniform(-1, 1, (B, Di)).astype(dt)
        wb = rng.normal(0, 0.2, (Do, Di)).astype(dt)
        b = rng.normal(0, 0.1, (Do,)).astype(dt)
        y = np.empty((B, Do), dt)
        # cheby
        W = rng.normal(0, 0.1, (Do, Di * 6)).astype(dt)
        getattr(lib, "metal_kan_cheby_forward" + sfx)(P(x), P(W), P(wb), P(b), P(y), B, Di, Do, 6, 1, 1)
        ref = O.kan_layer(x, "cheby", mode, W, wb, b, K=6)
        assert O.max_rel_err(y, ref) <= TOL[mode]
        # fastkan
        W = rng.normal(0, 0.1, (Do, Di * 8)).astype(dt)
        grid = np.linspace(-1, 1, 8).astype(dt)
        getattr(lib, "metal_kan_fastkan_forward" + sfx)(P(x), P(W), P(wb), P(grid), P(b), P(y), B, Di, Do, 8, 24.5, 1, 1)
        ref = O.kan_layer(x, "rbf", mode, W, wb, b, K=8, grid=grid, inv_den=24.5)
        assert O.max_rel_err(y, ref) <= TOL[mode]
        # bspline (grid = [min, inv_h] fp32)
        W = rng.normal(0, 0.1, (Do, Di * 8)).astype(dt)
        gp = np.array([-1.0, 2.5], np.float32)
        getattr(lib, "metal_kan_bspline_forward" + sfx)(P(x), P(W), P(wb), P(gp), P(b), P(y), B, Di, Do, 5, 3, 1, 1)
        ref = O.kan_layer(x, "bspline", mode, W, wb, b, K=8, grid_size=5, grid_min=-1.0, inv_h=2.5)
        assert O.max_rel_err(y, ref) <= TOL[mode]
        # wavkan
        W = rng.normal(0, 0.1, (Do, Di * 5)).astype(dt)
        tr = rng.uniform(-1, 1, (Di, 5)).astype(dt)
        isc = rng.uniform(0.5, 2, (Di, 5)).astype(dt)
        for wt in (0, 1, 2):
            getattr(lib, "metal_kan_wavkan_forward" + sfx)(P(x), P(W), P(wb), P(tr), P(isc), P(b), P(y), B, Di, Do, 5, wt, 1, 1)
            ref = O.kan_layer(x, "wavelet", mode, W, wb, b, K=5, translation=tr, inv_scale=isc,
                              wavelet_type=wt)
            assert O.max_rel_err(y, ref) <= TOL[mode]
        # relu (grid in the layer dtype, inv_h fp32)
        W = rng.normal(0, 0.1, (Do, Di * 7)).astype(dt)
        grid = np.linspace(-1, 1, 7).astype(dt)
        getattr(lib, "metal_kan_relu_forward" + sfx)(P(x), P(W), P(wb), P(grid), P(b), P(y), B, Di, Do, 7, 3.0, 1, 1)
        ref = O.kan_layer(x, "relu", mode, W, wb, b, K=7, grid=grid, inv_h=3.0)
        assert O.max_rel_err(y, ref) <= TOL[mode]
        # fourier (3 frequencies: 7 bases)
        getattr(lib, "metal_kan_fourier_forward" + sfx)(P(x), P(W), P(wb), P(b), P(y), B, Di, Do, 3, 1, 1)
        ref = O.kan_layer(x, "fourier", mode, W, wb, b, K=7, num_freqs=3)
        assert O.max_rel_err(y, ref) <= TOL[mode]
        # jacobi
        W = rng.normal(0, 0.1, (Do, Di * 5)).astype(dt)
        getattr(lib, "metal_kan_jacobi_forward" + sfx)(P(x), P(W), P(wb), P(b), P(y), B, Di, Do, 5, 1.0, 0.5, 1, 1)
        ref = O.kan_layer(x, "jacobi", mode, W, wb, b, K=5, alpha=1.0, beta=0.5)
        assert O.max_rel_err(y, ref) <= TOL[mode]


def test_host_abi_packed_cheby(mk):
    """metal_kan_forward_ternary_cheby / _int2_cheby (fused_kan.metal:2167-2280 semantics:
    clamp, Chebyshev terms, decoded weights, no base branch)."""
    lib = mk.get_metal_bridge()
    rng = np.random.default_rng(1)
    B, Di, Do, deg, gs = 33, 16, 24, 5, 32
    x = rng.uniform(-1.3, 1.3, (B, Di)).astype(np.float32)
    w = rng.normal(0, 0.05, (Do, Di * deg)).astype(np.float32)
    bias = rng.normal(0, 0.1, Do).astype(np.float32)
    y = np.empty((B, Do), np.float32)
    p, s = O.quantize_ternary(w, gs)
    lib.metal_kan_forward_ternary_cheby(P(x), P(p), P(s), P(bias), P(y), B, Di, Do, deg, gs, 1)
    ref = O.kan_layer(x, "cheby", "f32", O.dequantize_ternary(p, s, Di * deg, gs), None, bias, K=deg)
    assert O.max_rel_err(y, ref) <= 1e-5
    cb = np.array([-1.0, -0.33333, 0.33333, 1.0], np.float32)
    p, s = O.quantize_int2(w, gs, cb)
    lib.metal_kan_forward_int2_cheby(P(x), P(p), P(s), P(cb), P(bias), P(y), B, Di, Do, deg, gs, 1)
    ref = O.kan_layer(x, "cheby", "f32", O.dequantize_int2(p, s, cb, Di * deg, gs), None, bias, K=deg)
    assert O.max_rel_err(y, ref) <= 1e-5


def test_swiglu_and_benchmark_entry_points(mk):
    lib = mk.get_metal_bridge()
    rng = np.random.default_rng(2)
    g = rng.normal(0, 8, 10007).astype(np.float32)
    u = rng.normal(0, 1, 10007).astype(np.float32)
    out = np.empty_like(g)
    lib.metal_kan_swiglu_forward(P(g), P(u), P(out), g.size)
    np.testing.assert_allclose(out, O.swiglu(g, u), rtol=2e-6, atol=1e-6)
    l = make_layer("cheby", 64, 64, 4)
    x = rng.uniform(-1, 1, (1024, 64)).astype(np.float32)
    ms = l.benchmark(x, warmup=2, iters=5)
    assert 0 < ms < 1000


K_OF = {"cheby": 5, "rbf": 8, "bspline": 8, "wavelet": 6, "relu": 8, "fourier": 9, "jacobi": 5}


@pytest.mark.parametrize("basis", ["cheby", "rbf", "bspline", "wavelet", "relu", "fourier",
                                   "jacobi"])
def test_benchmark_entry_points_all_bases(mk, basis):
    """benchmark_metal_{cheby,fastkan,bspline,wavkan,relu,fourier,jacobi} (metal_kan_bridge.mm:1250-1371): a positive
    mean of milliseconds per host-pointer forward, and the Y each leaves behind is the layer's
    forward (fp32 path, 1e-5 against the oracle)."""
    lib = mk.get_metal_bridge()
    l = make_layer(basis, 48, 40, K_OF[basis], seed=6)
    rng = np.random.default_rng(6)
    l.bias = rng.normal(0, 0.1, 40).astype(np.float32)
    x = rng.uniform(-1, 1, (300, 48)).astype(np.float32)
    assert 0 < l.benchmark(x, warmup=1, iters=3) < 1000
    y = np.empty((300, 40), np.float32)
    W = getattr(l, l.MAIN)
    if basis == "cheby":
        ms = lib.benchmark_metal_cheby(P(x), P(W), P(l.w_base), P(l.bias), P(y), 300, 48, 40,
                                       l._terms(), 1, 1, 1, 3)
    elif basis == "rbf":
        ms = lib.benchmark_metal_fastkan(P(x), P(W), P(l.w_base), P(l.grid), P(l.bias), P(y), 300,
                                         48, 40, l.num_centers, l.inv_denominator, 1, 1, 1, 3)
    elif basis == "bspline":
        g = np.ascontiguousarray(l.grid, np.float32)
        ms = lib.benchmark_metal_bspline(P(x), P(W), P(l.w_base), P(g), P(l.bias), P(y), 300, 48,
                                         40, l.grid_size, l.spline_order, 1, 1, 1, 3)
    elif basis == "relu":
        g = np.ascontiguousarray(l.grid, np.float32)
        ms = lib.benchmark_metal_relu(P(x), P(W), P(l.w_base), P(g), P(l.bias), P(y), 300, 48, 40,
                                      l.num_grids, l.inv_h, 1, 1, 1, 3)
    elif basis == "fourier":
        ms = lib.benchmark_metal_fourier(P(x), P(W), P(l.w_base), P(l.bias), P(y), 300, 48, 40,
                                         l.num_frequencies, 1, 1, 1, 3)
    elif basis == "jacobi":
        ms = lib.benchmark_metal_jacobi(P(x), P(W), P(l.w_base), P(l.bias), P(y), 300, 48, 40,
                                        l.degree, l.alpha, l.beta, 1, 1, 1, 3)
    else:
        ms = lib.benchmark_metal_wavkan(P(x), P(W), P(l.w_base), P(l.translation),
                                        P(l._inv_scale), P(l.bias), P(y), 300, 48, 40,
                                        l.num_wavelets, l.wavelet_type, 1, 1, 1, 3)
    assert 0 < ms < 1000
    assert layer_err(y, l, x, "f32", basis) <= 1e-5


@pytest.mark.parametrize("mode", ["f32", "f16"])
def test_gated_goldens(mk, mode):
    r = group(BLOCKS, f"gated_{mode}")
    blk = mk.GatedKAN(32, 64, degree=4, dtype=np.float16 if mode == "f16" else np.float32)
    for nm in ("gate_kan", "up_kan", "down_kan"):
        getattr(blk, nm).w_cheby = r[f"{nm}.w_cheby"]
        getattr(blk, nm).w_base = r[f"{nm}.w_base"]
    y = blk(r["x"])
    assert y.dtype == r["y"].dtype
    assert O.max_rel_err(y, r["y"]) <= TOL[mode]
    x3 = np.tile(r["x"], (2, 1)).reshape(2, 6, 32)
    assert blk(x3).shape == (2, 6, 32)


@pytest.mark.parametrize("basis", ["cheby", "fastkan", "bspline", "wav"])
def test_metalkan_goldens(mk, basis):
    r = group(BLOCKS, f"net_{basis}")
    deg = {"cheby": 4, "fastkan": 8, "bspline": 5, "wav": 6}[basis]
    net = mk.MetalKAN([4, 16, 8, 2], basis_type=basis, degree=deg)
    for li, l in enumerate(net.layers):
        for attr in ("w_cheby", "w_rbf", "w_spline", "w_wav", "w_base", "bias", "grid",
                     "translation", "inv_scale"):
            k = f"{li}.{attr}"
            if k in r:
                setattr(l, "_inv_scale" if attr == "inv_scale" else attr, r[k])
    assert O.max_rel_err(net(r["x"]), r["y"]) <= 1e-5
    outs = net.async_stream([r["x"], r["x"][:7]])
    assert O.max_rel_err(outs[0], r["y"]) <= 1e-5 and outs[1].shape == (7, 2)


def test_chain_pipeline_golden(mk):
    r = group(BLOCKS, "chain")
    net = mk.MetalKAN([4, 16, 8, 2], basis_type="cheby", degree=4, pipeline=True)
    for li, l in enumerate(net.layers):
        l.w_cheby, l.w_base, l.bias = r[f"{li}.w_cheby"], r[f"{li}.w_base"], r[f"{li}.bias"]
    assert O.max_rel_err(net(r["x"]), r["y"]) <= 1e-5
    net.pipeline = False
    assert O.max_rel_err(net(r["x"]), r["y"]) <= 1e-5


def test_async_mode_host_abi(mk):
    lib = mk.get_metal_bridge()
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (64, 8)).astype(np.float32)
    W = rng.normal(0, 0.1, (16, 32)).astype(np.float32)
    ys = [np.zeros((64, 16), np.float32) for _ in range(3)]
    mk.set_async(True)
    try:
        for y in ys:
            lib.metal_kan_cheby_forward(P(x), P(W), None, None, P(y), 64, 8, 16, 4, 0, 0)
    finally:
        mk.sync()
        mk.set_async(False)
    ref = O.kan_layer(x, "cheby", "f32", W, K=4)
    for y in ys:
        assert O.max_rel_err(y, ref) <= 1e-5


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_torch_module(mk, dtype):
    import torch

    np.random.seed(0)
    layer = mk.TorchMetalKANLinear(16, 8, basis="cheby", degree=4).cuda()
    t = getattr(torch, dtype)
    x = torch.randn(10, 16, device="cuda").to(t)
    y = layer(x)
    assert y.dtype == t and y.shape == (10, 8) and y.is_cuda
    mode = {"float32": "f32", "float16": "f16", "bfloat16": "bf16"}[dtype]
    ref = O.kan_layer(x.float().cpu().numpy(), "cheby", mode, layer.weight.detach().cpu().numpy(),
                      layer.base_weight.detach().cpu().numpy(), layer.bias_param.detach().cpu().numpy(), K=4)
    assert O.max_rel_err(y.detach().float().cpu().numpy(), ref.astype(np.float32)) <= TOL[mode]
    net = mk.TorchMetalKAN([4, 8, 2], basis="cheby", degree=3).cuda()
    assert net(torch.randn(10, 4)).shape == (10, 2)  # CPU input -> CPU output


@pytest.mark.parametrize("B", [2500, 40000])
def test_host_forward_chunks(mk, B):
    """kan_forward_host (what layer(x) calls on host arrays) overlaps copies and kernels in two
    chunks from 2048 rows and four from 32768 (ragged last chunk here): every row of the result is
    the layer's, checked against the oracle on rows from each chunk."""
    np.random.seed(B)
    layer = mk.ChebyKAN(512, 256, degree=5).bfloat16()
    x = np.random.default_rng(B).uniform(-1, 1, (B, 512)).astype(O.act_dtype("bf16"))
    y = layer(x)
    assert y.shape == (B, 256)
    rows = np.unique(np.linspace(0, B - 1, 40).astype(int))
    err = layer_err(y[rows], layer, x[rows], "bf16", "cheby")
    assert err <= TOL["bf16"], f"max rel err {err:.3g}"
