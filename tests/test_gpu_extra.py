"""GPU parity of the composite layer kinds -- MultKAN, LowRankKAN, RationalKAN -- against the oracle
(oracle.kan_oracle.mult_layer / lowrank_layer / rational_layer, which the reference-class goldens in
tests/golden pin), through the layer classes, the reference's host-pointer entry points and the
benchmark entry points."""
import numpy as np
import pytest

from kan_cases import TOL, set_mode
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mk():
    import metal_kans

    return metal_kans


def P(a):
    return a.ctypes.data


def _err(y, ref, mode):
    return O.max_rel_err_rounded(np.asarray(y).astype(np.float64), np.asarray(ref, np.float64), mode)


# (D_in, D_out, num_mult, num_grids, B)
MULT = [(24, 40, None, 8, 130), (64, 96, 10, 6, 1024), (16, 9, 0, 5, 33), (300, 256, 128, 8, 4096)]


@pytest.mark.parametrize("mode", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("case", MULT, ids=lambda c: "-".join(map(str, c)))
def test_mult_vs_oracle(mk, case, mode):
    d_in, d_out, nm, ng, B = case
    np.random.seed(d_in + d_out)
    l = set_mode(mk.MultKAN(d_in, d_out, num_mult=nm, num_grids=ng), mode)
    rng = np.random.default_rng(B)
    l.bias = rng.normal(0, 0.1, l.internal_out).astype(l.dtype)
    x = rng.uniform(-1.2, 1.2, (B, d_in)).astype(np.float32)
    y = l(x)
    assert y.shape == (B, d_out) and y.dtype == l.dtype
    # the internal outputs are rounded to the layer dtype before the products (MPS output), so
    # the oracle is compared after its own final rounding, at the layer tolerance
    ref = O.mult_layer(x, mode, np.asarray(l.w_rbf, np.float32), np.asarray(l.w_base, np.float32),
                       np.asarray(l.bias, np.float32), grid=np.asarray(l.grid), inv_den=l.inv_denominator,
                       num_add=l.num_add, num_mult=l.num_mult)
    assert O.max_rel_err(y, ref) <= (TOL[mode] if mode == "f32" else 2 * TOL[mode])


# (D_in, D_out, rank, num_grids, B, base, bias)
LOWRANK = [(24, 40, 8, 8, 130, True, True), (128, 256, 16, 8, 2048, True, False),
           (40, 12, 6, 5, 1, False, True)]


@pytest.mark.parametrize("mode", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("case", LOWRANK, ids=lambda c: "-".join(map(str, c)))
def test_lowrank_vs_oracle(mk, case, mode):
    d_in, d_out, rank, ng, B, base, bias = case
    np.random.seed(rank + B)
    l = mk.LowRankKAN(d_in, d_out, rank=rank, num_grids=ng, bias=bias, use_base=base)
    rng = np.random.default_rng(rank)
    if bias:
        l.bias = rng.normal(0, 0.1, d_out).astype(np.float32)
    set_mode(l, mode)
    x = rng.uniform(-1.2, 1.2, (B, d_in)).astype(np.float32)
    y = l(x)
    ref = O.lowrank_layer(x, mode, np.asarray(l.w_down, np.float32), np.asarray(l.w_up, np.float32),
                          np.asarray(l.w_base, np.float32) if base else None,
                          np.asarray(l.bias, np.float32) if bias else None,
                          grid=np.asarray(l.grid), inv_den=l.inv_denominator, out_round=False)
    assert _err(y, ref, mode) <= TOL[mode]


# (D_in, D_out, p, q, B, base, bias, spread)
RATIONAL = [(24, 40, 4, 2, 130, True, True, 1.3), (64, 96, 6, 3, 1000, True, False, 0.9),
            (8, 5, 1, 0, 3, False, True, 1.0), (33, 70, 8, 8, 257, True, True, 1.5)]


@pytest.mark.parametrize("case", RATIONAL, ids=lambda c: "-".join(map(str, c)))
def test_rational_vs_oracle(mk, case):
    d_in, d_out, p, q, B, base, bias, spread = case
    np.random.seed(p * 10 + q)
    l = mk.RationalKAN(d_in, d_out, p_degree=p, q_degree=q, bias=bias, use_base=base)
    rng = np.random.default_rng(B)
    if bias:
        l.bias = rng.normal(0, 0.1, d_out).astype(np.float32)
    l.w_q = rng.normal(0, 0.5, l.w_q.shape).astype(np.float32)  # |Q| well away from 0
    x = rng.uniform(-spread, spread, (B, d_in)).astype(np.float32)
    y = l(x)
    ref = O.rational_layer(x, l.w_p, l.w_q, l.w_base if base else None, l.bias if bias else None,
                           p_degree=p, q_degree=q)
    assert O.max_rel_err(y, ref) <= TOL["f32"]


def test_host_entry_points(mk):
    """metal_kan_{mult,lowrank}_forward{,_fp16} and metal_kan_rational_forward on host pointers,
    and their benchmark_metal_* twins (a positive time, Y left behind = the forward)."""
    lib = mk.get_metal_bridge()
    rng = np.random.default_rng(3)
    B, Di, Do, K = 50, 20, 14, 8
    for dt, mode in ((np.float32, "f32"), (np.float16, "f16")):
        sfx = "" if mode == "f32" else "_fp16"
        x = rng.uniform(-1, 1, (B, Di)).astype(dt)
        grid = np.linspace(-2, 2, K).astype(dt)
        # mult: 6 additive + 8 multiplicative outputs, 22 internal ones
        na, nm = 6, 8
        W = rng.normal(0, 0.2, (na + 2 * nm, Di * K)).astype(dt)
        Wb = rng.normal(0, 0.2, (na + 2 * nm, Di)).astype(dt)
        b = rng.normal(0, 0.1, na + 2 * nm).astype(dt)
        y = np.empty((B, Do), dt)
        getattr(lib, "metal_kan_mult_forward" + sfx)(P(x), P(W), P(Wb), P(grid), P(b), P(y), B, Di,
                                                      Do, na, nm, K, 3.0625, 1, 1)
        ref = O.mult_layer(x, mode, W, Wb, b, grid=grid, inv_den=3.0625, num_add=na, num_mult=nm)
        assert O.max_rel_err(y, ref) <= 2 * TOL[mode]
        # lowrank: rank 5
        Wd = rng.normal(0, 0.2, (5, Di * K)).astype(dt)
        Wu = rng.normal(0, 0.3, (Do, 5)).astype(dt)
        Wb2 = rng.normal(0, 0.2, (Do, Di)).astype(dt)
        b2 = rng.normal(0, 0.1, Do).astype(dt)
        getattr(lib, "metal_kan_lowrank_forward" + sfx)(P(x), P(Wd), P(Wu), P(Wb2), P(grid), P(b2),
                                                         P(y), B, Di, Do, 5, K, 3.0625, 1, 1)
        ref = O.lowrank_layer(x, mode, Wd, Wu, Wb2, b2, grid=grid, inv_den=3.0625, out_round=False)
        assert _err(y, ref, mode) <= TOL[mode]
    x = rng.uniform(-1.2, 1.2, (B, Di)).astype(np.float32)
    Wp = rng.normal(0, 0.2, (Do, Di * 4)).astype(np.float32)
    Wq = rng.normal(0, 0.5, (Do, Di * 2)).astype(np.float32)
    Wb = rng.normal(0, 0.2, (Do, Di)).astype(np.float32)
    b = rng.normal(0, 0.1, Do).astype(np.float32)
    y = np.empty((B, Do), np.float32)
    lib.metal_kan_rational_forward(P(x), P(Wp), P(Wq), P(Wb), P(b), P(y), B, Di, Do, 4, 2, 1, 1)
    assert O.max_rel_err(y, O.rational_layer(x, Wp, Wq, Wb, b, p_degree=4, q_degree=2)) <= 1e-5
    ms = lib.benchmark_metal_rational(P(x), P(Wp), P(Wq), P(Wb), P(b), P(y), B, Di, Do, 4, 2, 1, 1,
                                      1, 3)
    assert 0 < ms < 1000
    for cls, kw in ((mk.MultKAN, dict(num_grids=6)), (mk.LowRankKAN, dict(rank=4, num_grids=6))):
        layer = cls(Di, Do, **kw)
        assert 0 < layer.benchmark(x, warmup=1, iters=3) < 1000


def test_rational_rejects_high_degree(mk):
    from metal_kans.device import KanError

    l = mk.RationalKAN(8, 4, p_degree=12, q_degree=6)  # p + q > 16
    with pytest.raises(KanError):
        l(np.zeros((2, 8), np.float32))


@pytest.mark.parametrize("basis", ["rational", "mult", "lowrank"])
def test_metalkan_composite_nets(mk, basis):
    """MetalKAN stacks of the composite kinds (metal_kan.py:74-84), layer by layer against the
    oracle, 3-D input."""
    np.random.seed(11)
    net = mk.MetalKAN([12, 16, 6], basis_type=basis, degree=4)
    x = np.random.default_rng(11).uniform(-1, 1, (2, 5, 12)).astype(np.float32)
    y = net(x)
    assert y.shape == (2, 5, 6)
    h = x.reshape(-1, 12)
    for l in net.layers:
        if basis == "rational":
            h = O.rational_layer(h, l.w_p, l.w_q, l.w_base, l.bias, p_degree=l.p_degree,
                                 q_degree=l.q_degree)
        elif basis == "mult":
            h = O.mult_layer(h, "f32", l.w_rbf, l.w_base, l.bias, grid=l.grid,
                             inv_den=l.inv_denominator, num_add=l.num_add, num_mult=l.num_mult)
        else:
            h = O.lowrank_layer(h, "f32", l.w_down, l.w_up, l.w_base, l.bias, grid=l.grid,
                                inv_den=l.inv_denominator)
    assert O.max_rel_err(y.reshape(-1, 6), h) <= 1e-5
