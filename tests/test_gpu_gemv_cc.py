"""GPU: the CUDA-core small-batch path (B <= 4) for ternary / INT8 / INT4 weights.

The kernel never expands the packed codes: it decodes them on chip into bytes and takes integer
dot products against a fixed-point copy of the basis values (two signed bytes per value, exact
for every operand-dtype value of magnitude >= 2^-6), scaling each 16-code sum by its group's
scale.  Ternary weights come out exactly as the reference's dequantiser rounded to the operand
dtype; INT8/INT4 weights enter as their exact fp32 dequantised values (q * scale + minimum), so
those cases are checked against the oracle fed the same exact weights.  Its outputs are compared with the oracle (tolerance of the fp16/bf16 path), with the
tensor-core path on the same layer, and a second call must be bit-identical (the split-K partials
are summed in a fixed order).
"""
import ctypes

import numpy as np
import pytest

from kan_cases import TOL, layer_err, make_layer, randomize_bias, set_mode
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu

CC, TC = 4, 2


def _quantize(mk, layer, q, gs):
    {"ternary": mk.to_ternary, "int8": mk.to_int8, "int4": mk.to_int4}[q](layer, group_size=gs)


def _plan(mk, layer, B, path=0):
    keep = []
    info = (ctypes.c_int * 6)()
    mk.get_metal_bridge().kan_forward_plan(ctypes.byref(layer._descriptor(keep)), B, path, info)
    return list(info)


# (format, mode, basis, K, D_in, D_out, B, group, base, bias, input map)
CASES = [
    ("ternary", "bf16", "cheby", 9, 1024, 256, 1, 64, True, True, "none"),
    ("ternary", "bf16", "cheby", 9, 1024, 100, 4, 64, True, True, "tanh"),       # ragged rows
    ("ternary", "f16", "rbf", 8, 1024, 192, 3, 32, True, False, "layernorm"),
    ("ternary", "bf16", "bspline", 8, 1024, 160, 2, 128, True, True, "none"),
    ("ternary", "bf16", "wavelet", 6, 1024, 96, 1, 64, False, True, "none"),
    ("ternary", "f16", "cheby", 5, 1536, 224, 4, 64, True, True, "none"),
    ("int8", "bf16", "cheby", 9, 512, 256, 1, 64, True, True, "none"),
    ("int8", "f16", "rbf", 8, 512, 200, 4, 32, True, True, "layernorm"),
    ("int8", "bf16", "wavelet", 6, 1024, 128, 2, 128, True, False, "tanh"),
    ("int4", "bf16", "cheby", 5, 512, 256, 4, 64, True, True, "none"),
    ("int4", "f16", "bspline", 8, 1024, 96, 1, 32, True, True, "none"),
    ("int4", "bf16", "cheby", 9, 1024, 130, 3, 128, False, True, "tanh"),
    ("ternary", "bf16", "relu", 8, 1024, 128, 2, 64, True, True, "none"),
    ("ternary", "f16", "fourier", 9, 1024, 96, 4, 64, True, True, "none"),
    ("int8", "bf16", "relu", 5, 1024, 64, 1, 64, True, False, "none"),
    ("int4", "f16", "fourier", 5, 1024, 160, 3, 32, False, True, "none"),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_cc_matches_oracle_and_tc(case):
    import metal_kans as mk

    fmt, mode, basis, K, d_in, d_out, B, gs, base, bias, imap = case
    layer = make_layer(basis, d_in, d_out, K, bias=bias, use_base=base, input_map=imap,
                       seed=B + K + d_out)
    if bias:
        randomize_bias(layer)
    _quantize(mk, layer, fmt, gs)
    set_mode(layer, mode)
    assert _plan(mk, layer, B)[0] == CC  # the automatic choice for B <= 4
    x = np.random.default_rng(d_out).normal(0, 1, (B, d_in)).astype(O.act_dtype(mode))
    y = layer.forward(x, path=CC)
    # INT8/INT4: this path multiplies by the exact fp32 dequantised weight (q * scale + minimum),
    # not its rounding to the operand dtype; ternary weights are exact either way
    err = layer_err(y, layer, x, mode, basis, exact_weights=fmt != "ternary")
    assert err <= TOL[mode], f"max rel err {err:.3g}"
    y_tc = layer.forward(x, path=TC)
    ref = np.abs(y_tc.astype(np.float64)).max()
    # the tensor-core path rounds INT8/INT4 weights to the operand dtype: the two paths may then
    # differ by the gap between the oracle with exact and with rounded weights, on top of each
    # one's own tolerance
    gap = 0.0
    if fmt != "ternary":
        from kan_cases import oracle_for_layer

        exact = oracle_for_layer(layer, x, mode, basis, out_round=False, exact_weights=True)
        rounded = oracle_for_layer(layer, x, mode, basis, out_round=False)
        gap = np.abs(exact - rounded).max()
    assert np.abs(y.astype(np.float64) - y_tc.astype(np.float64)).max() <= 2 * TOL[mode] * ref + gap
    np.testing.assert_array_equal(layer.forward(x, path=CC).view(np.uint16), y.view(np.uint16))


@pytest.fixture(scope="module", params=["ternary", "int8", "int4"])
def c5_layer(request):
    """BASELINE config 5's layer (4096 -> 4096, T_0..T_8 + base, group 64, bf16) with the
    format's weights: ternary from the benchmark's codes, INT8/INT4 quantised from N(0, 0.02)."""
    import metal_kans as mk

    fmt = request.param
    if fmt == "ternary":
        import bench

        _, layers = bench.get_spec("c5:ternary:1").build(mk)
        return fmt, layers[0]
    np.random.seed(5)
    l = mk.ChebyKAN(4096, 4096, degree=9, bias=False, use_base=True)
    rng = np.random.default_rng(5)
    l.w_cheby = rng.normal(0, 0.02, l.w_cheby.shape).astype(np.float32)
    l.w_base = rng.normal(0, 0.02, l.w_base.shape).astype(np.float32)
    _quantize(mk, l, fmt, 64)
    return fmt, l.bfloat16()


@pytest.mark.parametrize("B", [1, 2, 4])
def test_cc_c5_layer(c5_layer, B):
    """The C5 layer at B <= 4 on the CUDA-core path (K split over several CTAs per row block,
    partials summed by the last one): oracle, tensor-core agreement, determinism."""
    import metal_kans as mk

    fmt, l = c5_layer
    plan = _plan(mk, l, B)
    assert plan[0] == CC and plan[2] > 1, plan
    x = np.random.default_rng(B).uniform(-1, 1, (B, 4096)).astype(O.act_dtype("bf16"))
    y = l.forward(x)
    err = layer_err(y, l, x, "bf16", "cheby", exact_weights=fmt != "ternary")
    assert err <= TOL["bf16"], f"{fmt} B={B}: max rel err {err:.3g}"
    np.testing.assert_array_equal(l.forward(x, path=CC).view(np.uint16), y.view(np.uint16))


@pytest.mark.parametrize("gs", [16, 64])
@pytest.mark.parametrize("B", [1, 3])
def test_cc_ternary_code3(gs, B):
    """Ternary codes equal to 3 (which the reference's dequantiser maps to 0): the byte-permute
    decoder, against the oracle on the layer's own dequantised weights."""
    import metal_kans as mk

    layer = make_layer("cheby", 1024, 384, 9, seed=gs + B)
    randomize_bias(layer)
    mk.to_ternary(layer, group_size=gs)
    rng = np.random.default_rng(gs)
    for name in (layer.MAIN, "w_base"):
        pk = layer._packed(name)
        words = pk.w_packed.view(np.uint32)
        # turn one code in about 32 into a 3
        field = rng.integers(0, 16, words.shape).astype(np.uint32)
        hit = rng.random(words.shape) < 0.5
        words |= np.where(hit, np.uint32(3) << (2 * field), np.uint32(0)).astype(np.uint32)
        assert not pk._no_code3()
    set_mode(layer, "bf16")
    assert _plan(mk, layer, B)[0] == CC
    x = np.random.default_rng(B).normal(0, 1, (B, 1024)).astype(O.act_dtype("bf16"))
    y = layer.forward(x)
    # the layer's weight attributes hold the dequantised copies made before the edit: the oracle
    # takes the edited packed weights' own dequantisation (rounded to bf16 inside kan_layer)
    ref = O.kan_layer(x, "cheby", "bf16", layer._packed(layer.MAIN).dequantize(),
                      layer._packed("w_base").dequantize(), np.asarray(layer.bias, np.float32),
                      K=layer._terms(), out_round=False)
    err = O.max_rel_err_rounded(np.asarray(y).astype(np.float64), ref, "bf16")
    assert err <= TOL["bf16"], f"max rel err {err:.3g}"


def test_cc_rejects_unsupported():
    import metal_kans as mk
    from metal_kans.device import KanError

    l = make_layer("cheby", 1024, 256, 9, seed=2)
    mk.to_ternary(l, group_size=64)
    l.bfloat16()
    x = np.zeros((5, 1024), O.act_dtype("bf16"))  # B > 4
    with pytest.raises(KanError):
        l.forward(x, path=CC)
    m = make_layer("cheby", 1024, 256, 9, seed=3)
    mk.to_int2(m, group_size=64)  # INT2 codebook: the tensor-core small-batch kernel's
    m.bfloat16()
    with pytest.raises(KanError):
        m.forward(x[:2], path=CC)
    f = make_layer("cheby", 1024, 256, 9, seed=4)
    mk.to_ternary(f, group_size=64)  # fp32 layers keep the exact path
    with pytest.raises(KanError):
        f.forward(np.zeros((2, 1024), np.float32), path=CC)
    j = make_layer("jacobi", 1024, 256, 4, seed=5)
    mk.to_ternary(j, group_size=64)  # Jacobi values exceed 1: no 14-bit fixed-point basis
    j.bfloat16()
    with pytest.raises(KanError):
        j.forward(x[:2], path=CC)
    assert _plan(mk, j, 2)[0] != CC
    g = make_layer("cheby", 1024, 256, 9, seed=6)
    mk.to_ternary(g, group_size=48)  # group index by shift: power-of-two groups only
    g.bfloat16()
    with pytest.raises(KanError):
        g.forward(x[:2], path=CC)
