"""GPU: the tensor-core small-batch kernels for 2-bit packed weights (ternary / INT2 codebook).

Two kernels serve the path: ternary weights in groups of 64/128 codes at 5 <= B <= 16 run the
8-bit kernel (codes as signed bytes, the fixed-point basis, exact int32 sums per group scaled in an
epilogue; every basis but Jacobi); the others the 16-bit kernel (codes decoded into operand-dtype
weights, Chebyshev layers).  Both decode the packed codes on chip (never a dense copy), so the
weights they multiply are exactly the oracle's dequantised weights rounded to the operand dtype;
outputs are compared with the oracle (tolerance of the fp16/bf16 path), with the tensor-core path on
the same layer, and the automatic path choice is checked to pick them for the BASELINE small-batch
shapes.  The plan's operand bits name the kernel each case runs.
"""
import numpy as np
import pytest

from kan_cases import TOL, layer_err, set_mode
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu

GEMV, TC = 3, 2

# (format, mode, B, D_in, D_out, K, group, base, bias, input map)
CASES = [
    ("ternary", "bf16", 1, 1024, 256, 9, 64, True, True, "none"),
    ("ternary", "bf16", 16, 1024, 512, 9, 64, True, False, "none"),
    ("int2", "bf16", 16, 1024, 384, 9, 64, True, True, "none"),   # ragged last row block
    ("ternary", "f16", 7, 1024, 256, 5, 32, True, True, "none"),
    ("int2", "f16", 33, 1024, 256, 4, 128, False, True, "none"),
    ("ternary", "bf16", 64, 1024, 256, 9, 64, True, True, "none"),
    ("int2", "bf16", 16, 1024, 256, 9, 32, True, True, "tanh"),
    ("ternary", "bf16", 16, 576, 256, 8, 64, False, True, "none"),  # ragged last K split
]


def _layer(mk, fmt, mode, d_in, d_out, K, gs, base, bias, imap, seed):
    np.random.seed(seed)
    l = mk.ChebyKAN(d_in, d_out, degree=K, bias=bias, use_base=base, input_map=imap)
    rng = np.random.default_rng(seed)
    l.w_cheby = rng.normal(0, 0.05, l.w_cheby.shape).astype(np.float32)
    if base:
        l.w_base = rng.normal(0, 0.05, l.w_base.shape).astype(np.float32)
    if bias:
        l.bias = rng.normal(0, 0.1, d_out).astype(np.float32)
    if fmt == "ternary":
        mk.to_ternary(l, group_size=gs)
    else:
        mk.to_int2(l, group_size=gs)
    return set_mode(l, mode)


def _plan(mk, layer, B, path=GEMV):
    import ctypes

    keep = []
    info = (ctypes.c_int * 6)()
    mk.get_metal_bridge().kan_forward_plan(ctypes.byref(layer._descriptor(keep)), B, path, info)
    return list(info)


def _bits(fmt, B, gs):
    return 8 if fmt == "ternary" and 5 <= B <= 16 and gs in (64, 128) else 16


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_gemv_matches_oracle_and_tc(case):
    import metal_kans as mk

    fmt, mode, B, d_in, d_out, K, gs, base, bias, imap = case
    l = _layer(mk, fmt, mode, d_in, d_out, K, gs, base, bias, imap, seed=B + K)
    assert _plan(mk, l, B)[1] == _bits(fmt, B, gs)
    x = np.random.default_rng(B).uniform(-1.2, 1.2, (B, d_in)).astype(O.act_dtype(mode))
    y = l.forward(x, path=GEMV)
    err = layer_err(y, l, x, mode, "cheby")
    assert err <= TOL[mode], f"max rel err {err:.3g}"
    y_tc = l.forward(x, path=TC)
    d = np.abs(y.astype(np.float64) - y_tc.astype(np.float64)).max()
    assert d <= 2 * TOL[mode] * np.abs(y_tc.astype(np.float64)).max()
    # deterministic: a second call is bit-identical
    np.testing.assert_array_equal(l.forward(x, path=GEMV).view(np.uint16), y.view(np.uint16))


def test_gemv_rejects_unsupported_layers():
    import metal_kans as mk
    from metal_kans.device import KanError

    l = _layer(mk, "ternary", "bf16", 1024, 256, 9, 64, True, True, "none", seed=1)
    x = np.zeros((65, 1024), O.act_dtype("bf16"))  # B > 64
    with pytest.raises(KanError):
        l.forward(x, path=GEMV)
    d = mk.ChebyKAN(1024, 256, degree=9).bfloat16()  # dense weights
    with pytest.raises(KanError):
        d.forward(x[:4], path=GEMV)


@pytest.mark.parametrize("fmt", ["ternary", "int2"])
@pytest.mark.parametrize("B", [1, 16])
def test_c5_layer_small_batch(fmt, B):
    """BASELINE config 5 shape (4096 -> 4096, T_0..T_8 + base, group 64, bf16) at B <= 16: the
    automatic path is the small-batch kernel and matches the oracle."""
    import metal_kans as mk
    from metal_kans.quantization import attach_packed, packed_from_codes

    D, K, gs = 4096, 9, 64
    rng = np.random.default_rng(7)
    np.random.seed(7)
    l = mk.ChebyKAN(D, D, degree=K, bias=False, use_base=True)
    for nm, cols in (("w_cheby", D * K), ("w_base", D)):
        g = cols // gs
        if fmt == "ternary":
            codes = rng.integers(0, 3, (D, cols)).astype(np.uint32)
            s = rng.uniform(0.01, 0.05, (D, g)).astype(np.float32)
            cb = None
        else:
            codes = rng.integers(0, 4, (D, cols)).astype(np.uint32)
            s = rng.uniform(0.5, 1.5, (D, g)).astype(np.float32)
            cb = rng.normal(0, 0.03, 4).astype(np.float32)
        attach_packed(l, nm, packed_from_codes(fmt, O._pack2(codes), s, (D, cols), gs, cb))
    l.bfloat16()
    x = rng.uniform(-1, 1, (B, D)).astype(O.act_dtype("bf16"))
    # the automatic path: the CUDA-core small-batch kernel for ternary weights at B <= 4, this
    # kernel otherwise
    import ctypes

    keep = []
    info = (ctypes.c_int * 6)()
    mk.get_metal_bridge().kan_forward_plan(ctypes.byref(l._descriptor(keep)), B, 0, info)
    auto = 4 if (fmt == "ternary" and B <= 4) else GEMV
    assert info[0] == auto
    y_auto = l.forward(x)
    np.testing.assert_array_equal(y_auto.view(np.uint16), l.forward(x, path=auto).view(np.uint16))
    y = l.forward(x, path=GEMV)
    err = layer_err(y, l, x, "bf16", "cheby")
    assert err <= TOL["bf16"], f"max rel err {err:.3g}"


# the 8-bit kernel on every basis it takes: (basis, mode, B, D_in, D_out, K, group, base, bias, map)
I8_CASES = [
    ("rbf", "f16", 5, 1024, 300, 8, 64, True, True, "layernorm"),   # ragged last row block
    ("bspline", "bf16", 8, 1024, 256, 8, 128, True, False, "none"),
    ("wavelet", "bf16", 9, 512, 384, 6, 64, False, True, "none"),
    ("relu", "f16", 16, 1024, 128, 8, 64, True, True, "none"),
    ("fourier", "bf16", 12, 1024, 256, 9, 64, True, True, "none"),
    ("cheby", "f16", 16, 2048, 640, 5, 128, True, True, "tanh"),
]


@pytest.mark.parametrize("case", I8_CASES, ids=lambda c: "-".join(map(str, c)))
def test_gemv_i8_bases(case):
    import metal_kans as mk
    from kan_cases import make_layer, randomize_bias

    basis, mode, B, d_in, d_out, K, gs, base, bias, imap = case
    l = make_layer(basis, d_in, d_out, K, bias=bias, use_base=base, input_map=imap, seed=B + K)
    if bias:
        randomize_bias(l)
    mk.to_ternary(l, group_size=gs)
    set_mode(l, mode)
    plan = _plan(mk, l, B, 0)
    assert plan[0] == GEMV and plan[1] == 8, plan  # the automatic choice at 5 <= B <= 16
    x = np.random.default_rng(B).normal(0, 1, (B, d_in)).astype(O.act_dtype(mode))
    y = l.forward(x)
    err = layer_err(y, l, x, mode, basis)
    assert err <= TOL[mode], f"max rel err {err:.3g}"
    y_tc = l.forward(x, path=TC)
    d = np.abs(y.astype(np.float64) - y_tc.astype(np.float64)).max()
    assert d <= 2 * TOL[mode] * np.abs(y_tc.astype(np.float64)).max()
    np.testing.assert_array_equal(l.forward(x).view(np.uint16), y.view(np.uint16))


@pytest.mark.parametrize("B", [6, 16])
def test_gemv_i8_code3(B):
    """Ternary codes equal to 3 (the reference's dequantiser maps them to 0) in the 8-bit
    kernel's byte-permute decoder, against the oracle on the edited packed weights."""
    import metal_kans as mk
    from kan_cases import make_layer, randomize_bias

    layer = make_layer("cheby", 1024, 384, 9, seed=B)
    randomize_bias(layer)
    mk.to_ternary(layer, group_size=64)
    rng = np.random.default_rng(B)
    for name in (layer.MAIN, "w_base"):
        pk = layer._packed(name)
        words = pk.w_packed.view(np.uint32)
        field = rng.integers(0, 16, words.shape).astype(np.uint32)
        hit = rng.random(words.shape) < 0.5
        words |= np.where(hit, np.uint32(3) << (2 * field), np.uint32(0)).astype(np.uint32)
    set_mode(layer, "bf16")
    assert _plan(mk, layer, B, 0)[:2] == [GEMV, 8]
    x = np.random.default_rng(B).normal(0, 1, (B, 1024)).astype(O.act_dtype("bf16"))
    y = layer.forward(x)
    ref = O.kan_layer(x, "cheby", "bf16", layer._packed(layer.MAIN).dequantize(),
                      layer._packed("w_base").dequantize(), np.asarray(layer.bias, np.float32),
                      K=layer._terms(), out_round=False)
    err = O.max_rel_err_rounded(np.asarray(y).astype(np.float64), ref, "bf16")
    assert err <= TOL["bf16"], f"max rel err {err:.3g}"


def test_gemv_i8_aborts_and_recovers():
    """With a wait limit of 200 cycles the 8-bit kernel's first wait for a basis tile (behind the
    basis pre-pass) expires; the call reports the timeout, the next call with the default limit
    matches the oracle."""
    import ctypes

    import metal_kans as mk
    from kan_cases import make_layer
    from metal_kans.device import KanError

    layer = make_layer("cheby", 2048, 1024, 9, seed=4)
    mk.to_ternary(layer, group_size=64)
    layer.bfloat16()
    x = np.random.default_rng(6).normal(0, 1, (12, 2048)).astype(O.act_dtype("bf16"))
    assert _plan(mk, layer, 12)[:2] == [GEMV, 8]
    lib = mk.get_metal_bridge()
    lib.kan_set_wait_limit(200)
    try:
        with pytest.raises(KanError, match="bounded wait"):
            layer.forward(x, path=GEMV)
    finally:
        lib.kan_set_wait_limit(0)
    code = ctypes.c_int(0)
    lib.kan_device_error(ctypes.byref(code))
    assert code.value == 0
    y = layer.forward(x, path=GEMV)
    err = layer_err(y, layer, x, "bf16", "cheby")
    assert err <= TOL["bf16"], f"after the aborted call: max-rel-err {err:.3e}"
