"""GPU: small-batch kernel for 2-bit packed weights (ternary / INT2 codebook).

The kernel decodes the packed codes on chip (never a dense copy), so its operand values must be
exactly the oracle's dequantised weights rounded to the operand dtype; outputs are compared with
the oracle (tolerance of the fp16/bf16 path), with the tensor-core path on the same layer, and the
automatic path choice is checked to pick this kernel for the BASELINE small-batch shapes.
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


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_gemv_matches_oracle_and_tc(case):
    import metal_kans as mk

    fmt, mode, B, d_in, d_out, K, gs, base, bias, imap = case
    l = _layer(mk, fmt, mode, d_in, d_out, K, gs, base, bias, imap, seed=B + K)
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
