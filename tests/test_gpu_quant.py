"""GPU: quantised layers (INT8/INT4/ternary/INT2) -- packed layouts, bit-exact dequantisation and
forward parity with the dequantised weights."""
import ctypes

import numpy as np
import pytest

from conftest import group, load_npz
from kan_cases import TOL, layer_err, make_layer, oracle_for_layer, set_mode
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mk():
    import metal_kans

    return metal_kans


QUANTS = ["int8", "int4", "ternary", "int2"]


def _quantize(mk, layer, q, gs):
    if q == "int8":
        mk.to_int8(layer, group_size=gs)
    elif q == "int4":
        mk.to_int4(layer, group_size=gs)
    elif q == "ternary":
        mk.to_ternary(layer, group_size=gs)
    else:
        mk.to_int2(layer, group_size=gs)


def _oracle_pack(q, w, gs):
    if q in ("int8", "int4"):
        bits = 8 if q == "int8" else 4
        qw, s, b, pin = O.quantize_affine(w, bits, gs, "bridge")
        return O.dequantize_affine_matrix(qw, s, b, bits, gs, w.shape, pin), (qw, s, b)
    if q == "ternary":
        p, s = O.quantize_ternary(w, gs, "bridge")
        return O.dequantize_ternary(p, s, w.shape[1], gs), (p, s)
    p, s = O.quantize_int2(w, gs, None, "bridge")
    return O.dequantize_int2(p, s, np.array([-1, -0.33333, 0.33333, 1], np.float32),
                             w.shape[1], gs), (p, s)


@pytest.mark.parametrize("q", QUANTS)
def test_packed_layout_and_dequant_bit_exact(mk, q):
    """Host quantiser output (packed arrays) and GPU/host dequantisation equal the oracle."""
    rng = np.random.default_rng(4)
    w = rng.normal(0, 0.02, (96, 8 * 9 + 3)).astype(np.float32)  # ragged rows
    gs = 64 if q in ("int8", "int4") else 32
    deq_ref, packed_ref = _oracle_pack(q, w, gs)
    if q in ("int8", "int4"):
        qw = mk.QuantizedWeight(w, bits=8 if q == "int8" else 4, group_size=gs)
        np.testing.assert_array_equal(qw.qweight, packed_ref[0])
        np.testing.assert_array_equal(qw.scales, packed_ref[1])
        np.testing.assert_array_equal(qw.biases, packed_ref[2])
    elif q == "ternary":
        qw = mk.TernaryQuantizedWeight(w, group_size=gs)
        np.testing.assert_array_equal(qw.w_packed, packed_ref[0])
        np.testing.assert_array_equal(qw.scales, packed_ref[1])
    else:
        qw = mk.Int2QuantizedWeight(w, group_size=gs)
        np.testing.assert_array_equal(qw.w_packed, packed_ref[0])
        np.testing.assert_array_equal(qw.scales, packed_ref[1])
    np.testing.assert_array_equal(qw.dequantize(), deq_ref)
    # device dequantiser (kan_dequantize) into fp32 / bf16 / f16
    keep = []
    ws = mk.device.KanWeight()
    qw._fill_struct(ws, keep)
    lib = mk.get_metal_bridge()
    from metal_kans._engine import BFLOAT16, DeviceBuffer

    for dt, npdt in ((0, np.float32), (1, np.float16), (2, BFLOAT16)):
        out = DeviceBuffer(w.size * np.dtype(npdt).itemsize)
        lib.kan_dequantize(ctypes.byref(ws), w.shape[0], w.shape[1], ctypes.c_void_p(out.ptr),
                           dt, None)
        got = np.empty(w.shape, npdt)
        out.download(got)
        lib.kan_stream_synchronize(None)
        np.testing.assert_array_equal(got, deq_ref.astype(npdt))


@pytest.mark.parametrize("q", QUANTS)
@pytest.mark.parametrize("basis,K", [("cheby", 9), ("rbf", 8), ("bspline", 8), ("wavelet", 6)])
def test_quantized_layer_fp32_forward(mk, q, basis, K):
    """After to_*(), the layer is fp32 (reference behaviour) and its packed-weight forward equals
    the fp32 forward of the dequantised weights."""
    layer = make_layer(basis, 32, 48, K, seed=7)
    _quantize(mk, layer, q, 64 if q in ("int8", "int4") else 32)
    assert layer.dtype == np.float32
    assert layer._packed(layer.MAIN) is not None
    x = np.random.default_rng(0).uniform(-1, 1, (77, 32)).astype(np.float32)
    y = layer(x)
    assert layer_err(y, layer, x, "f32", basis) <= 1e-5


@pytest.mark.parametrize("q", QUANTS)
@pytest.mark.parametrize("mode", ["f16", "bf16"])
@pytest.mark.parametrize("path", [0, 1, 2])
def test_quantized_layer_lowp_forward(mk, q, mode, path):
    """Quantised layer in f16/bf16: packed decode (SIMT) or dequantised dense copy (tensor cores)."""
    layer = make_layer("cheby", 64, 128, 9, seed=8)
    _quantize(mk, layer, q, 64)
    set_mode(layer, mode)
    # after .half()/.bfloat16() the weights are plain low-precision arrays (reference semantics)
    x = np.random.default_rng(1).uniform(-1, 1, (200, 64)).astype(np.float32)
    y = layer.forward(x, path=path)
    assert layer_err(y, layer, x, mode, "cheby") <= TOL[mode]


def test_packed_stays_authoritative_until_reassigned(mk):
    layer = make_layer("cheby", 16, 16, 4, seed=9)
    mk.to_int4(layer)
    assert layer._packed("w_cheby") is not None
    layer.w_cheby = np.zeros_like(layer.w_cheby)
    assert layer._packed("w_cheby") is None
    x = np.random.default_rng(0).uniform(-1, 1, (8, 16)).astype(np.float32)
    np.testing.assert_allclose(layer(x), oracle_for_layer(layer, x, "f32", "cheby"), atol=1e-6)


def test_reference_style_checks(mk):
    """Behavioural checks of the reference tests (test_metal_kans.py:163-174,
    test_optimizations.py:104-137): round-trip error bounds and cosine similarity floors."""
    np.random.seed(42)
    w = np.random.normal(0, 1, (32, 64)).astype(np.float32)
    assert np.max(np.abs(w - mk.QuantizedWeight(w, 8, 32).dequantize())) < 0.05
    assert np.max(np.abs(w - mk.QuantizedWeight(w, 4, 32).dequantize())) < 0.35
    for fn, attr, floor in ((mk.to_ternary, "_w_cheby_ternary", 0.4), (mk.to_int2, "_w_cheby_int2", 0.5)):
        layer = mk.ChebyKAN(16, 8, degree=4)
        x = np.random.uniform(-0.8, 0.8, (4, 16)).astype(np.float32)
        y0 = layer(x)
        fn(layer, group_size=32)
        assert hasattr(layer, attr)
        y1 = layer(x)
        cos = np.dot(y0.ravel(), y1.ravel()) / (np.linalg.norm(y0) * np.linalg.norm(y1) + 1e-8)
        assert cos > floor


BLOCKS = load_npz("blocks_small.npz")


def test_gated_int4_golden(mk):
    """GatedKAN.to_int4 through the reference classes (fp32 forward of dequantised weights)."""
    r = group(BLOCKS, "gated_int4")
    np.random.seed(3)  # same seed and call order as the golden script -> same weights
    blk = mk.GatedKAN(d_model=64, d_ffn=128, degree=5)
    blk.to_int4(group_size=64)
    for nm in ("gate_kan", "up_kan", "down_kan"):
        l = getattr(blk, nm)
        for attr in ("w_cheby", "w_base"):
            q = getattr(l, f"_{attr}_quantized")
            np.testing.assert_array_equal(q.qweight, r[f"{nm}.{attr}.qweight"])
            np.testing.assert_array_equal(q.scales, r[f"{nm}.{attr}.scales"])
            np.testing.assert_array_equal(q.biases, r[f"{nm}.{attr}.biases"])
            np.testing.assert_array_equal(getattr(l, attr), r[f"{nm}.{attr}.deq"])
    y = blk(r["x"])
    assert O.max_rel_err(y, r["y"]) <= 1e-5


@pytest.mark.parametrize("case", [(256, 640, 5120, "bf16", False, "int4"),
                                  (256, 600, 5200, "f16", True, None),
                                  (128, 384, 7680, "bf16", True, "ternary"),
                                  (64, 601, 5120, "bf16", True, "int8")],
                         ids=lambda c: "-".join(map(str, c)))
def test_gated_pair_matches_separate_launches(mk, case):
    """Gate and up in one tensor-core launch (shared basis tiles, SwiGLU in the epilogue) give the
    same hidden activations and output, bit for bit, as the separate gate, up and SwiGLU
    launches (at these shapes the pair fills >= 120 wide tiles, so it takes the one launch, and
    the separate launches do not split K either, so every output sums its K blocks in the same
    order); the block output agrees with the oracle."""
    from metal_kans._engine import DeviceBuffer

    d_model, d_ffn, B, mode, bias, quant = case
    np.random.seed(11)
    blk = mk.GatedKAN(d_model=d_model, d_ffn=d_ffn, degree=4, has_bias=bias)
    if bias:
        rng = np.random.default_rng(5)
        for l in blk._layers():
            l.bias = rng.normal(0, 0.1, l.out_features).astype(np.float32)
    if quant == "int4":
        blk.to_int4(group_size=64)
    elif quant == "ternary":
        blk.to_ternary(group_size=64)
    elif quant == "int8":
        blk.to_int8(group_size=64)
    blk.bfloat16() if mode == "bf16" else blk.half()
    act = blk.gate_kan.dtype
    x = np.random.default_rng(B).normal(0, 1, (B, d_model)).astype(np.float32).astype(act)
    lib = mk.get_metal_bridge()
    keep = []
    descs = [l._descriptor(keep) for l in blk._layers()]
    pair = blk._pair(descs[0], descs[1], keep)
    assert pair, "pair packing refused a compatible gate/up"
    n0 = lib.kan_launch_count()
    dx = DeviceBuffer.from_array(x)
    outs = []
    for p in (pair, 0):  # one launch for gate + up, then the separate launches
        dh = DeviceBuffer(B * d_ffn * 2)
        dy = DeviceBuffer(B * d_model * 2)
        lib.kan_gated_forward_pair(*(ctypes.byref(d) for d in descs), ctypes.c_void_p(p),
                                   ctypes.c_void_p(dx.ptr), ctypes.c_void_p(dh.ptr),
                                   ctypes.c_void_p(dy.ptr), B, None)
        h = dh.download(np.empty((B, d_ffn), act))
        y = dy.download(np.empty((B, d_model), act))
        lib.kan_stream_synchronize(None)
        outs.append((h.view(np.uint16).copy(), y.view(np.uint16).copy()))
        if p:  # gate + up as one launch, then down
            assert lib.kan_launch_count() - n0 == 2
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    # the public forward takes the fused launch; oracle of the block: each layer rounded to the
    # act dtype, SwiGLU rounded, down projection unrounded
    y = blk(x)
    xf = x.astype(np.float32)
    g = oracle_for_layer(blk.gate_kan, xf, mode, "cheby")
    u = oracle_for_layer(blk.up_kan, xf, mode, "cheby")
    hid = O.swiglu(g, u).astype(np.float32).astype(act).astype(np.float32)
    ref = oracle_for_layer(blk.down_kan, hid, mode, "cheby", out_round=False)
    assert O.max_rel_err_rounded(y.astype(np.float64), ref, mode) <= TOL[mode]
