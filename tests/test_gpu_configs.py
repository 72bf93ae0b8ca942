"""GPU parity at every BASELINE configuration, on the exact launch plans the benchmark times.

Each test builds the configuration's layers with the benchmark's own workload definitions
(bench.py: same seeds, shapes, weight formats and batch), runs them on the device with the
production kernel plan (named through kan_forward_plan and asserted), and compares a row sample
of every layer's output with the float64 oracle fed the device's own input rows, at the BASELINE
tolerance (2e-3 for f16/bf16 operands, final rounding of the result allowed).  Rows are sampled
from every 128-row tile, so every CTA row block (and every cluster split) is checked.
"""
import ctypes

import numpy as np
import pytest

from kan_cases import TOL
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mk():
    import metal_kans

    assert metal_kans.is_metal_available()
    return metal_kans


@pytest.fixture(scope="module")
def bench():
    import bench as b

    return b


def _download(buf_ptr, shape, dtype, mk):
    out = np.empty(shape, dtype)
    lib = mk.get_metal_bridge()
    lib.kan_memcpy(ctypes.c_void_p(out.ctypes.data), ctypes.c_void_p(buf_ptr), out.nbytes, 2, None)
    lib.kan_stream_synchronize(None)
    return out


def _sample(B, per_tile=2):
    """Rows spread over every 128-row tile (first, last and a middle row of the batch too)."""
    rows = set()
    for t in range(0, B, 128):
        hi = min(B, t + 128)
        rows.update(np.linspace(t, hi - 1, per_tile).round().astype(int).tolist())
    rows.update([0, B // 2, B - 1])
    return np.array(sorted(rows))


def _run(mk, bench, w, obj, layers):
    """Run the workload once on the device at its full batch; returns (x, [outputs per layer or
    intermediate buffer], y)."""
    from metal_kans._engine import DeviceBuffer

    x = w.rows(0, w.B)
    keep = []
    dx = DeviceBuffer.from_array(x)
    dy = DeviceBuffer(w.B * w.d_out * x.dtype.itemsize)
    step, inter = bench.device_step(mk, obj, layers, w.B, dx.ptr, dy.ptr, keep)
    step()
    y = _download(dy.ptr, (w.B, w.d_out), x.dtype, mk)
    code = ctypes.c_int(0)
    mk.get_metal_bridge().kan_device_error(ctypes.byref(code))
    assert code.value == 0, f"device error word {code.value}"
    return x, inter, y, keep


def _layer_err(bench, layer, x_rows, y_rows, mode):
    ref = bench._oracle_layer(layer, x_rows, mode, out_round=False)
    return O.max_rel_err_rounded(y_rows.astype(np.float64), ref, mode)


def test_c2_fastkan_layernorm_b4096(mk, bench):
    """C2: FastKAN fp16 256->256 with the LayerNorm input at B=4096 -- 32 row tiles, K split over
    a cluster (distributed-shared-memory reduction)."""
    w = bench.get_spec("c2")
    obj, layers = w.build(mk)
    plan = bench.plan_of(mk, layers, w.B)[0]
    assert plan["path"] == "tc" and plan["splits"] > 1, plan
    x, _, y, _ = _run(mk, bench, w, obj, layers)
    idx = _sample(w.B, per_tile=8)
    err = _layer_err(bench, layers[0], x[idx], y[idx], "f16")
    assert err <= TOL["f16"], f"C2 max-rel-err {err:.3e} (plan {plan})"


def test_c3_bspline_net_b8192(mk, bench):
    """C3: the BSpline net 784->512->512->10 fp16 at B=8192 -- the 512-wide layers on wide tiles
    (BN = 512) with K split in two and the two-round cluster reduction; every layer checked with
    the device's own input, then the whole net against the oracle chain."""
    w = bench.get_spec("c3")
    obj, layers = w.build(mk)
    plans = bench.plan_of(mk, layers, w.B)
    assert plans[0]["path"] == "tc" and plans[0]["BN"] == 512 and plans[0]["splits"] == 2, plans
    assert plans[1]["BN"] == 512 and plans[1]["splits"] == 2, plans
    x, inter, y, _ = _run(mk, bench, w, obj, layers)
    h1 = _download(inter[0].ptr, (w.B, 512), np.float16, mk)
    h2 = _download(inter[1].ptr, (w.B, 512), np.float16, mk)
    idx = _sample(w.B)
    for i, (l, xi, yi) in enumerate(((layers[0], x, h1), (layers[1], h1, h2), (layers[2], h2, y))):
        err = _layer_err(bench, l, xi[idx], yi[idx], "f16")
        assert err <= TOL["f16"], f"C3 layer {i}: max-rel-err {err:.3e} (plan {plans[i]})"
    ref = bench.oracle_rows(w, layers, x[idx])
    err = O.max_rel_err_rounded(y[idx].astype(np.float64), ref, "f16")
    assert err <= TOL["f16"], f"C3 net: max-rel-err {err:.3e}"


def _silu_grad(g):
    s = 1.0 / (1.0 + np.exp(-np.clip(g, -20, 20)))
    return s * (1.0 + g * (1.0 - s))


def test_c4_gated_int4_t16384(mk, bench):
    """C4: GatedKAN 2048/5632, INT4 g64 weights, bf16, 16384 tokens -- gate and up as one
    wide-tile launch with SwiGLU in its epilogue (22 wide N tiles), then the down projection.
    H is checked against SwiGLU of the exact gate/up outputs, with the bf16 rounding of gate and
    up propagated elementwise; Y against the down layer fed the device's H."""
    w = bench.get_spec("c4")
    obj, layers = w.build(mk)
    x, inter, y, _ = _run(mk, bench, w, obj, layers)
    H = _download(inter[0].ptr, (w.B, bench.C4_H), x.dtype, mk)
    idx = _sample(w.B, per_tile=1)[::2]
    xr = x[idx]
    g = bench._oracle_layer(layers[0], xr, "bf16", out_round=False)
    u = bench._oracle_layer(layers[1], xr, "bf16", out_round=False)
    href = O.swiglu(g, u).astype(np.float64)
    s = 1.0 / (1.0 + np.exp(-np.clip(g, -20, 20)))
    # gate and up are each rounded to bf16 (half an ulp, 2^-9 relative) before SwiGLU
    prop = 2.0 ** -9 * (np.abs(u * g * _silu_grad(g)) + np.abs(g * s * u))
    Hr = H[idx].astype(np.float64)
    excess = np.abs(Hr - href) - prop - O.half_ulp(href, "bf16")
    err_h = float(np.max(np.maximum(excess, 0.0)) / np.max(np.abs(href)))
    assert err_h <= TOL["bf16"], f"C4 hidden: max-rel-err {err_h:.3e}"
    err_y = _layer_err(bench, layers[2], H[idx], y[idx], "bf16")
    assert err_y <= TOL["bf16"], f"C4 down: max-rel-err {err_y:.3e}"


@pytest.fixture(scope="module", params=["ternary", "int2"])
def c5_layer(request, mk, bench):
    w = bench.get_spec(f"c5:{request.param}:4096")
    obj, layers = w.build(mk)
    return request.param, obj, layers


@pytest.mark.parametrize("B", [256, 4096])
def test_c5_tensor_core_path(mk, bench, c5_layer, B):
    """C5: 4096 -> 4096 Chebyshev T_0..T_8 + base, 2-bit weights (ternary / INT2 codebook), bf16,
    on the tensor-core path: B=256 runs 32 narrow tiles with K split over 4-CTA clusters, B=4096
    runs 256 wide tiles (BN = 512, two N = 256 accumulators per basis block)."""
    kind, obj, layers = c5_layer
    w = bench.get_spec(f"c5:{kind}:{B}")
    plan = bench.plan_of(mk, layers, B)[0]
    assert plan["path"] == "tc", plan
    if B == 256:
        assert plan["splits"] == 4 and plan["BN"] == 256, plan
    else:
        assert plan["BN"] == 512, plan
    x, _, y, _ = _run(mk, bench, w, obj, layers)
    idx = _sample(B, per_tile=4 if B == 256 else 1)
    err = _layer_err(bench, layers[0], x[idx], y[idx], "bf16")
    assert err <= TOL["bf16"], f"C5 {kind} B={B}: max-rel-err {err:.3e} (plan {plan})"
