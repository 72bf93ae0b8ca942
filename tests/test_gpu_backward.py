"""GPU: the fp32 backward (weight, bias and input gradients) against the float64 oracle.

The oracle's backward (oracle.kan_oracle.kan_layer_backward) restates the reference's backward
kernels and is itself checked against finite differences of the forward restatement on the CPU
(tests/test_oracle.py).  Here every gradient the engine returns -- through the reference's layer
API (layer.backward, MetalKAN.backward, GatedKAN.backward), the device entry point kan_backward,
and torch autograd -- is compared with it at the fp32 tolerance.
"""
import ctypes

import numpy as np
import pytest

from kan_cases import make_layer
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu

TOL32 = 1e-5


def _oracle_grads(layer, x, dY):
    kw = {}
    if layer.MAIN == "w_rbf":
        kw = dict(grid=np.asarray(layer.grid, np.float64), inv_den=layer.inv_denominator)
    elif layer.MAIN == "w_spline":
        kw = dict(grid_size=layer.grid_size, grid_min=float(layer.grid[0]), inv_h=float(layer.grid[1]))
    elif layer.MAIN == "w_relu":
        kw = dict(grid=np.asarray(layer.grid, np.float64), inv_h=layer.inv_h)
    basis = {"w_cheby": "cheby", "w_rbf": "rbf", "w_spline": "bspline", "w_relu": "relu"}[layer.MAIN]
    return O.kan_layer_backward(x, dY, basis, getattr(layer, layer.MAIN),
                                layer.w_base if layer.has_base else None, K=layer._terms(), **kw)


def _check(got, ref, what):
    err = O.max_rel_err(got, ref)
    assert err <= TOL32, f"{what}: max-rel-err {err:.3e}"


# (basis, K, B, D_in, D_out, base, bias, input spread)
CASES = [
    ("cheby", 5, 300, 40, 70, True, True, 1.3),    # inputs beyond the clamp
    ("cheby", 9, 64, 64, 64, False, False, 0.9),
    ("rbf", 8, 257, 33, 20, True, True, 1.5),
    ("bspline", 8, 200, 24, 50, True, False, 1.4),  # inputs beyond the grid
    ("cheby", 4, 1, 130, 3, True, True, 1.0),
    ("relu", 8, 150, 36, 44, True, True, 2.4),    # inputs beyond the outer tents
    ("relu", 5, 64, 70, 16, False, True, 1.9),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
@pytest.mark.parametrize("fused", [True, False])
def test_layer_backward(case, fused):
    basis, K, B, d_in, d_out, base, bias, spread = case
    if fused is False and basis != "cheby":
        pytest.skip("the unfused variant is a Chebyshev entry point")
    layer = make_layer(basis, d_in, d_out, K, bias=bias, use_base=base, seed=K + B)
    rng = np.random.default_rng(B)
    x = rng.uniform(-spread, spread, (B, d_in)).astype(np.float32)
    dY = rng.normal(0, 1, (B, d_out)).astype(np.float32)
    layer.forward(x)
    dX = layer.backward(dY, fused=fused) if basis == "cheby" else layer.backward(dY)
    rdX, rdW, rdWb, rdb = _oracle_grads(layer, x, dY)
    _check(dX, rdX, "dX")
    _check(getattr(layer, "grad_" + layer.MAIN), rdW, "dW")
    if base:
        _check(layer.grad_w_base, rdWb, "dW_base")
    if bias:
        _check(layer.grad_bias, rdb, "dbias")
    assert len(layer.parameters()) == 1 + int(base) + int(bias)
    layer.zero_grad()
    assert not np.any(getattr(layer, "grad_" + layer.MAIN))


def test_backward_3d_input_and_errors():
    import metal_kans as mk

    layer = mk.ChebyKAN(8, 6, degree=4)
    with pytest.raises(RuntimeError):
        layer.backward(np.zeros((2, 6), np.float32))  # before any forward
    x = np.random.default_rng(0).uniform(-1, 1, (2, 3, 8)).astype(np.float32)
    y = layer(x)
    dX = layer.backward(np.ones_like(y))
    assert dX.shape == x.shape
    layer.half()
    layer(x)
    with pytest.raises(RuntimeError):
        layer.backward(np.ones((6, 6), np.float32))  # fp16 layers do not train


def test_metalkan_net_backward():
    """Backward of a 3-layer Chebyshev net: each layer's gradients with the oracle fed that
    layer's own (recomputed) input, and dX of the net."""
    import metal_kans as mk

    np.random.seed(4)
    net = mk.MetalKAN([12, 16, 8, 5], basis_type="cheby", degree=4)
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (40, 12)).astype(np.float32)
    dY = rng.normal(0, 1, (40, 5)).astype(np.float32)
    net(x)
    dX = net.backward(dY)
    h = [x]
    for l in net.layers[:-1]:
        h.append(O.kan_layer(h[-1], "cheby", "f32", l.w_cheby, l.w_base, l.bias, K=4))
    g = dY
    for l, hin in zip(reversed(net.layers), reversed(h)):
        rdX, rdW, rdWb, rdb = O.kan_layer_backward(hin, g, "cheby", l.w_cheby, l.w_base, K=4)
        _check(l.grad_w_cheby, rdW, "dW")
        _check(l.grad_w_base, rdWb, "dW_base")
        _check(l.grad_bias, rdb, "dbias")
        g = rdX
    _check(dX, g, "net dX")
    assert len(net.parameters()) == 9


def test_gated_backward():
    """GatedKAN (fp32): down -> SwiGLU -> gate/up backward (gated_kan.py:145-219)."""
    import metal_kans as mk

    np.random.seed(6)
    blk = mk.GatedKAN(d_model=24, d_ffn=40, degree=4, has_bias=True)
    rng = np.random.default_rng(6)
    x = rng.normal(0, 0.7, (30, 24)).astype(np.float32)
    dY = rng.normal(0, 1, (30, 24)).astype(np.float32)
    blk(x)
    dX = blk.backward(dY)
    L = {n: getattr(blk, n) for n in ("gate_kan", "up_kan", "down_kan")}
    fwd = lambda l, h: O.kan_layer(h, "cheby", "f32", l.w_cheby, l.w_base, l.bias, K=4,  # noqa
                                   out_round=False)
    g, u = fwd(L["gate_kan"], x), fwd(L["up_kan"], x)
    hid = O.swiglu(g, u)
    rdh, rdWd, rdWbd, rdbd = O.kan_layer_backward(hid, dY, "cheby", L["down_kan"].w_cheby,
                                                  L["down_kan"].w_base, K=4)
    dg, du = O.swiglu_backward(rdh, g, u)
    rg = O.kan_layer_backward(x, dg, "cheby", L["gate_kan"].w_cheby, L["gate_kan"].w_base, K=4)
    ru = O.kan_layer_backward(x, du, "cheby", L["up_kan"].w_cheby, L["up_kan"].w_base, K=4)
    tol = 4 * TOL32  # three layers and the gating compose
    for got, ref, what in ((L["down_kan"].grad_w_cheby, rdWd, "down dW"),
                           (L["gate_kan"].grad_w_cheby, rg[1], "gate dW"),
                           (L["up_kan"].grad_w_base, ru[2], "up dW_base"),
                           (dX, rg[0] + ru[0], "dX")):
        assert O.max_rel_err(got, ref) <= tol, what
    assert len(blk.get_trainable_params()) == 9


def test_kan_backward_device_api():
    """kan_backward on device buffers (the entry point the torch operator uses), optional
    outputs skipped."""
    import metal_kans as mk
    from metal_kans._engine import DeviceBuffer

    layer = make_layer("rbf", 20, 30, 8, seed=9)
    rng = np.random.default_rng(9)
    x = rng.uniform(-2, 2, (50, 20)).astype(np.float32)
    dY = rng.normal(0, 1, (50, 30)).astype(np.float32)
    keep = []
    L = layer._descriptor(keep)
    lib = mk.get_metal_bridge()
    bx, by = DeviceBuffer.from_array(x), DeviceBuffer.from_array(dY)
    bdx, bdw = DeviceBuffer(x.nbytes), DeviceBuffer(layer.w_rbf.nbytes)
    lib.kan_backward(ctypes.byref(L), ctypes.c_void_p(bx.ptr), ctypes.c_void_p(by.ptr),
                     ctypes.c_void_p(bdx.ptr), ctypes.c_void_p(bdw.ptr), None, None, 50, None)
    dX = bdx.download(np.empty_like(x))
    dW = bdw.download(np.empty_like(layer.w_rbf))
    lib.kan_stream_synchronize(None)
    rdX, rdW, _, _ = _oracle_grads(layer, x, dY)
    _check(dX, rdX, "dX")
    _check(dW, rdW, "dW")
    layer.half()
    from metal_kans.device import KanError

    with pytest.raises(KanError):  # fp32 only
        lib.kan_backward(ctypes.byref(layer._descriptor(keep)), ctypes.c_void_p(bx.ptr),
                         ctypes.c_void_p(by.ptr), ctypes.c_void_p(bdx.ptr), None, None, None, 50,
                         None)


@pytest.mark.parametrize("basis,K", [("cheby", 4), ("rbf", 6), ("bspline", 5), ("relu", 6)])
def test_torch_autograd(basis, K):
    """TorchMetalKANLinear is differentiable on the GPU: gradients of x and of every parameter
    equal the oracle's."""
    import torch

    import metal_kans as mk

    np.random.seed(K)
    layer = mk.TorchMetalKANLinear(12, 7, basis=basis, degree=K).cuda()
    x = torch.empty(33, 12, device="cuda").uniform_(-1.2, 1.2).requires_grad_(True)
    y = layer(x)
    gy = torch.randn_like(y)
    y.backward(gy)
    ml = layer.metal_layer
    terms = ml._terms()
    kw = {}
    if basis == "rbf":
        kw = dict(grid=layer.grid.cpu().numpy(), inv_den=ml.inv_denominator)
    elif basis == "bspline":
        kw = dict(grid_size=ml.grid_size, grid_min=float(ml.grid[0]), inv_h=float(ml.grid[1]))
    elif basis == "relu":
        kw = dict(grid=layer.grid.cpu().numpy(), inv_h=ml.inv_h)
    name = basis
    wb = layer.base_weight.detach().cpu().numpy() if layer.base_weight is not None else None
    rdX, rdW, rdWb, rdb = O.kan_layer_backward(x.detach().cpu().numpy(), gy.cpu().numpy(), name,
                                               layer.weight.detach().cpu().numpy(), wb, K=terms,
                                               **kw)
    _check(x.grad.cpu().numpy(), rdX, "x.grad")
    _check(layer.weight.grad.cpu().numpy(), rdW, "weight.grad")
    if wb is not None:
        _check(layer.base_weight.grad.cpu().numpy(), rdWb, "base_weight.grad")
    _check(layer.bias_param.grad.cpu().numpy(), rdb, "bias.grad")


def test_torch_gated_module_and_compile():
    """TorchGatedKAN trains end to end (loss decreases over a few SGD steps), and the custom
    operators trace under torch.compile (aot_eager backend: fake tensors + autograd formula, no
    code generation) with the same outputs and gradients as eager."""
    import torch

    import metal_kans as mk

    torch.manual_seed(0)
    np.random.seed(0)
    blk = mk.TorchGatedKAN(16, 32, degree=4).cuda()
    x = torch.randn(64, 16, device="cuda")
    target = torch.randn(64, 16, device="cuda")
    opt = torch.optim.SGD(blk.parameters(), lr=0.05)
    losses = []
    for _ in range(5):
        opt.zero_grad()
        loss = torch.nn.functional.mse_loss(blk(x), target)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0]
    lin = mk.TorchMetalKANLinear(16, 8, basis="cheby", degree=4).cuda()
    compiled = torch.compile(lin, backend="aot_eager", fullgraph=True)
    xe = torch.randn(10, 16, device="cuda", requires_grad=True)
    xc = xe.detach().clone().requires_grad_(True)
    ye, yc = lin(xe), compiled(xc)
    torch.testing.assert_close(yc, ye)
    ye.sum().backward()
    yc.sum().backward()
    torch.testing.assert_close(xc.grad, xe.grad)
