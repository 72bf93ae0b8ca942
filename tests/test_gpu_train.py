"""GPU: the fp32 training step and the optimisers.

* the optimiser kernels (AdamW, Adam with coupled decay, SGD with momentum / Nesterov, Lion)
  against the float64 restatement of the reference's update formulas (oracle.optim_update), for
  given gradients;
* the fused ``train_step`` of the Chebyshev / RBF / B-spline layers against the same step
  composed from the layer API (forward, MSE gradient, backward, optim.AdamW) -- the same kernels,
  so bit-identical -- and against the oracle (forward, MSE gradient, backward, AdamW in float64);
* optimisers over ``parameters()``: the layers see their updated weights on the next forward;
* ``MetalKAN.train_step`` / ``build_train_step`` reduce the loss of a small regression.
"""
import math

import numpy as np
import pytest

from kan_cases import make_layer
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mk():
    import metal_kans

    return metal_kans


def P(a):
    return a.ctypes.data


@pytest.mark.parametrize("op", ["adamw", "adam", "sgd", "sgd_nesterov", "lion"])
def test_optimizer_kernels_vs_oracle(mk, op):
    lib = mk.get_metal_bridge()
    rng = np.random.default_rng(1)
    n = 100_003
    p = rng.normal(0, 1, n).astype(np.float32)
    g = rng.normal(0, 0.1, n).astype(np.float32)
    m = rng.normal(0, 0.01, n).astype(np.float32)
    v = np.abs(rng.normal(0, 0.001, n)).astype(np.float32)
    p0, m0, v0 = p.copy(), m.copy(), v.copy()
    lr, b1, b2, eps, wd, t = 1e-3, 0.9, 0.999, 1e-8, 0.05, 3
    lr_t = lr * math.sqrt(1 - b2 ** t) / (1 - b1 ** t)
    if op in ("adamw", "adam"):
        getattr(lib, f"metal_kan_{op}_step")(P(p), P(g), P(m), P(v), lr, b1, b2, eps, wd, lr_t, n)
        rp, rm, rv = O.optim_update(op, p0, g, m0, v0, lr=lr, beta1=b1, beta2=b2, eps=eps,
                                    weight_decay=wd, lr_t=lr_t)
        np.testing.assert_allclose(v, rv, rtol=1e-6, atol=2 * np.spacing(np.float32(rv.max())))
    elif op.startswith("sgd"):
        nest = op.endswith("nesterov")
        lib.metal_kan_sgd_step(P(p), P(g), P(m), 0.01, 0.9, wd, int(nest), n)
        rp, rm, _ = O.optim_update("sgd", p0, g, m0, lr=0.01, beta1=0.9, weight_decay=wd,
                                   nesterov=nest)
    else:
        lib.metal_kan_lion_step(P(p), P(g), P(m), 1e-4, 0.9, 0.99, wd, n)
        rp, rm, _ = O.optim_update("lion", p0, g, m0, lr=1e-4, beta1=0.9, beta2=0.99,
                                   weight_decay=wd)
    np.testing.assert_allclose(m, rm, rtol=1e-6, atol=2 * np.spacing(np.float32(np.abs(rm).max())))
    # the step itself (p - p0) to fp32 rounding of p
    np.testing.assert_allclose(p, rp, rtol=0, atol=2 * np.spacing(np.abs(p0)).max())


@pytest.mark.parametrize("basis,K", [("cheby", 5), ("rbf", 8), ("bspline", 8)])
def test_fused_train_step_matches_composed_step(mk, basis, K):
    """train_step == forward + MSE gradient + backward + AdamW from the layer API, bit for bit,
    over three steps."""
    a = make_layer(basis, 24, 18, K, seed=3)
    b = make_layer(basis, 24, 18, K, seed=3)
    rng = np.random.default_rng(5)
    x = rng.uniform(-1.1, 1.1, (70, 24)).astype(np.float32)
    target = rng.normal(0, 1, (70, 18)).astype(np.float32)
    hyper = dict(lr=3e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01)
    b.forward(x)
    b.backward(np.zeros((70, 18), np.float32))  # allocate the gradient arrays
    opt = mk.optim.AdamW(b.parameters(), lr=hyper["lr"], betas=(0.9, 0.999), eps=1e-8,
                         weight_decay=0.01)
    lib = mk.get_metal_bridge()
    for _ in range(3):
        a.train_step(x, target, **hyper)
        y = b.forward(x)
        dY = np.empty_like(y)
        lib.metal_kan_calc_mse_loss_backward(P(y), P(target), P(dY), y.size, 2.0 / 70)
        b.backward(dY)
        opt.step()
    for name in (a.MAIN, "w_base", "bias"):
        np.testing.assert_array_equal(getattr(a, name), getattr(b, name), err_msg=name)


@pytest.mark.parametrize("basis,K", [("cheby", 6), ("rbf", 8), ("bspline", 8)])
def test_fused_train_step_vs_oracle(mk, basis, K):
    """One AdamW step of the fused train_step against the float64 oracle step."""
    layer = make_layer(basis, 20, 12, K, seed=8)
    rng = np.random.default_rng(8)
    x = rng.uniform(-1.3, 1.3, (64, 20)).astype(np.float32)
    target = rng.normal(0, 1, (64, 12)).astype(np.float32)
    W0, Wb0, b0 = (np.array(getattr(layer, n), np.float64) for n in (layer.MAIN, "w_base", "bias"))
    kw = {}
    if basis == "rbf":
        kw = dict(grid=np.asarray(layer.grid, np.float64), inv_den=layer.inv_denominator)
    elif basis == "bspline":
        kw = dict(grid_size=layer.grid_size, grid_min=float(layer.grid[0]), inv_h=float(layer.grid[1]))
    ob = {"cheby": "cheby", "rbf": "rbf", "bspline": "bspline"}[basis]
    y = O.kan_layer(x, ob, "f32", W0, Wb0, b0, K=K, out_round=False, round_weights=False, **kw)
    dY = O.mse_grad(y, target)
    _, dW, dWb, db = O.kan_layer_backward(x, dY, ob, W0, Wb0, K=K, **kw)
    lr, b1, b2, eps, wd = 1e-2, 0.9, 0.999, 1e-8, 0.01
    lr_t = lr * math.sqrt(1 - b2) / (1 - b1)
    layer.train_step(x, target, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd)
    for name, p0, g in ((layer.MAIN, W0, dW), ("w_base", Wb0, dWb), ("bias", b0, db)):
        rp, _, _ = O.optim_update("adamw", p0, g, np.zeros_like(p0), np.zeros_like(p0), lr=lr,
                                  beta1=b1, beta2=b2, eps=eps, weight_decay=wd, lr_t=lr_t)
        got = np.asarray(getattr(layer, name), np.float64) - p0
        want = rp - p0
        # at step 1 AdamW moves each weight by ~lr * sign(g): compare where the gradient is
        # clearly nonzero (elsewhere its sign is decided by rounding noise)
        sel = np.abs(g) > 1e-3 * np.abs(g).max()
        assert sel.mean() > 0.5
        np.testing.assert_allclose(got[sel], want[sel], rtol=1e-3, atol=1e-7, err_msg=name)


def test_optimizer_updates_reach_the_device(mk):
    """After optim.SGD steps the layer's next forward uses the updated host arrays."""
    np.random.seed(2)
    layer = mk.ChebyKAN(16, 8, degree=4)
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, (32, 16)).astype(np.float32)
    layer.forward(x)
    layer.backward(rng.normal(0, 1, (32, 8)).astype(np.float32))
    opt = mk.optim.SGD(layer.parameters(), lr=0.1, momentum=0.9)
    opt.step()
    y = layer.forward(x)
    ref = O.kan_layer(x, "cheby", "f32", layer.w_cheby, layer.w_base, layer.bias, K=4)
    assert O.max_rel_err(y, ref) <= 1e-5


@pytest.mark.parametrize("opt_name", ["AdamW", "Adam", "SGD", "Lion"])
def test_metalkan_training_reduces_loss(mk, opt_name):
    np.random.seed(0)
    net = mk.MetalKAN([6, 16, 3], basis_type="cheby", degree=4)
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (256, 6)).astype(np.float32)
    target = np.stack([np.sin(2 * x[:, 0]), x[:, 1] * x[:, 2], np.cos(x[:, 3])], 1).astype(np.float32)
    net(x)
    net.backward(np.zeros((256, 3), np.float32))
    kw = {"AdamW": dict(lr=1e-2), "Adam": dict(lr=1e-2), "SGD": dict(lr=0.02, momentum=0.9),
          "Lion": dict(lr=3e-3)}[opt_name]
    opt = getattr(mk.optim, opt_name)(net.parameters(), **kw)
    step = mk.build_train_step(net, opt)
    loss0 = float(((net(x) - target) ** 2).mean())
    for _ in range(30):
        step(x, target)
    loss1 = float(((net(x) - target) ** 2).mean())
    assert loss1 < 0.8 * loss0, (loss0, loss1)


def test_single_layer_net_uses_fused_step(mk):
    np.random.seed(1)
    net = mk.MetalKAN([8, 4], basis_type="fastkan", degree=6)
    rng = np.random.default_rng(1)
    x = rng.uniform(-1, 1, (128, 8)).astype(np.float32)
    target = rng.normal(0, 0.5, (128, 4)).astype(np.float32)
    loss0 = float(((net(x) - target) ** 2).mean())
    for _ in range(40):
        net.train_step(x, target, lr=1e-2)
    assert float(((net(x) - target) ** 2).mean()) < loss0
    assert net.layers[0]._fused_opt_state["step"] == 40
