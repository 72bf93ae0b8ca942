"""GPU: the tensor-core kernel's bounded-wait abort path.

Every pipeline wait of the kernel (a stage filled or freed by another warp role) has a limit; on
expiry the kernel sets the device error word, skips its remaining work, still waits (with the
full limit) for every copy and MMA it has in flight, joins every CTA and cluster barrier and
frees its TMEM.  kan_set_wait_limit() shortens the pipeline waits to a few hundred cycles, so the
MMA warp gives up on the first basis tile long before the producers can deliver it: the call must
report KAN_ERR_DEVICE_TIMEOUT, and the next call with the default limit must run normally and
match the oracle (the context stays usable).  Nothing here faults or hangs a GPU: every wait is
bounded, and no wait is left to run without a limit.
"""
import numpy as np
import pytest

from kan_cases import TOL, layer_err, make_layer, set_mode

pytestmark = pytest.mark.gpu

TC = 2

# (basis, mode, D_in, D_out, K, B, input map, expected (BN, splits))
CASES = [
    ("rbf", "f16", 256, 256, 8, 512, "layernorm", (256, 4)),    # cluster split-K, staged LN tile
    ("cheby", "bf16", 512, 512, 9, 8192, "none", (512, 2)),    # wide tiles, two-round reduction
    ("cheby", "bf16", 256, 256, 5, 16384, "none", (256, 1)),   # one CTA per tile, no cluster
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[1]}-{c[2]}x{c[3]}-B{c[5]}")
def test_short_wait_limit_aborts_and_recovers(case):
    import ctypes

    import metal_kans as mk
    from metal_kans.device import KanError

    basis, mode, d_in, d_out, K, B, imap, (bn, splits) = case
    layer = set_mode(make_layer(basis, d_in, d_out, K, input_map=imap, seed=3), mode)
    x = np.random.default_rng(5).normal(0, 1, (B, d_in)).astype(np.float32)
    lib = mk.get_metal_bridge()
    keep = []
    info = (ctypes.c_int * 6)()
    lib.kan_forward_plan(ctypes.byref(layer._descriptor(keep)), B, TC, info)
    assert (info[0], info[1], info[2]) == (TC, bn, splits), list(info)

    lib.kan_set_wait_limit(200)
    try:
        with pytest.raises(KanError, match="bounded wait"):
            layer.forward(x, path=TC)
    finally:
        lib.kan_set_wait_limit(0)
    code = ctypes.c_int(0)
    lib.kan_device_error(ctypes.byref(code))
    assert code.value == 0  # reading the error word cleared it

    y = layer.forward(x, path=TC)
    lib.kan_device_error(ctypes.byref(code))
    assert code.value == 0
    err = layer_err(y, layer, x, mode, basis)
    assert err <= TOL[mode], f"after the aborted call: max-rel-err {err:.3e}"
