"""GPU, two or more devices: one process runs tensor-core layers on device 0, then device 1, then
device 0 again (kan_set_device).  Each kernel's dynamic shared-memory limit is raised once per
device, so the first launch on device 1 must still get it; every layer object is created after its
device is selected (device buffers belong to the device that allocated them).  Skipped with fewer
than two GPUs."""
import ctypes

import numpy as np
import pytest

from kan_cases import TOL, layer_err, make_layer, set_mode
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu

TC = 2


def _device_count():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("case", [("cheby", "bf16", 512, 512, 9, 4096), ("rbf", "f16", 256, 256, 8, 2048)],
                         ids=lambda c: f"{c[0]}-{c[1]}")
def test_tensor_core_layer_on_each_device(case):
    import metal_kans as mk

    basis, mode, d_in, d_out, K, B = case
    lib = mk.get_metal_bridge()
    start = ctypes.c_int(0)
    lib.kan_get_device(ctypes.byref(start))
    try:
        for dev in (0, 1, 0):
            lib.kan_set_device(dev)
            layer = set_mode(make_layer(basis, d_in, d_out, K, seed=dev + 1), mode)
            x = np.random.default_rng(dev).normal(0, 1, (B, d_in)).astype(O.act_dtype(mode))
            y = layer.forward(x, path=TC)
            err = layer_err(y, layer, x, mode, basis)
            assert err <= TOL[mode], f"device {dev}: max rel err {err:.3g}"
    finally:
        lib.kan_set_device(start.value)
