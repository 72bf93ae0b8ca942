"""GPU: the split-K fp32 kernel of the CUDA-core path (dense fp32 layers of >= 256 rows with short
K, BASELINE config 1's shape): 64 x 64 output tiles, the input features split over a
thread-block cluster of S CTAs whose partial tiles are summed through distributed shared memory
in rank order.  Outputs against the oracle at the fp32 tolerance (1e-5), the plan's cluster size,
and bit-identical repeated calls (a fixed summation order)."""
import ctypes

import numpy as np
import pytest

from kan_cases import TOL, layer_err, make_layer, randomize_bias
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu

SIMT = 1

# (basis, D_in, D_out, K, B, base, bias, input map, expected cluster size)
CASES = [
    ("cheby", 64, 64, 9, 1024, False, False, "tanh", 8),
    ("rbf", 48, 100, 8, 700, True, True, "layernorm", 8),      # ragged rows and columns
    ("bspline", 30, 64, 8, 256, True, False, "none", 8),       # last CTAs' slices short
    ("wavelet", 40, 200, 6, 2048, True, True, "none", 2),      # 128 tiles: two splits
    ("cheby", 256, 64, 4, 512, True, True, "none", 8),
    ("fourier", 16, 64, 9, 300, False, True, "none", 8),
    ("relu", 64, 33, 8, 256, True, True, "none", 8),
]


def _splits(mk, layer, B):
    keep = []
    info = (ctypes.c_int * 6)()
    mk.get_metal_bridge().kan_forward_plan(ctypes.byref(layer._descriptor(keep)), B, 0, info)
    assert info[0] == SIMT, list(info)
    return info[2]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c[:5])))
def test_splitk_matches_oracle(case):
    import metal_kans as mk

    basis, d_in, d_out, K, B, base, bias, imap, S = case
    layer = make_layer(basis, d_in, d_out, K, bias=bias, use_base=base, input_map=imap,
                       seed=d_in + B)
    if bias:
        randomize_bias(layer)
    assert _splits(mk, layer, B) == S
    x = np.random.default_rng(B).uniform(-1.2, 1.2, (B, d_in)).astype(np.float32)
    y = layer.forward(x)
    err = layer_err(y, layer, x, "f32", basis)
    assert err <= TOL["f32"], f"max rel err {err:.3g}"
    np.testing.assert_array_equal(layer.forward(x), y)


def test_small_batches_keep_the_tile_kernel():
    """Below 256 rows (and for packed weights) the tile kernels run, as before."""
    import metal_kans as mk

    layer = make_layer("cheby", 64, 64, 9, bias=False, use_base=False, seed=1)
    assert _splits(mk, layer, 128) == 0
    x = np.random.default_rng(2).uniform(-1, 1, (128, 64)).astype(np.float32)
    err = layer_err(layer.forward(x), layer, x, "f32", "cheby")
    assert err <= TOL["f32"], f"max rel err {err:.3g}"
