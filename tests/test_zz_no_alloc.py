"""GPU: kan_gated_forward_noalloc, the GatedKAN entry point for callers that cannot allocate.

Callers inside a memory arena or a serving runtime that forbids cudaMalloc after start-up cannot
use kan_gated_forward(), which allocates its gate/up scratch on first use.  The no-allocation
variant keeps that scratch in a fixed device array; this test calls both through the C ABI on the
same layers and inputs and requires the same output, twice in a row (the second call sees the
first call's leftovers in the shared array), for an fp32 block and a bf16 block whose weights are
packed for the tensor cores.  The file sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest

from kan_cases import TOL
from oracle import kan_oracle as O

pytestmark = pytest.mark.gpu


def _run(mk, blk, fn, x):
    """Forward of a GatedKAN through a raw C-ABI entry point on device buffers."""
    from metal_kans._engine import DeviceBuffer

    lib = mk.get_metal_bridge()
    act = blk.gate_kan.dtype
    x2 = np.ascontiguousarray(np.asarray(x).astype(act))
    B = x2.shape[0]
    keep = []
    descs = [l._descriptor(keep) for l in (blk.gate_kan, blk.up_kan, blk.down_kan)]
    dx = DeviceBuffer.from_array(x2)
    dh = DeviceBuffer(B * blk.d_ffn * act.itemsize)
    dy = DeviceBuffer(B * blk.d_model * act.itemsize)
    getattr(lib, fn)(*(ctypes.byref(d) for d in descs), ctypes.c_void_p(dx.ptr),
                     ctypes.c_void_p(dh.ptr), ctypes.c_void_p(dy.ptr), B, None)
    y = np.empty((B, blk.d_model), act)
    dy.download(y)
    lib.kan_stream_synchronize(None)
    return y


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_noalloc_matches_gated_forward_twice(mode):
    import metal_kans as mk

    np.random.seed(21)
    blk = mk.GatedKAN(d_model=128, d_ffn=256, degree=5)
    if mode == "bf16":
        blk.bfloat16()
    rng = np.random.default_rng(5)
    for call in range(2):
        x = rng.normal(0, 1, (192 + 64 * call, 128)).astype(np.float32)
        ref = _run(mk, blk, "kan_gated_forward", x)
        got = _run(mk, blk, "kan_gated_forward_noalloc", x)
        assert got.dtype == ref.dtype and got.shape == ref.shape
        assert O.max_rel_err(got, ref) <= TOL[mode], f"call {call}"


def test_noalloc_rejects_oversized_batch():
    import metal_kans as mk

    from metal_kans._engine import DeviceBuffer

    np.random.seed(22)
    blk = mk.GatedKAN(d_model=64, d_ffn=4096, degree=4)  # fp32: 2 * B * 4096 * 4 bytes
    lib = mk.get_metal_bridge()
    keep = []
    descs = [l._descriptor(keep) for l in (blk.gate_kan, blk.up_kan, blk.down_kan)]
    B = 1025  # 2 * 1025 * 4096 * 4 > 32 MiB
    # real buffers of the full size, so that even a missed check could not read out of bounds
    dx, dh, dy = DeviceBuffer(B * 64 * 4), DeviceBuffer(B * 4096 * 4), DeviceBuffer(B * 64 * 4)
    with pytest.raises(mk.KanError, match="32 MiB"):
        lib.kan_gated_forward_noalloc(*(ctypes.byref(d) for d in descs), ctypes.c_void_p(dx.ptr),
                                      ctypes.c_void_p(dh.ptr), ctypes.c_void_p(dy.ptr), B, None)
    lib.kan_stream_synchronize(None)
