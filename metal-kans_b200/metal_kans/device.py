"""ctypes loader of the CUDA engine ``libkan_cuda.so`` (replaces the reference's Metal loader).

Same public functions as the reference's ``metal_kans/device.py``: ``get_metal_bridge()``,
``is_metal_available()``, ``set_async()``, ``sync()``.  Differences, by design:

* the library is built ahead of time (``python metal-kans_b200/build.py``), never on import;
* there is no CPU or Metal fallback -- without a CUDA device ``get_metal_bridge()`` raises;
* every exported function has an ``errcheck``: a negative status raises :class:`KanError`
  carrying ``kan_last_error()`` (the reference ignores its forward return codes).
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KAN_CUDA_LIB", os.path.join(_HERE, "_lib", "libkan_cuda.so"))

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()

vp = ctypes.c_void_p
i32 = ctypes.c_int
f32 = ctypes.c_float
i64 = ctypes.c_longlong
sz = ctypes.c_size_t


class KanError(RuntimeError):
    """A libkan_cuda call returned a negative status."""


class KanWeight(ctypes.Structure):
    """``kan_weight`` of include/kan_cuda.h."""

    _fields_ = [("format", ctypes.c_int32), ("group_size", ctypes.c_int32),
                ("padded_cols", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("data", vp), ("scales", vp), ("biases", vp), ("codebook", vp)]


class KanLayer(ctypes.Structure):
    """``kan_layer`` of include/kan_cuda.h."""

    _fields_ = [("basis", ctypes.c_int32), ("act_dtype", ctypes.c_int32),
                ("D_in", ctypes.c_int32), ("D_out", ctypes.c_int32), ("K", ctypes.c_int32),
                ("has_base", ctypes.c_int32), ("has_bias", ctypes.c_int32),
                ("input_map", ctypes.c_int32), ("wavelet_type", ctypes.c_int32),
                ("grid_size", ctypes.c_int32), ("inv_den", ctypes.c_float),
                ("grid_min", ctypes.c_float), ("inv_h", ctypes.c_float),
                ("ln_eps", ctypes.c_float), ("grid", vp), ("translation", vp),
                ("inv_scale", vp), ("bias", vp), ("w", KanWeight), ("wb", KanWeight),
                ("tc_weights", vp), ("alpha", ctypes.c_float), ("beta", ctypes.c_float)]


# enum values of include/kan_cuda.h
KAN_F32, KAN_F16, KAN_BF16 = 0, 1, 2
KAN_CHEBY, KAN_RBF, KAN_BSPLINE, KAN_WAVELET, KAN_RELU, KAN_FOURIER, KAN_JACOBI = range(7)
KAN_MAP_NONE, KAN_MAP_TANH, KAN_MAP_LAYERNORM = 0, 1, 2
KAN_W_DENSE, KAN_W_INT8, KAN_W_INT4, KAN_W_TERNARY, KAN_W_INT2 = 0, 1, 2, 3, 4
KAN_WFLAG_TERNARY_NO3 = 1
KAN_PATH_AUTO, KAN_PATH_SIMT, KAN_PATH_TC, KAN_PATH_GEMV, KAN_PATH_GEMV_CC = 0, 1, 2, 3, 4

# (name, restype, argtypes) of every exported symbol
SIGNATURES = [
    ("kan_last_error", ctypes.c_char_p, []),
    ("kan_abi_version", i32, []),
    ("kan_launch_count", i64, []),
    ("metal_kan_init", i32, [ctypes.c_char_p]),
    ("metal_kan_set_async", i32, [i32]),
    ("metal_kan_sync", i32, []),
    ("metal_kan_cheby_forward", i32, [vp] * 5 + [i32] * 6),
    ("metal_kan_cheby_forward_fp16", i32, [vp] * 5 + [i32] * 6),
    ("metal_kan_fastkan_forward", i32, [vp] * 6 + [i32] * 4 + [f32, i32, i32]),
    ("metal_kan_fastkan_forward_fp16", i32, [vp] * 6 + [i32] * 4 + [f32, i32, i32]),
    ("metal_kan_bspline_forward", i32, [vp] * 6 + [i32] * 7),
    ("metal_kan_bspline_forward_fp16", i32, [vp] * 6 + [i32] * 7),
    ("metal_kan_wavkan_forward", i32, [vp] * 7 + [i32] * 7),
    ("metal_kan_wavkan_forward_fp16", i32, [vp] * 7 + [i32] * 7),
    ("metal_kan_chain_pipeline_cheby", i32,
     [vp, vp, i32, i32, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(vp),
      ctypes.POINTER(vp), ctypes.POINTER(vp)]),
    ("metal_kan_swiglu_forward", i32, [vp, vp, vp, i32]),
    ("metal_kan_quantize_int8", i32, [vp] * 4 + [i32, i32]),
    ("metal_kan_quantize_int4", i32, [vp] * 4 + [i32, i32]),
    ("metal_kan_dequantize_int8", i32, [vp] * 4 + [i32, i32]),
    ("metal_kan_dequantize_int4", i32, [vp] * 4 + [i32, i32]),
    ("metal_kan_quantize_ternary", i32, [vp] * 3 + [i32] * 3),
    ("metal_kan_quantize_int2", i32, [vp] * 4 + [i32] * 3),
    ("metal_kan_dequantize_ternary", i32, [vp] * 3 + [i32] * 3),
    ("metal_kan_dequantize_int2", i32, [vp] * 4 + [i32] * 3),
    ("metal_kan_forward_ternary_cheby", i32, [vp] * 5 + [i32] * 6),
    ("metal_kan_forward_int2_cheby", i32, [vp] * 6 + [i32] * 6),
    ("benchmark_metal_cheby", ctypes.c_double, [vp] * 5 + [i32] * 8),
    ("benchmark_metal_fastkan", ctypes.c_double, [vp] * 6 + [i32] * 4 + [f32] + [i32] * 4),
    ("benchmark_metal_bspline", ctypes.c_double, [vp] * 6 + [i32] * 9),
    ("benchmark_metal_wavkan", ctypes.c_double, [vp] * 7 + [i32] * 9),
    ("kan_forward", i32, [ctypes.POINTER(KanLayer), vp, vp, i32, vp]),
    ("kan_forward_path", i32, [ctypes.POINTER(KanLayer), vp, vp, i32, i32, vp]),
    ("kan_forward_plan", i32, [ctypes.POINTER(KanLayer), i32, i32, ctypes.POINTER(i32)]),
    ("kan_backward", i32, [ctypes.POINTER(KanLayer), vp, vp, vp, vp, vp, vp, i32, vp]),
    ("kan_swiglu_backward", i32, [vp, vp, vp, vp, vp, i64, vp]),
    ("metal_kan_cheby_backward", i32, [vp] * 8 + [i32] * 6),
    ("metal_kan_cheby_backward_fused", i32, [vp] * 8 + [i32] * 6),
    ("metal_kan_fastkan_backward", i32, [vp] * 9 + [i32] * 4 + [f32] + [i32] * 2),
    ("metal_kan_bspline_backward", i32, [vp] * 8 + [i32] * 4 + [f32, f32] + [i32] * 2),
    ("metal_kan_swiglu_backward", i32, [vp] * 5 + [i32]),
    ("metal_kan_relu_backward", i32, [vp] * 9 + [i32] * 4 + [f32] + [i32] * 2),
    ("metal_kan_relu_forward", i32, [vp] * 6 + [i32] * 4 + [f32] + [i32] * 2),
    ("metal_kan_relu_forward_fp16", i32, [vp] * 6 + [i32] * 4 + [f32] + [i32] * 2),
    ("metal_kan_fourier_forward", i32, [vp] * 5 + [i32] * 6),
    ("metal_kan_fourier_forward_fp16", i32, [vp] * 5 + [i32] * 6),
    ("metal_kan_jacobi_forward", i32, [vp] * 5 + [i32] * 4 + [f32, f32] + [i32] * 2),
    ("metal_kan_jacobi_forward_fp16", i32, [vp] * 5 + [i32] * 4 + [f32, f32] + [i32] * 2),
    ("benchmark_metal_relu", ctypes.c_double, [vp] * 6 + [i32] * 4 + [f32] + [i32] * 4),
    ("benchmark_metal_fourier", ctypes.c_double, [vp] * 5 + [i32] * 8),
    ("benchmark_metal_jacobi", ctypes.c_double, [vp] * 5 + [i32] * 4 + [f32, f32] + [i32] * 4),
    ("metal_kan_mult_forward", i32, [vp] * 6 + [i32] * 6 + [f32] + [i32] * 2),
    ("metal_kan_mult_forward_fp16", i32, [vp] * 6 + [i32] * 6 + [f32] + [i32] * 2),
    ("metal_kan_lowrank_forward", i32, [vp] * 7 + [i32] * 5 + [f32] + [i32] * 2),
    ("metal_kan_lowrank_forward_fp16", i32, [vp] * 7 + [i32] * 5 + [f32] + [i32] * 2),
    ("metal_kan_rational_forward", i32, [vp] * 6 + [i32] * 7),
    ("benchmark_metal_mult", ctypes.c_double, [vp] * 6 + [i32] * 6 + [f32] + [i32] * 4),
    ("benchmark_metal_lowrank", ctypes.c_double, [vp] * 7 + [i32] * 5 + [f32] + [i32] * 4),
    ("benchmark_metal_rational", ctypes.c_double, [vp] * 6 + [i32] * 9),
    ("kan_set_wait_limit", i32, [i64]),
    ("kan_forward_host", i32, [ctypes.POINTER(KanLayer), vp, vp, i32]),
    ("kan_gated_forward", i32, [ctypes.POINTER(KanLayer)] * 3 + [vp, vp, vp, i32, vp]),
    ("kan_gated_forward_pair", i32, [ctypes.POINTER(KanLayer)] * 3 + [vp, vp, vp, vp, i32, vp]),
    ("kan_tc_pair_bytes", i32, [ctypes.POINTER(KanLayer), ctypes.POINTER(KanLayer),
                                ctypes.POINTER(ctypes.c_size_t)]),
    ("kan_tc_pack_pair", i32, [ctypes.POINTER(KanLayer), ctypes.POINTER(KanLayer), vp, vp]),
    ("kan_gated_forward_noalloc", i32, [ctypes.POINTER(KanLayer)] * 3 + [vp, vp, vp, i32, vp]),
    ("kan_tc_packed_bytes", i32, [ctypes.POINTER(KanLayer), ctypes.POINTER(sz)]),
    ("kan_tc_pack", i32, [ctypes.POINTER(KanLayer), vp, vp]),
    ("kan_dequantize", i32, [ctypes.POINTER(KanWeight), i32, i32, vp, i32, vp]),
    ("kan_swiglu", i32, [vp, vp, vp, i64, i32, vp]),
    ("kan_mult_combine", i32, [vp, vp, i32, i32, i32, i32, vp]),
    ("kan_train_step", i32, [vp] * 3 + [i32] + [vp] * 6 + [i32, vp, i32, vp]),
    ("kan_optim_step", i32, [i32] + [vp] * 4 + [i64, vp, i32, vp]),
    ("metal_kan_adamw_step", i32, [vp] * 4 + [f32] * 6 + [i32]),
    ("metal_kan_adam_step", i32, [vp] * 4 + [f32] * 6 + [i32]),
    ("metal_kan_sgd_step", i32, [vp] * 3 + [f32] * 3 + [i32, i32]),
    ("metal_kan_lion_step", i32, [vp] * 3 + [f32] * 4 + [i32]),
    ("metal_kan_calc_mse_loss_backward", i32, [vp] * 3 + [i32, f32]),
    ("metal_kan_cheby_train_step", i32, [vp] * 11 + [i32] * 6 + [f32] * 6),
    ("metal_kan_fastkan_train_step", i32, [vp] * 12 + [i32] * 4 + [f32] + [i32] * 2 + [f32] * 6),
    ("metal_kan_bspline_train_step", i32, [vp] * 11 + [i32] * 4 + [f32] * 2 + [i32] * 2 + [f32] * 6),
    ("kan_lowrank_up", i32, [vp] * 6 + [i32] * 7 + [vp]),
    ("kan_rational_forward", i32, [vp] * 6 + [i32] * 7 + [vp]),
    ("kan_convert", i32, [vp, i32, vp, i32, i64, vp]),
    ("kan_device_count", i32, [ctypes.POINTER(i32)]),
    ("kan_set_device", i32, [i32]),
    ("kan_get_device", i32, [ctypes.POINTER(i32)]),
    ("kan_malloc", i32, [ctypes.POINTER(vp), sz]),
    ("kan_free", i32, [vp]),
    ("kan_host_alloc", i32, [ctypes.POINTER(vp), sz]),
    ("kan_host_free", i32, [vp]),
    ("kan_memcpy", i32, [vp, vp, sz, i32, vp]),
    ("kan_memset", i32, [vp, i32, sz, vp]),
    ("kan_stream_synchronize", i32, [vp]),
    ("kan_default_stream", vp, []),
    ("kan_device_error", i32, [ctypes.POINTER(i32)]),
]

_NO_CHECK = {"kan_last_error", "kan_abi_version", "kan_launch_count", "kan_default_stream"}


def _errcheck_int(lib):
    def check(result, func, args):
        if result != 0:
            msg = lib.kan_last_error().decode(errors="replace")
            raise KanError(f"{func.__name__} returned {result}: {msg}")
        return result
    return check


def _errcheck_double(lib):
    def check(result, func, args):
        if result < 0:
            msg = lib.kan_last_error().decode(errors="replace")
            raise KanError(f"{func.__name__} failed: {msg}")
        return result
    return check


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """dlopen the engine and declare every symbol (no device initialisation)."""
    if not os.path.exists(path):
        raise KanError(f"{path} is missing: build it with `python metal-kans_b200/build.py`")
    lib = ctypes.CDLL(path)
    chk_i, chk_d = _errcheck_int(lib), _errcheck_double(lib)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
        if name in _NO_CHECK:
            continue
        fn.errcheck = chk_d if res is ctypes.c_double else chk_i
    return lib


def get_metal_bridge() -> ctypes.CDLL:
    """Return the loaded CUDA engine (the reference's name for its loaded bridge).

    Initialises the current CUDA device on first use; raises :class:`KanError` when the
    library is missing or no CUDA device is visible.
    """
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            lib = load_library()
            lib.metal_kan_init(None)
            _lib = lib
    return _lib


def is_metal_available() -> bool:
    """True when the engine loads and a CUDA device is visible (name kept for drop-in use)."""
    try:
        lib = get_metal_bridge()
        n = i32(0)
        lib.kan_device_count(ctypes.byref(n))
        return n.value > 0
    except Exception:
        return False


is_cuda_available = is_metal_available

_async = threading.local()


def async_enabled() -> bool:
    return getattr(_async, "on", False)


def set_async(enabled: bool) -> None:
    """Async mode: forwards enqueue and return; results are complete after :func:`sync`."""
    lib = get_metal_bridge()
    if not enabled:
        sync()
    _async.on = bool(enabled)
    lib.metal_kan_set_async(1 if enabled else 0)


def sync() -> None:
    """Wait for all queued work and complete pending result copies."""
    lib = get_metal_bridge()
    lib.metal_kan_sync()
    from . import _engine

    _engine.flush_pending()
