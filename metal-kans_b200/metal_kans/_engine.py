"""Host-side engine plumbing shared by the layer classes.

* :class:`DeviceBuffer` -- device memory owned through the C ABI (``kan_malloc``/``kan_free``);
* :class:`DeviceLayerMixin` -- read-only NumPy weights mirrored on the device: assigning a weight
  attribute bumps its version and the next forward re-uploads it; in-place writes are refused
  (the arrays are read-only), so a stale device copy can never be used;
* dtype helpers (f32 / f16 / bf16 via ``ml_dtypes``) and the async result queue.
"""
from __future__ import annotations

import ctypes
import threading
import weakref
from typing import Dict, Optional, Tuple

import numpy as np

from . import device as D

try:
    import ml_dtypes

    BFLOAT16 = np.dtype(ml_dtypes.bfloat16)
except Exception:  # pragma: no cover - ml_dtypes is part of the image
    BFLOAT16 = None

_KAN_DTYPE = {np.dtype(np.float32): D.KAN_F32, np.dtype(np.float16): D.KAN_F16}
if BFLOAT16 is not None:
    _KAN_DTYPE[BFLOAT16] = D.KAN_BF16


def kan_dtype(dt) -> int:
    dt = np.dtype(dt)
    if dt not in _KAN_DTYPE:
        raise TypeError(f"unsupported activation dtype {dt}")
    return _KAN_DTYPE[dt]


def lib():
    return D.get_metal_bridge()


class DeviceBuffer:
    """A device allocation made through the engine; freed with the object."""

    __slots__ = ("ptr", "nbytes", "_lib")

    def __init__(self, nbytes: int):
        self._lib = lib()
        p = ctypes.c_void_p()
        self._lib.kan_malloc(ctypes.byref(p), max(int(nbytes), 16))
        self.ptr = p.value
        self.nbytes = int(nbytes)

    def __del__(self):
        try:
            if self.ptr:
                self._lib.kan_free(ctypes.c_void_p(self.ptr))
        except Exception:
            pass
        self.ptr = None

    def upload(self, arr: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(arr)
        assert a.nbytes <= self.nbytes
        if a.nbytes:
            self._lib.kan_memcpy(ctypes.c_void_p(self.ptr), ctypes.c_void_p(a.ctypes.data),
                                 a.nbytes, 1, None)
        return self

    def download(self, out: np.ndarray) -> np.ndarray:
        assert out.flags["C_CONTIGUOUS"] and out.nbytes <= self.nbytes
        if out.nbytes:
            self._lib.kan_memcpy(ctypes.c_void_p(out.ctypes.data), ctypes.c_void_p(self.ptr),
                                 out.nbytes, 2, None)
        return out

    @classmethod
    def from_array(cls, arr: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(arr)
        return cls(a.nbytes).upload(a)


class _Scratch:
    """Grow-only device buffers keyed by role, reused across calls of one layer/net."""

    def __init__(self):
        self._bufs: Dict[str, DeviceBuffer] = {}

    def get(self, key: str, nbytes: int) -> DeviceBuffer:
        b = self._bufs.get(key)
        if b is None or b.nbytes < nbytes:
            b = DeviceBuffer(max(nbytes, 256))
            self._bufs[key] = b
        return b


# ---------------------------------------------------------------------------------------------
# async results (set_async): D2H into pinned memory, copied out by device.sync()
# ---------------------------------------------------------------------------------------------
_pending = []


class _Pinned:
    def __init__(self, nbytes):
        self._lib = lib()
        p = ctypes.c_void_p()
        self._lib.kan_host_alloc(ctypes.byref(p), max(nbytes, 16))
        self.ptr = p.value
        self.nbytes = nbytes

    def __del__(self):
        try:
            self._lib.kan_host_free(ctypes.c_void_p(self.ptr))
        except Exception:
            pass


# ---------------------------------------------------------------------------------------------
# results in pinned host memory: a device->host copy into pageable memory goes through the
# driver's staging buffers at a fraction of the link rate, so forward() returns arrays backed by
# page-locked buffers from a small pool (a buffer goes back to the pool when its array dies)
# ---------------------------------------------------------------------------------------------
_PIN_MIN = 1 << 16            # smaller results stay in ordinary memory
_PIN_POOL_BYTES = 1 << 30     # pooled (idle) page-locked bytes kept for reuse
_pin_pool: Dict[int, list] = {}
_pin_pool_bytes = 0
_pin_lock = threading.Lock()


def _pin_take(nbytes: int) -> "_Pinned":
    size = 1 << max(16, (int(nbytes) - 1).bit_length())
    with _pin_lock:
        lst = _pin_pool.get(size)
        if lst:
            global _pin_pool_bytes
            _pin_pool_bytes -= size
            return lst.pop()
    return _Pinned(size)


def _pin_give(buf: "_Pinned") -> None:
    global _pin_pool_bytes
    with _pin_lock:
        if _pin_pool_bytes + buf.nbytes <= _PIN_POOL_BYTES:
            _pin_pool.setdefault(buf.nbytes, []).append(buf)
            _pin_pool_bytes += buf.nbytes
            return
    del buf  # over the pool's budget: freed


class _PinnedOwner:
    """Base object of a pinned result array: holds the buffer, returns it to the pool."""

    def __init__(self, buf: "_Pinned", shape, dtype):
        self._buf = buf
        self.__array_interface__ = {"data": (buf.ptr, False), "shape": tuple(shape),
                                    "typestr": "|V%d" % np.dtype(dtype).itemsize, "version": 3}

    def __del__(self):
        try:
            _pin_give(self._buf)
        except Exception:
            pass


def pinned_empty(shape, dtype) -> np.ndarray:
    """np.empty(shape, dtype) in page-locked memory when the result is large enough to matter."""
    dtype = np.dtype(dtype)
    nbytes = int(np.prod(shape)) * dtype.itemsize
    if nbytes < _PIN_MIN:
        return np.empty(shape, dtype)
    return np.asarray(_PinnedOwner(_pin_take(nbytes), shape, dtype)).view(dtype)


def fetch(dev: DeviceBuffer, out: np.ndarray) -> np.ndarray:
    """Copy a device result into ``out``: now, or after ``sync()`` in async mode."""
    L = lib()
    if not D.async_enabled():
        dev.download(out)
        L.kan_stream_synchronize(None)
        code = ctypes.c_int(0)
        L.kan_device_error(ctypes.byref(code))
        if code.value:
            raise D.KanError(f"a kernel's bounded wait expired (device error {code.value})")
        return out
    pin = _Pinned(out.nbytes)
    if out.nbytes:
        L.kan_memcpy(ctypes.c_void_p(pin.ptr), ctypes.c_void_p(dev.ptr), out.nbytes, 2, None)
    _pending.append((pin, out, dev))
    return out


def flush_pending() -> None:
    L = lib()
    L.kan_stream_synchronize(None)
    while _pending:
        pin, out, _dev = _pending.pop(0)
        if out.nbytes:
            ctypes.memmove(out.ctypes.data, pin.ptr, out.nbytes)


# ---------------------------------------------------------------------------------------------
# layers: read-only weights mirrored on the device
# ---------------------------------------------------------------------------------------------
_PARAM_OWNERS: dict = {}


def param_updated(arr) -> None:
    """Tell the layer owning weight array ``arr`` (as handed out by its parameters()) that the
    array was changed in place: its device copy is refreshed before the next forward."""
    ent = _PARAM_OWNERS.get(id(arr))
    if ent is None:
        return
    owner = ent[0]()
    if owner is not None and getattr(owner, ent[1], None) is arr:
        owner._bump(ent[1])


class DeviceLayerMixin:
    """Weight attributes named in ``_WEIGHTS`` are stored read-only and mirrored on the device."""

    _WEIGHTS: Tuple[str, ...] = ()

    def __setattr__(self, name, value):
        if not name.startswith("_"):
            # any public assignment (a weight, a basis parameter, a flag) invalidates the cached
            # kernel descriptor
            d = self.__dict__
            d["_pver"] = d.get("_pver", 0) + 1
        if name in type(self)._WEIGHTS and isinstance(value, np.ndarray):
            v = np.array(value, order="C", copy=True)
            v.flags.writeable = False
            object.__setattr__(self, name, v)
            vers = self.__dict__.setdefault("_versions", {})
            vers[name] = vers.get(name, 0) + 1
            return
        object.__setattr__(self, name, value)

    def _version(self, name: str) -> int:
        return self.__dict__.get("_versions", {}).get(name, 0)

    def _bump(self, name: str) -> None:
        """The host array of weight ``name`` was changed in place (an optimiser step): a new
        version, so that the device copies and packed weights of the old one are not used."""
        vers = self.__dict__.setdefault("_versions", {})
        vers[name] = vers.get(name, 0) + 1
        self.__dict__["_pver"] = self.__dict__.get("_pver", 0) + 1

    def _register_param(self, name: str):
        """The weight array of ``name``, recorded so that an optimiser can report in-place
        updates of it (parameters() of the layers)."""
        arr = getattr(self, name)
        _PARAM_OWNERS[id(arr)] = (weakref.ref(self), name)
        return arr

    def _dev(self, name: str, dtype=None) -> DeviceBuffer:
        """Device copy of weight ``name`` (optionally cast to ``dtype``), uploaded when stale."""
        cache = self.__dict__.setdefault("_dev_cache", {})
        arr = getattr(self, name)
        key = (name, None if dtype is None else np.dtype(dtype).str)
        ver = self._version(name)
        hit = cache.get(key)
        if hit is not None and hit[0] == ver:
            return hit[1]
        a = arr if dtype is None else np.asarray(arr).astype(dtype)
        buf = DeviceBuffer.from_array(a)
        cache[key] = (ver, buf)
        return buf

    def _dev_array(self, key: str, arr: np.ndarray, ver_key: Optional[str] = None) -> DeviceBuffer:
        """Device copy of a derived array, cached under ``key`` until ``ver_key`` changes."""
        cache = self.__dict__.setdefault("_dev_cache", {})
        ver = self._version(ver_key) if ver_key else 0
        hit = cache.get(("derived", key))
        if hit is not None and hit[0] == ver:
            return hit[1]
        buf = DeviceBuffer.from_array(np.ascontiguousarray(arr))
        cache[("derived", key)] = (ver, buf)
        return buf

    def _scratch(self) -> _Scratch:
        s = self.__dict__.get("_scratch_bufs")
        if s is None:
            s = _Scratch()
            object.__setattr__(self, "_scratch_bufs", s)
        return s


def as_activation(x, dtype, d_in: int) -> Tuple[np.ndarray, tuple]:
    """Cast ``x`` to the layer dtype, flatten leading dims, make C-contiguous
    (reference forward prologue, e.g. cheby_kan.py:97-113)."""
    if not isinstance(x, np.ndarray) or x.dtype != dtype:
        x = np.asarray(x).astype(dtype)
    orig = x.shape
    if x.ndim > 2:
        x = x.reshape(-1, d_in)
    if x.ndim == 1:
        x = x.reshape(1, -1)
    if not x.flags["C_CONTIGUOUS"]:
        x = np.ascontiguousarray(x)
    if x.shape[1] != d_in:
        raise ValueError(f"Expected in_features={d_in}, got {x.shape[1]}")
    return x, orig


def restore_shape(y: np.ndarray, orig: tuple, d_out: int) -> np.ndarray:
    if len(orig) > 2:
        return y.reshape(*orig[:-1], d_out)
    return y
