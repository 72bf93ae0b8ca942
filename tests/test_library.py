"""CPU: the C-ABI library loads, exports every symbol of include/kan_cuda.h, and its host
quantisers are bit-exact with the oracle (host code only -- no kernel runs here)."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO
from oracle import kan_oracle as O

HEADER = os.path.join(REPO, "include", "kan_cuda.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\*\s]+?\**\s*(\w+)\s*\(", src, flags=re.M))
                  - {"if", "defined"})


@pytest.fixture(scope="module")
def lib():
    from metal_kans.device import load_library

    return load_library()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 45
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_loader_declares_every_symbol():
    from metal_kans.device import SIGNATURES

    assert sorted(n for n, _, _ in SIGNATURES) == declared_functions()


def test_abi_version_and_errors(lib):
    assert lib.kan_abi_version() == 100
    from metal_kans.device import KanError

    with pytest.raises(KanError):
        lib.metal_kan_quantize_int8(None, None, None, None, 0, 0)


def _p(a):
    return a.ctypes.data


@pytest.mark.parametrize("bits", [8, 4])
def test_host_affine_quantiser_bit_exact(lib, bits):
    rng = np.random.default_rng(bits)
    for shape, gs in (((64, 576), 64), ((33, 100), 32), ((7, 130), 128)):
        w = rng.normal(0, 0.02, shape).astype(np.float32)
        qw, s, b, pin = O.quantize_affine(w, bits, gs, "bridge")
        padded = O._pad_rows(w, gs)
        G = padded.size // gs
        q = np.empty_like(qw)
        cs = np.empty((G, 1), np.float32)
        cb = np.empty((G, 1), np.float32)
        fn = lib.metal_kan_quantize_int8 if bits == 8 else lib.metal_kan_quantize_int4
        fn(_p(padded), _p(q), _p(cs), _p(cb), G, gs)
        np.testing.assert_array_equal(q, qw)
        np.testing.assert_array_equal(cs, s)
        np.testing.assert_array_equal(cb, b)
        out = np.empty((G, gs), np.float32)
        dq = lib.metal_kan_dequantize_int8 if bits == 8 else lib.metal_kan_dequantize_int4
        dq(_p(q), _p(cs), _p(cb), _p(out), G, gs)
        np.testing.assert_array_equal(out, O.dequantize_affine(qw, s, b, bits, gs))


def test_host_2bit_quantisers_bit_exact(lib):
    rng = np.random.default_rng(5)
    cbk = np.array([-1.0, -0.33333, 0.33333, 1.0], np.float32)
    for shape, gs in (((16, 576), 64), ((7, 100), 32), ((3, 37), 16)):
        w = rng.normal(0, 0.03, shape).astype(np.float32)
        D, Kd = shape
        words, G = (Kd + 15) // 16, (Kd + gs - 1) // gs
        P = np.empty((D, words), np.uint32)
        S = np.empty((D, G), np.float32)
        lib.metal_kan_quantize_ternary(_p(w), _p(P), _p(S), D, Kd, gs)
        p, s = O.quantize_ternary(w, gs)
        np.testing.assert_array_equal(P, p)
        np.testing.assert_array_equal(S, s)
        lib.metal_kan_quantize_int2(_p(w), _p(P), _p(S), _p(cbk), D, Kd, gs)
        p, s = O.quantize_int2(w, gs, cbk)
        np.testing.assert_array_equal(P, p)
        np.testing.assert_array_equal(S, s)
