"""Generate the committed golden fixtures from the REFERENCE's own Python code.

Run in the development container only (it needs the reference source tree):

    python tests/golden/make_goldens.py [--reference /path/to/metal-kans]

What is real reference code here and what is restated:

* quantisers / dequantisers: the reference's NumPy code paths in ``metal_kans/quantization.py``
  run unchanged (the stand-in bridge returns -1 so the reference falls back to them).  These
  fixtures pin the oracle's quantisers bit-exactly.
* layers: the reference's classes (``ChebyKAN``, ``FastKAN``, ``BSplineKAN``, ``WavKAN``,
  ``ReLUKAN``, ``FourierKAN``, ``JacobiKAN``, ``MultKAN``, ``LowRankKAN``, ``RationalKAN``,
  ``GatedKAN``, ``MetalKAN``) run unchanged -- construction, weight init order, ``.half()``,
  casts, reshapes, ``to_int*`` -- with the Metal/MPS arithmetic supplied by
  ``oracle/fake_bridge.py`` (the Metal kernels cannot run off macOS).

The fixtures are small (``.npz``).  The GPU tests compare the CUDA engine against them.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))


def _save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print("wrote", os.path.relpath(path, REPO), sum(a.nbytes for a in arrays.values()), "bytes")


def layer_goldens(mk):
    """Reference layer classes at the shapes of the reference's own tests (8 -> 16, seed 42)."""
    out = {}
    cases = [
        ("cheby_k4", lambda: mk.ChebyKAN(8, 16, degree=4), (-1.0, 1.0), 128),
        ("cheby_k8_nobias", lambda: mk.ChebyKAN(8, 16, degree=8, bias=False), (-1.2, 1.2), 64),
        ("cheby_k9_nobase", lambda: mk.ChebyKAN(8, 16, degree=9, use_base=False), (-1.0, 1.0), 64),
        ("fastkan_c8", lambda: mk.FastKAN(8, 16, num_centers=8), (-1.0, 1.0), 128),
        ("fastkan_c5_range2", lambda: mk.FastKAN(8, 16, num_centers=5, grid_range=(-2, 2)), (-2.5, 2.5), 64),
        ("bspline_g5", lambda: mk.BSplineKAN(8, 16, grid_size=5, spline_order=3), (-0.9, 0.9), 64),
        ("bspline_g5_outside", lambda: mk.BSplineKAN(8, 16, grid_size=5), (-1.7, 1.7), 64),
        ("wav_mexican", lambda: mk.WavKAN(8, 16, num_wavelets=6, wavelet_type="mexican_hat"), (-1.0, 1.0), 64),
        ("wav_morlet", lambda: mk.WavKAN(8, 16, num_wavelets=6, wavelet_type="morlet"), (-1.0, 1.0), 64),
        ("wav_dog", lambda: mk.WavKAN(8, 16, num_wavelets=6, wavelet_type="dog"), (-1.0, 1.0), 64),
        ("relu_g8", lambda: mk.ReLUKAN(8, 16, num_grids=8), (-1.2, 1.2), 64),
        ("relu_g5_range2", lambda: mk.ReLUKAN(8, 16, num_grids=5, grid_range=(-2, 2)), (-2.0, 2.0), 64),
        ("fourier_f4", lambda: mk.FourierKAN(8, 16, num_frequencies=4), (-1.0, 1.0), 64),
        ("fourier_f3_nobase", lambda: mk.FourierKAN(8, 16, num_frequencies=3, use_base=False), (-2.0, 2.0), 64),
        ("jacobi_d4", lambda: mk.JacobiKAN(8, 16, degree=4), (-1.2, 1.2), 64),
        ("jacobi_d6_ab", lambda: mk.JacobiKAN(8, 16, degree=6, alpha=0.5, beta=1.5), (-1.0, 1.0), 64),
        ("mult_g8", lambda: mk.MultKAN(8, 16, num_grids=8), (-1.0, 1.0), 64),
        ("mult_m3_nobias", lambda: mk.MultKAN(8, 16, num_mult=3, num_grids=5, bias=False), (-1.5, 1.5), 64),
        ("lowrank_r4", lambda: mk.LowRankKAN(8, 16, rank=4, num_grids=8), (-1.0, 1.0), 64),
        ("lowrank_r6_nobase", lambda: mk.LowRankKAN(8, 16, rank=6, num_grids=6, use_base=False), (-1.5, 1.5), 64),
        ("rational_p4q2", lambda: mk.RationalKAN(8, 16, p_degree=4, q_degree=2), (-1.3, 1.3), 64),
        ("rational_p6q3_nobias", lambda: mk.RationalKAN(8, 16, p_degree=6, q_degree=3, bias=False), (-1.0, 1.0), 64),
    ]
    for name, ctor, (lo, hi), B in cases:
        for mode in (("f32",) if name.startswith("rational") else ("f32", "f16")):
            np.random.seed(42)
            layer = ctor()
            x = np.random.uniform(lo, hi, (B, 8)).astype(np.float32)
            if mode == "f16":
                layer.half()
                xin = x.astype(np.float16)
            else:
                xin = x
            y = layer(xin)
            rec = {"x": xin, "y": y}
            for attr in ("w_cheby", "w_rbf", "w_spline", "w_wav", "w_relu", "w_fourier", "w_jacobi",
                         "w_down", "w_up", "w_p", "w_q", "w_base", "bias", "grid", "translation",
                         "_inv_scale"):
                if hasattr(layer, attr):
                    rec[attr.lstrip("_")] = np.asarray(getattr(layer, attr))
            meta = dict(has_base=layer.has_base, has_bias=layer.has_bias)
            for attr in ("degree", "num_centers", "inv_denominator", "grid_size", "num_wavelets",
                         "wavelet_type", "num_grids", "inv_h", "num_frequencies", "alpha", "beta",
                         "num_add", "num_mult", "rank", "p_degree", "q_degree"):
                if hasattr(layer, attr):
                    meta[attr] = getattr(layer, attr)
            for k, v in meta.items():
                rec["meta_" + k] = np.asarray(v)
            out[f"{name}_{mode}"] = rec
    flat = {f"{case}/{k}": v for case, rec in out.items() for k, v in rec.items()}
    _save("layers_small.npz", **flat)


def c1_golden(mk):
    """BASELINE config 1 at full size: ChebyKAN fp32, B=1024, 64 -> 64, T_0..T_8 of tanh(x).

    The reference counts terms in ``degree`` (T_0..T_8 = degree 9); tanh(x) is applied before the
    layer (the reference clamps to [-1, 1], the identity on tanh's range).  No base, no bias.
    """
    rng = np.random.default_rng(0)
    x = rng.uniform(-1.0, 1.0, (1024, 64)).astype(np.float32)
    W = rng.normal(0.0, np.sqrt(1.0 / (64 * 9)), (64, 64, 9)).astype(np.float32)
    layer = mk.ChebyKAN(64, 64, degree=9, bias=False, use_base=False)
    layer.w_cheby = W.reshape(64, 64 * 9).copy()
    y = layer(np.tanh(x))
    _save("c1_cheby_f32.npz", x=x, w_cheby=layer.w_cheby, y=y)


def quant_goldens(mk, fb):
    """Reference NumPy quantisers/dequantisers (quantization.py) run unchanged."""
    fb.quant_semantics = "fallback"
    rng = np.random.default_rng(7)
    rec = {}
    # INT8 / INT4 on a ragged row length (padding exercised) and the test's N(0,1) [32, 64]
    for tag, w, gs in (("n01_32x64_g32", rng.normal(0, 1, (32, 64)).astype(np.float32), 32),
                       ("ragged_12x100_g64", rng.normal(0, 0.02, (12, 100)).astype(np.float32), 64),
                       ("const_4x64_g64", np.full((4, 64), 0.25, np.float32), 64)):
        for bits in (8, 4):
            qw = mk.QuantizedWeight(w, bits=bits, group_size=gs)
            rec[f"aff{bits}_{tag}/w"] = w
            rec[f"aff{bits}_{tag}/qweight"] = qw.qweight
            rec[f"aff{bits}_{tag}/scales"] = qw.scales
            rec[f"aff{bits}_{tag}/biases"] = qw.biases
            rec[f"aff{bits}_{tag}/deq"] = np.ascontiguousarray(qw.dequantize())
            rec[f"aff{bits}_{tag}/gs"] = np.asarray(gs)
    for tag, w, gs in (("n_8x72_g32", rng.normal(0, 0.05, (8, 72)).astype(np.float32), 32),
                       ("n_6x100_g64", rng.normal(0, 0.02, (6, 100)).astype(np.float32), 64),
                       ("zeros_2x40_g16", np.zeros((2, 40), np.float32), 16)):
        t = mk.TernaryQuantizedWeight(w, group_size=gs)
        rec[f"tern_{tag}/w"] = w
        rec[f"tern_{tag}/packed"] = t.w_packed
        rec[f"tern_{tag}/scales"] = t.scales
        rec[f"tern_{tag}/deq"] = t.dequantize()
        rec[f"tern_{tag}/gs"] = np.asarray(gs)
        cb = np.array([-1.0, -0.33333, 0.33333, 1.0], np.float32)
        i2 = mk.Int2QuantizedWeight(w, group_size=gs, codebook=cb)
        rec[f"int2_{tag}/w"] = w
        rec[f"int2_{tag}/packed"] = i2.w_packed
        rec[f"int2_{tag}/scales"] = i2.scales
        rec[f"int2_{tag}/codebook"] = cb
        rec[f"int2_{tag}/deq"] = i2.dequantize()
        rec[f"int2_{tag}/gs"] = np.asarray(gs)
    _save("quant_reference_numpy.npz", **rec)
    fb.quant_semantics = "bridge"


def block_goldens(mk):
    """GatedKAN d=32/h=64 (fp32, fp16) and a 3-layer MetalKAN stack, through the reference."""
    rec = {}
    for mode in ("f32", "f16"):
        np.random.seed(42)
        blk = mk.GatedKAN(d_model=32, d_ffn=64, degree=4,
                          dtype=np.float16 if mode == "f16" else np.float32)
        x = np.random.uniform(-0.8, 0.8, (6, 32)).astype(np.float32)
        xin = x.astype(np.float16) if mode == "f16" else x
        y = blk(xin)
        rec[f"gated_{mode}/x"] = xin
        rec[f"gated_{mode}/y"] = y
        for nm in ("gate_kan", "up_kan", "down_kan"):
            l = getattr(blk, nm)
            rec[f"gated_{mode}/{nm}.w_cheby"] = l.w_cheby
            rec[f"gated_{mode}/{nm}.w_base"] = l.w_base
    # INT4-quantised GatedKAN (to_int4 replaces weights by the dequantised fp32 arrays).
    # Row lengths are multiples of the group size (like the BASELINE config-4 shapes): when they
    # are not, the reference's QuantizedWeight.dequantize returns a non-contiguous slice of the
    # padded matrix (quantization.py:123) whose raw pointer the layer forward then hands to the
    # bridge, which reads the rows misaligned -- a reference defect the engine does not copy.
    np.random.seed(3)
    blk = mk.GatedKAN(d_model=64, d_ffn=128, degree=5)
    blk.to_int4(group_size=64)
    x = np.random.normal(0, 1, (10, 64)).astype(np.float32)
    rec["gated_int4/x"] = x
    rec["gated_int4/y"] = blk(x)
    for nm in ("gate_kan", "up_kan", "down_kan"):
        l = getattr(blk, nm)
        for attr in ("w_cheby", "w_base"):
            q = getattr(l, f"_{attr}_quantized")
            rec[f"gated_int4/{nm}.{attr}.qweight"] = q.qweight
            rec[f"gated_int4/{nm}.{attr}.scales"] = q.scales
            rec[f"gated_int4/{nm}.{attr}.biases"] = q.biases
            rec[f"gated_int4/{nm}.{attr}.deq"] = np.ascontiguousarray(getattr(l, attr))
    # MetalKAN stacks
    for basis, deg in (("cheby", 4), ("fastkan", 8), ("bspline", 5), ("wav", 6)):
        np.random.seed(11)
        net = mk.MetalKAN([4, 16, 8, 2], basis_type=basis, degree=deg)
        x = np.random.uniform(-0.8, 0.8, (32, 4)).astype(np.float32)
        rec[f"net_{basis}/x"] = x
        rec[f"net_{basis}/y"] = net(x)
        for li, l in enumerate(net.layers):
            for attr in ("w_cheby", "w_rbf", "w_spline", "w_wav", "w_relu", "w_fourier", "w_jacobi",
                         "w_down", "w_up", "w_p", "w_q", "w_base", "bias", "grid", "translation",
                         "_inv_scale"):
                if hasattr(l, attr):
                    rec[f"net_{basis}/{li}.{attr.lstrip('_')}"] = np.asarray(getattr(l, attr))
    # pipelined Cheby chain (reference hard-codes degree 4 there, so use degree 4)
    np.random.seed(5)
    net = mk.MetalKAN([4, 16, 8, 2], basis_type="cheby", degree=4, pipeline=True)
    x = np.random.uniform(-1, 1, (128, 4)).astype(np.float32)
    rec["chain/x"] = x
    rec["chain/y"] = net(x)
    for li, l in enumerate(net.layers):
        rec[f"chain/{li}.w_cheby"] = l.w_cheby
        rec[f"chain/{li}.w_base"] = l.w_base
        rec[f"chain/{li}.bias"] = l.bias
    _save("blocks_small.npz", **rec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("KAN_REFERENCE"),
                    help="the reference source tree (or set KAN_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path to the reference tree> or set KAN_REFERENCE")
    sys.path.insert(0, args.reference)
    sys.path.insert(0, REPO)
    import metal_kans as mk  # the reference package
    assert os.path.abspath(mk.__file__).startswith(os.path.abspath(args.reference)), mk.__file__
    from oracle import fake_bridge

    fb = fake_bridge.install(mk)
    layer_goldens(mk)
    c1_golden(mk)
    quant_goldens(mk, fb)
    block_goldens(mk)


if __name__ == "__main__":
    main()
