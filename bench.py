"""Benchmark of the fused KAN forward on B200: rows/s at N GPUs, roofline, CPU baseline, e2e.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5:ternary:65536]
                    [--shard strong|weak] [--impl engine|reference]

Default workload (N=1): BASELINE config 5 at its largest batch -- ChebyKAN 4096 -> 4096, T_0..T_8
+ SiLU base branch, ternary 2-bit weights in 64-code groups (fp16-valued scales ~ U(0.01, 0.05)),
x ~ U(-1, 1) in bf16, B = 65536 rows: 22.0 TFLOP per step, the largest single-GPU configuration
of BASELINE.json.  Other lines: c1 (ChebyKAN fp32), c2 (FastKAN fp16 + LayerNorm), c3 (BSpline
784-512-512-10 net fp16), c4 (GatedKAN bf16, INT4 weights), c5:<ternary|int2>:<B>.  All inputs are
synthetic and seeded; weights are random with BASELINE's shapes and distributions.

Timing: W untimed warm-up steps; then K steps, each preceded (outside the timed interval) by a
256 MiB write that flushes the 126 MB L2, timed with CUDA events on the engine's stream;
barrier + synchronize before and after; the max over ranks is reported.  `value` is whole-job
rows/s.  Multi-GPU (torchrun), `--shard strong` (default): the config's global batch is split into
contiguous row blocks, one per rank, weights replicated, no data-path collective; for c5 with
B <= 16 the layer is output-sharded instead (each rank 1/N of the output columns, then one NCCL
all-gather inside the timed step; the line also gives the step time without the gather).
`--shard weak` runs the full batch on every rank.  `e2e` times the public API (`layer(x)` on a
NumPy array in page-locked host memory: host->device copy, kernels, device->host copy).
`parity` compares a row sample of the timed output with the float64 oracle after the timed
region (the checker; it never feeds the measurement).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(REPO, "metal-kans_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "fused KAN layer rows/sec at 1/2/4/8 B200; % tensor-pipe or HBM roofline"
DEFAULT_CONFIG = "c5:ternary:65536"
TOL = {"f32": 1e-5, "f16": 2e-3, "bf16": 2e-3}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per step, like roofline.achieved: the
# step's one launch, or the sum of its launches for the nets (c3) and the GatedKAN block (c4); each
# from an ncu capture summarised under profiles/ (file named per entry).  `scale` > 1: captured on
# a smaller batch of the same layer and scaled by the rows processed (the summary says why that
# holds); the line reports the scale.
TRAFFIC = {
    "c1": {"bytes": 451328, "src": "profiles/kan_simt_dense_kernel_c1_cheby_fp32_b1024.md"},
    "c2": {"bytes": 3386368, "src": "profiles/kan_tc_kernel_c2_fastkan_fp16_b4096.md"},
    "c4": {"bytes": 2487623424 + 234930432,
           "src": "profiles/kan_tc_kernel_c4_gated_int4_bf16_t16384.md",
           "note": "both launches of a step: gate + up pair, then down"},
    "c3": {"bytes": 20279296 + 512 + 13347328 + 16128 + 8580608,
           "src": "profiles/kan_tc_kernel_c3_bspline_fp16_b8192.md",
           "note": "the net's three launches of a step"},
    "c5:ternary:4096": {"bytes": 470647552 + 23311616,
                        "src": "profiles/kan_tc_kernel_c5_ternary_bf16_b4096.md"},
    "c5:ternary:16": {"bytes": 53773568 + 152064,
                      "src": "profiles/kan_gemv_kernel_c5_ternary_bf16_b16.md"},
    "c5:ternary:1": {"bytes": 52557312 + 40448,
                     "src": "profiles/kan_gemv_cc_kernel_c5_ternary_bf16_b1.md",
                     "note": "the main kernel; the pre-pass reads 40 KB"},
    "c5:ternary:65536": {"bytes": 5892764672 + 527818752,
                         "src": "profiles/kan_tc_kernel_c5_ternary_bf16_b65536.md"},
}


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": p["hbm_gbs"], "tensor": p["bf16_tflops"],
                "tensor_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "src": "measured"}
    except Exception:
        return {"hbm": 6650.0, "tensor": 1590.0, "tensor_sustained": 1400.0, "src": "fallback"}


# --------------------------------------------------------------------------------------------
# workloads.  Weights come from seed 0 (identical on every rank).  Inputs are generated in
# 1024-row blocks, block b from seed (100, b): any contiguous row range of the global batch is
# the same whichever rank (and however many ranks) generate it.
# --------------------------------------------------------------------------------------------
X_BLOCK = 1024


class Workload:
    """One BASELINE config: its weights and input generator, the engine builder, the algorithmic
    work, the CPU restatement of the reference path (timed baseline) and the oracle (checker)."""

    bound = "tensor"
    bytes = 0.0
    kind = None

    def rows(self, lo, hi):
        """Input rows [lo, hi) of the global batch."""
        parts = []
        for b in range(lo // X_BLOCK, (hi + X_BLOCK - 1) // X_BLOCK):
            blk = self.gen(np.random.default_rng([100, b]), X_BLOCK)
            s, e = max(lo, b * X_BLOCK) - b * X_BLOCK, min(hi, (b + 1) * X_BLOCK) - b * X_BLOCK
            parts.append(blk[s:e])
        return np.ascontiguousarray(np.concatenate(parts)) if parts else None


def _bf16():
    from metal_kans._engine import BFLOAT16

    return BFLOAT16


def spec_c1():
    rw = np.random.default_rng(0)
    w = Workload()
    w.key, w.B, w.dtype, w.d_in, w.d_out = "c1", 1024, "f32", 64, 64
    w.name = "ChebyKAN fp32 64->64, T_0..T_8 of tanh(x) (BASELINE config 1)"
    w.W = {"w_cheby": rw.normal(0, np.sqrt(1 / 576), (64, 576)).astype(np.float32)}
    w.gen = lambda rng, n: rng.uniform(-1, 1, (n, 64)).astype(np.float32)
    w.flops_per_row = 2.0 * 64 * 64 * 9
    w.cfg = {"D_in": 64, "D_out": 64, "K": 9, "basis": "cheby", "input_map": "tanh",
             "note": "fp32 runs on CUDA cores (SIMT); roofline shown against the bf16 tensor peak"}

    def build(mk):
        l = mk.ChebyKAN(64, 64, degree=9, bias=False, use_base=False, input_map="tanh")
        l.w_cheby = w.W["w_cheby"]
        return l, [l]
    w.build = build

    def cpu(xs):
        from oracle import kan_oracle as O

        return O.kan_layer_cpu_f32(xs, "cheby", w.W["w_cheby"], K=9, input_map="tanh")
    w.cpu = cpu
    return w


def spec_c2():
    rw = np.random.default_rng(0)
    w = Workload()
    w.key, w.B, w.dtype, w.d_in, w.d_out = "c2", 4096, "f16", 256, 256
    w.name = "FastKAN RBF fp16 256->256, 8 centres, LayerNorm input (BASELINE config 2)"
    w.W = {"w_rbf": rw.normal(0.0, 0.1, (256, 256 * 8)).astype(np.float32),
           "w_base": rw.normal(0.0, 1.0 / 16.0, (256, 256)).astype(np.float32),
           "bias": np.zeros(256, np.float32)}
    w.gen = lambda rng, n: rng.normal(0.0, 1.0, (n, 256)).astype(np.float16)
    w.flops_per_row = 2.0 * 256 * 256 * (8 + 1)
    w.cfg = {"D_in": 256, "D_out": 256, "K": 8, "basis": "rbf", "input_map": "layernorm",
             "sigma": 4 / 7, "grid": [-2.0, 2.0], "has_base": True}

    def build(mk):
        l = mk.FastKAN(256, 256, num_centers=8, grid_range=(-2.0, 2.0), bias=True, use_base=True,
                       input_map="layernorm")
        l.inv_denominator = 1.0 / (4.0 / 7.0) ** 2  # 3.0625: exp(-((x-c)/sigma)^2)
        l.w_rbf, l.w_base, l.bias = w.W["w_rbf"], w.W["w_base"], w.W["bias"]
        l.half()
        return l, [l]
    w.build = build

    def cpu(xs):
        from oracle import kan_oracle as O

        g = np.linspace(-2.0, 2.0, 8).astype(np.float32)
        return O.kan_layer_cpu_f32(xs.astype(np.float32), "rbf", w.W["w_rbf"], w.W["w_base"],
                                   w.W["bias"], K=8, grid=g, inv_den=3.0625,
                                   input_map="layernorm")
    w.cpu = cpu
    return w


C3_DIMS = [784, 512, 512, 10]


def spec_c3():
    rw = np.random.default_rng(0)
    w = Workload()
    w.key, w.B, w.dtype, w.d_in, w.d_out = "c3", 8192, "f16", 784, 10
    w.name = "BSplineKAN net 784-512-512-10 fp16, cubic, grid 5 on [-1,1] (BASELINE config 3)"
    w.W = []
    for di, do in zip(C3_DIMS, C3_DIMS[1:]):
        w.W.append({"w_spline": rw.normal(0, 0.1, (do, di * 8)).astype(np.float32),
                    "w_base": rw.normal(0, 1.0 / np.sqrt(di), (do, di)).astype(np.float32),
                    "bias": np.zeros(do, np.float32)})
    w.gen = lambda rng, n: rng.uniform(-1, 1, (n, 784)).astype(np.float16)
    w.flops_per_row = 2.0 * sum(a * b for a, b in zip(C3_DIMS, C3_DIMS[1:])) * 9
    w.cfg = {"dims": C3_DIMS, "K": 8, "basis": "bspline", "grid_size": 5, "has_base": True}

    def build(mk):
        # MetalKAN passes `degree` as the B-spline grid size (metal_kan.py:76-77): 5 -> 8 bases
        net = mk.MetalKAN(C3_DIMS, basis_type="bspline", degree=5, bias=True, use_base=True)
        for l, p in zip(net.layers, w.W):
            l.w_spline, l.w_base, l.bias = p["w_spline"], p["w_base"], p["bias"]
        net.half()
        return net, list(net.layers)
    w.build = build

    def cpu(xs):
        from oracle import kan_oracle as O

        h = xs.astype(np.float32)
        for p in w.W:
            h = O.kan_layer_cpu_f32(h, "bspline", p["w_spline"], p["w_base"], p["bias"],
                                    grid_size=5, grid_min=-1.0, inv_h=2.5)
        return h
    w.cpu = cpu
    return w


C4_D, C4_H, C4_K = 2048, 5632, 5


def spec_c4():
    rw = np.random.default_rng(0)
    w = Workload()
    w.key, w.B, w.dtype, w.d_in, w.d_out = "c4", 16384, "bf16", C4_D, C4_D
    w.name = ("GatedKAN FFN bf16, INT4 block-affine weights (group 64), Cheby T_0..T_4 "
              "(BASELINE config 4)")
    w.W = {}
    for nm, (do, di) in (("gate", (C4_H, C4_D)), ("up", (C4_H, C4_D)), ("down", (C4_D, C4_H))):
        w.W[nm] = (rw.normal(0, 0.02, (do, di * C4_K)).astype(np.float32),
                   rw.normal(0, 0.02, (do, di)).astype(np.float32))
    w.gen = lambda rng, n: rng.normal(0, 1, (n, C4_D)).astype(np.float32).astype(_bf16())
    w.flops_per_row = 2.0 * 3 * C4_H * C4_D * (C4_K + 1)
    w.cfg = {"d_model": C4_D, "d_ffn": C4_H, "K": C4_K, "basis": "cheby", "has_base": True,
             "weights": "int4 g64, fp32 scale/min (reference layout)"}

    def build(mk):
        blk = mk.GatedKAN(C4_D, C4_H, degree=C4_K, has_base=True, has_bias=False)
        for nm, l in zip(("gate", "up", "down"), blk._layers()):
            l.w_cheby, l.w_base = w.W[nm]
        blk.to_int4(group_size=64)
        blk.bfloat16()
        return blk, list(blk._layers())
    w.build = build

    def cpu(xs):
        from oracle import kan_oracle as O

        x = xs.astype(np.float32)
        g = O.kan_layer_cpu_f32(x, "cheby", *w.W["gate"], K=C4_K)
        u = O.kan_layer_cpu_f32(x, "cheby", *w.W["up"], K=C4_K)
        h = (g / (1.0 + np.exp(-np.clip(g, -20, 20))) * u).astype(np.float32)
        return O.kan_layer_cpu_f32(h, "cheby", *w.W["down"], K=C4_K)
    w.cpu = cpu
    w.cpu_note = "fp32 weights before INT4 quantisation (same shapes and work)"
    return w


C5_D, C5_K, C5_GS = 4096, 9, 64


def spec_c5(B=65536, kind="ternary"):
    from metal_kans.quantization import pack_codes

    rw = np.random.default_rng(0)
    w = Workload()
    w.key, w.B, w.dtype, w.d_in, w.d_out, w.kind = f"c5:{kind}:{B}", B, "bf16", C5_D, C5_D, kind
    w.name = (f"ChebyKAN 4096->4096 T_0..T_8 + base, {kind} 2-bit weights (group 64), bf16 "
              f"(BASELINE config 5)")
    w.W = {}
    for nm, cols in (("w_cheby", C5_D * C5_K), ("w_base", C5_D)):
        groups = (cols + C5_GS - 1) // C5_GS
        if kind == "ternary":
            codes = rw.integers(0, 3, (C5_D, cols), dtype=np.uint8)
            scales = rw.uniform(0.01, 0.05, (C5_D, groups)).astype(np.float16).astype(np.float32)
            cb = None
        else:
            codes = rw.integers(0, 4, (C5_D, cols), dtype=np.uint8)
            scales = np.ones((C5_D, groups), np.float32)
            cb = rw.normal(0, 0.03, 4).astype(np.float16).astype(np.float32)
        w.W[nm] = (pack_codes(codes), scales, (C5_D, cols), cb)
    w.gen = lambda rng, n: rng.uniform(-1, 1, (n, C5_D)).astype(np.float32).astype(_bf16())
    w.flops_per_row = 2.0 * C5_D * C5_D * (C5_K + 1)
    w.weight_bytes = float(sum(p.nbytes + s.nbytes for p, s, _, _ in w.W.values()))
    w.bound = "hbm" if B <= 16 else "tensor"
    w.cfg = {"D_in": C5_D, "D_out": C5_D, "K": C5_K, "basis": "cheby", "has_base": True,
             "weights": f"{kind} 2-bit g{C5_GS}", "packed_weight_bytes": int(w.weight_bytes)}

    def build(mk):
        from metal_kans.quantization import attach_packed, packed_from_codes

        l = mk.ChebyKAN(C5_D, C5_D, degree=C5_K, bias=False, use_base=True)
        for nm in ("w_cheby", "w_base"):
            p, s, shape, cb = w.W[nm]
            attach_packed(l, nm, packed_from_codes(kind, p, s, shape, C5_GS, cb))
        l.bfloat16()
        return l, [l]
    w.build = build
    cache = {}

    def cpu(xs):
        from oracle import kan_oracle as O

        if not cache:
            for nm in ("w_cheby", "w_base"):
                p, s, shape, cb = w.W[nm]
                cache[nm] = (O.dequantize_ternary(p, s, shape[1], C5_GS) if kind == "ternary"
                             else O.dequantize_int2(p, s, cb, shape[1], C5_GS))
        return O.kan_layer_cpu_f32(xs.astype(np.float32), "cheby", cache["w_cheby"],
                                   cache["w_base"], K=C5_K)
    w.cpu = cpu
    return w


def get_spec(config, rows=0):
    """The Workload of "c1".."c4" or "c5:<ternary|int2>:<B>"; rows > 0 keeps the config's layer
    and runs a batch of `rows` rows instead (smaller cases for profiling)."""
    parts = config.split(":")
    if parts[0] == "c5":
        kind = parts[1] if len(parts) > 1 else "ternary"
        B = int(parts[2]) if len(parts) > 2 else 65536
        w = spec_c5(B=rows or B, kind=kind)
    else:
        w = {"c1": spec_c1, "c2": spec_c2, "c3": spec_c3, "c4": spec_c4}[parts[0]]()
        if rows:
            w.B = rows
            w.cfg = {**w.cfg, "rows_override": rows}
    w.cfg = {"B": w.B, **w.cfg}
    return w


# --------------------------------------------------------------------------------------------
# oracle of a workload on a row sample (the checker: float64, reference rounding points)
# --------------------------------------------------------------------------------------------
def _oracle_layer(l, x, mode, out_round):
    from oracle import kan_oracle as O

    W = np.asarray(getattr(l, l.MAIN)).astype(np.float32)
    wb = np.asarray(l.w_base).astype(np.float32) if l.has_base else None
    b = np.asarray(l.bias).astype(np.float32) if l.has_bias else None
    kw = {}
    if l.MAIN == "w_rbf":
        kw = dict(grid=np.asarray(l.grid).astype(np.float32), inv_den=l.inv_denominator)
    elif l.MAIN == "w_spline":
        kw = dict(grid_size=l.grid_size, grid_min=float(l.grid[0]), inv_h=float(l.grid[1]))
    basis = {"w_cheby": "cheby", "w_rbf": "rbf", "w_spline": "bspline"}[l.MAIN]
    return O.kan_layer(x, basis, mode, W, wb, b, K=l._terms(),
                       input_map=getattr(l, "input_map", "none"), out_round=out_round, **kw)


def oracle_rows(w, layers, x):
    """Unrounded float64 oracle output of the workload for input rows x: intermediate layers
    rounded to the act dtype as the engine stores them, the last one left unrounded."""
    from oracle import kan_oracle as O

    mode = w.dtype
    if w.key == "c4":
        g = _oracle_layer(layers[0], x, mode, True)
        u = _oracle_layer(layers[1], x, mode, True)
        act = O.act_dtype(mode)
        h = O.swiglu(g, u).astype(np.float32).astype(act)
        return _oracle_layer(layers[2], h, mode, False)
    h = x
    for i, l in enumerate(layers):
        h = _oracle_layer(l, h, mode, i < len(layers) - 1)
    return h


def parity_check(w, layers, x_local, y_local, n_rows=64):
    """max-rel-err (final rounding allowed) of a row sample of the timed output vs the oracle."""
    from oracle import kan_oracle as O

    B = y_local.shape[0]
    idx = np.unique(np.linspace(0, B - 1, min(n_rows, B)).round().astype(np.int64))
    ref = oracle_rows(w, layers, np.ascontiguousarray(x_local[idx]))
    err = O.max_rel_err_rounded(np.asarray(y_local[idx]).astype(np.float64), ref, w.dtype)
    return {"max_rel_err": err, "tol": TOL[w.dtype], "rows": int(idx.size), "ok": err <= TOL[w.dtype],
            "check": "float64 oracle (reference rounding points) on a row sample of the timed "
                     "output, final rounding allowed"}


# --------------------------------------------------------------------------------------------
# measurement helpers
# --------------------------------------------------------------------------------------------
class Clocks:
    """SM clock and clock-event reasons sampled every 2 ms by NVML (reads only) in a thread that
    runs from just before the timed region to its end."""

    NAMES = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
             ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, cuda_index):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml as N
            import torch

            N.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
            try:
                h = N.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[cuda_index]) if vis else cuda_index
                h = N.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            self._N, self._h = N, h
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # no NVML: the line says so
            self.error = str(e)

    def _run(self):
        N, h = self._N, self._h
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM))
                self.reasons |= N.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception:
                pass
            time.sleep(0.002)

    def stop(self):
        if self._t is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                    "error": getattr(self, "error", "nvml unavailable")}
        self._stop.set()
        self._t.join()
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": [n for n, bit in self.NAMES if self.reasons & bit]}


def blas_on_all_cores():
    """A context in which NumPy's BLAS uses every host core of this process (torchrun sets
    OMP_NUM_THREADS=1 when it starts several processes), and that thread count."""
    import contextlib

    cores = len(os.sched_getaffinity(0))
    try:
        from threadpoolctl import threadpool_limits

        return threadpool_limits(limits=cores, user_api="blas"), cores
    except Exception:
        return contextlib.nullcontext(), int(os.environ.get("OMP_NUM_THREADS", cores))


def cpu_sample(w, budget_s, min_calls=1):
    """Time the CPU restatement of the reference path on a bounded row sample of the workload
    (threads: NumPy's BLAS on every host core of this process)."""
    ctx, cores = blas_on_all_cores()
    with ctx:
        return _cpu_sample(w, budget_s, min_calls, cores)


def _cpu_sample(w, budget_s, min_calls, cores):
    sample = min(w.B, 512)
    xs = w.rows(0, sample)
    w.cpu(xs)  # warm-up (also builds cached dequantised weights)
    n, t0 = 0, time.perf_counter()
    while n < min_calls or time.perf_counter() - t0 < budget_s:
        w.cpu(xs)
        n += 1
    dt = time.perf_counter() - t0
    note = getattr(w, "cpu_note", "")
    desc = (f"{n} calls x {sample} rows of the same workload, float32 NumPy restatement of the "
            f"reference's fp32 path (the reference runs only on Metal; BLAS on {cores} threads)"
            f"{', ' + note if note else ''}, {dt:.1f} s")
    return n * sample / dt, cores, desc, n, dt


def device_step(mk, obj, layers, B, x_ptr, y_ptr, keep):
    """A closure that enqueues the workload on device buffers; descriptors are built once.
    Returns (step, buffers holding the intermediate activations)."""
    lib = mk.get_metal_bridge()
    from metal_kans import GatedKAN
    from metal_kans._engine import DeviceBuffer

    if isinstance(obj, GatedKAN):
        descs = [l._descriptor(keep) for l in layers]
        # gate + up packed as one tensor-core matrix (one launch, SwiGLU in its epilogue)
        pair = obj._pair(descs[0], descs[1], keep)
        esz = np.dtype(obj.gate_kan.dtype).itemsize
        h = DeviceBuffer(B * obj.d_ffn * esz)
        keep.append(h)
        args = ([ctypes.byref(d) for d in descs] +
                [ctypes.c_void_p(pair), ctypes.c_void_p(x_ptr), ctypes.c_void_p(h.ptr),
                 ctypes.c_void_p(y_ptr), B, None])
        return (lambda: lib.kan_gated_forward_pair(*args)), [h]
    esz = np.dtype(layers[0].dtype).itemsize
    width = max(l.out_features for l in layers)
    bufs = [DeviceBuffer(B * width * esz), DeviceBuffer(B * width * esz)]
    keep.extend(bufs)
    calls, cur = [], x_ptr
    for i, l in enumerate(layers):
        nxt = y_ptr if i == len(layers) - 1 else bufs[i % 2].ptr
        d = l._descriptor(keep)
        keep.append(d)
        calls.append((ctypes.byref(d), ctypes.c_void_p(cur), ctypes.c_void_p(nxt)))
        cur = nxt

    def run():
        for d, xi, yo in calls:
            lib.kan_forward(d, xi, yo, B, None)
    return run, bufs


def plan_of(mk, layers, B):
    """The kernel plan of each layer's launch (kan_forward_plan): path, tile width, splits."""
    lib = mk.get_metal_bridge()
    names = {1: "simt", 2: "tc", 3: "small-batch tensor cores", 4: "small-batch CUDA cores"}
    out = []
    for l in layers:
        keep = []
        d = l._descriptor(keep)
        info = (ctypes.c_int * 6)()
        lib.kan_forward_plan(ctypes.byref(d), int(B), 0, info)
        e = {"path": names.get(info[0], str(info[0]))}
        if info[0] == 2:
            e.update(BN=info[1], splits=info[2], grid=[info[3], info[4], info[2]])
        elif info[0] == 3:
            e.update(row_blocks=info[3])
        elif info[0] == 4:
            e.update(row_blocks=info[3], splits=info[2])
        out.append(e)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--shard", default="strong", choices=["strong", "weak"])
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--parity-rows", type=int, default=64)
    ap.add_argument("--rows", type=int, default=0,
                    help="override the global batch (smaller cases of a config for profiling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import metal_kans as mk
    from metal_kans._engine import DeviceBuffer
    from metal_kans.parallel import shard_range

    lib = mk.get_metal_bridge()
    lib.kan_set_device(local)
    w = get_spec(args.config, args.rows)
    obj, layers = w.build(mk)
    oshard = world > 1 and w.key.startswith("c5") and w.B <= 16
    strong = world > 1 and args.shard == "strong" and not oshard
    if strong:
        lo, hi = shard_range(w.B, world, rank)
    else:
        lo, hi = 0, w.B
    B = hi - lo                       # this rank's rows
    rows_per_step = w.B if (oshard or strong or world == 1) else world * w.B
    x = w.rows(lo, hi)
    stream = torch.cuda.ExternalStream(lib.kan_default_stream())
    keep = []
    esz = x.dtype.itemsize
    dx = DeviceBuffer.from_array(x)
    dy = DeviceBuffer(B * w.d_out * esz)
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[w.dtype]
    if oshard:
        # each rank computes its column block into a torch tensor on the engine's stream; the
        # NCCL all-gather (ordered after it by torch's stream semantics) assembles Y[B, D_out]
        from metal_kans.parallel import OutputShardedLayer

        sharded = OutputShardedLayer(obj)
        y_loc = torch.empty((B, sharded.local.out_features), dtype=tdt, device="cuda")
        gathered = torch.empty((world, B, sharded.width), dtype=tdt, device="cuda")
        y_full = torch.empty((B, w.d_out), dtype=tdt, device="cuda")
        run_local, _ = device_step(mk, sharded.local, [sharded.local], B, dx.ptr,
                                   y_loc.data_ptr(), keep)

        def step():
            run_local()
            sharded.gather_into(y_loc, gathered, y_full)
        plan = plan_of(mk, [sharded.local], B)
    else:
        step, _ = device_step(mk, obj, layers, B, dx.ptr, dy.ptr, keep)
        if w.key == "c4":
            plan = ([{"launch": "gate + up as one tensor-core launch (wide tiles, SwiGLU in the "
                                "epilogue)"}] + plan_of(mk, layers[2:], B))
        else:
            plan = plan_of(mk, layers, B)

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")

    def barrier():
        torch.cuda.synchronize()
        lib.kan_stream_synchronize(None)
        if dist is not None:
            dist.barrier()
            torch.cuda.synchronize()

    def timed(fn, steps):
        """Per-step CUDA-event times (ms) of `fn`, L2 flushed before each step."""
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        with torch.cuda.stream(stream):
            for i in range(steps):
                flush.zero_()  # L2 flush, outside the timed interval
                ev[i][0].record(stream)
                fn()
                ev[i][1].record(stream)
        barrier()
        return [a.elapsed_time(b) for a, b in ev]

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    barrier()
    clocks = Clocks(local)
    n0 = lib.kan_launch_count()
    times = timed(step, args.steps)
    clk = clocks.stop()
    launches = lib.kan_launch_count() - n0
    total_ms = max_over_ranks(sum(times))
    ms_step = total_ms / args.steps
    value = rows_per_step * args.steps / (total_ms / 1e3)
    no_gather = None
    if oshard:
        t_local = max_over_ranks(sum(timed(run_local, args.steps)))
        no_gather = {"ms_per_step": t_local / args.steps,
                     "value": rows_per_step * args.steps / (t_local / 1e3),
                     "note": "each rank's column block without the NCCL all-gather"}

    # roofline of this rank's launches (the per-GPU work divided by the per-step device time)
    pk = peaks()
    kern_s = statistics.mean(times) / 1e3
    rank_rows = B
    if w.bound == "tensor":
        flops = w.flops_per_row * rank_rows
        achieved = flops / kern_s / 1e12
        # a run held at the power cap (sw_power_cap seen during the timed region) is compared
        # with the measured sustained GEMM rate, a run at full clocks with the burst rate
        capped = "sw_power_cap" in clk.get("reasons", [])
        peak = pk["tensor_sustained"] if capped else pk["tensor"]
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_src": pk["src"] + " bf16 dense (" + ("sustained, power-capped run"
                                                          if capped else "burst") + ")",
                "algorithmic_flops_per_step": flops}
    else:
        per_rank_w = w.weight_bytes / (world if oshard else 1)
        cols = w.d_out / (world if oshard else 1)
        nbytes = per_rank_w + x.nbytes + rank_rows * cols * esz
        achieved = nbytes / kern_s / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s",
                "frac": achieved / pk["hbm"], "peak_src": pk["src"] + " copy",
                "algorithmic_bytes_per_step": nbytes}
    tr = TRAFFIC.get(w.key if not args.rows else f"{w.key}@{args.rows}")
    roof["traffic"] = tr["bytes"] if tr else None
    if tr:
        roof["traffic_src"] = tr["src"] + (f" ({tr['note']})" if "note" in tr else "")
        if tr.get("scale"):
            roof["traffic_scale"] = tr["scale"]
        if strong and w.bound == "tensor":
            # the capture is of a full-batch launch; a rank's launch covers B / N rows, and the
            # traffic of this tensor-bound kernel (input re-reads per N panel, output writes)
            # grows with the rows it processes
            roof["traffic"] = tr["bytes"] * B / w.B
            roof["traffic_scale"] = f"{B}/{w.B} of the full-batch capture (this rank's rows)"

    # parity of the timed output (rank 0's rows; the gathered full output when output-sharded)
    parity = None
    if rank == 0 and args.parity_rows > 0:
        if oshard:
            yt = y_full.cpu()
        else:
            yt = torch.empty((B, w.d_out), dtype=tdt)
            lib.kan_memcpy(ctypes.c_void_p(yt.data_ptr()), ctypes.c_void_p(dy.ptr),
                           B * w.d_out * esz, 2, None)
            lib.kan_stream_synchronize(None)
        y_np = (yt.view(torch.int16).numpy().view(x.dtype) if tdt == torch.bfloat16
                else yt.numpy())
        parity = parity_check(w, layers, x, y_np, args.parity_rows)

    e2e = (e2e_measure(sharded if oshard else obj, w, x, args, barrier, max_over_ranks,
                       rows_per_step) if args.e2e_steps > 0 else None)
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        v, cores, desc, _, _ = cpu_sample(w, args.cpu_seconds)
        cpu = {"value": v, "unit": "rows/s", "cores": cores, "kind": "port", "sample": desc}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        par = (f"output-shard x{world} + NCCL all-gather" if oshard else
               (f"batch-shard x{world} (global batch split, weights replicated)" if strong else
                (f"batch x{world} (full batch per rank)" if world > 1 else "single GPU")))
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "strong" if (oshard or strong or world == 1) else "weak",
            "vs_baseline": None, "dtype": w.dtype,
            "data": "synthetic (seeded; BASELINE shapes and distributions)",
            "config": {"workload": w.name, **w.cfg, "per_gpu_rows": B, "parallelism": par,
                       "plan": plan, "l2": "flushed (256 MiB write) before every timed step"},
            "roofline": roof, "parity": parity, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk, "cpu_baseline": cpu,
        }
        if no_gather:
            line["without_gather"] = no_gather
        print(json.dumps(line), flush=True)
    del keep
    if dist is not None:
        dist.destroy_process_group()


def e2e_measure(obj, w, x, args, barrier, max_over_ranks, rows_per_step):
    """Public-API throughput: obj(x) on this rank's host rows in pinned memory, returning host y
    (wall clock, max over ranks)."""
    from metal_kans._engine import _Pinned

    pin = _Pinned(x.nbytes)
    xh = np.frombuffer((ctypes.c_char * x.nbytes).from_address(pin.ptr),
                       dtype=x.dtype).reshape(x.shape)
    xh[...] = x
    for _ in range(args.warmup):
        y = obj(xh)
    barrier()
    n = max(3, args.e2e_steps)
    t0 = time.perf_counter()
    for _ in range(n):
        y = obj(xh)
    barrier()
    dt = max_over_ranks(time.perf_counter() - t0)
    return {"value": rows_per_step * n / dt, "unit": "rows/s", "steps": n,
            "h2d_bytes_per_step": int(x.nbytes), "d2h_bytes_per_step": int(y.nbytes),
            "api": f"{type(obj).__name__}.forward(numpy in pinned host memory), wall clock"}


def reference_arm(args, rank, world):
    """The reference path on host cores (its CPU restatement; the reference itself runs only on
    Metal): same config, metric and unit; rank 0 runs, other ranks exit."""
    if rank != 0:
        return
    w = get_spec(args.config, args.rows)
    sample = min(w.B, 512)
    xs = w.rows(0, sample)
    ctx, cores = blas_on_all_cores()
    with ctx:
        for _ in range(args.warmup):
            w.cpu(xs)
        steps, t0 = 0, time.perf_counter()
        while steps < args.steps and (steps < 1 or time.perf_counter() - t0 < 120.0):
            w.cpu(xs)
            steps += 1
        dt = time.perf_counter() - t0
    value = steps * sample / dt
    note = getattr(w, "cpu_note", "")
    line = {"metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE shapes and distributions)",
            "config": {"workload": w.name, **w.cfg, "per_step_rows": sample},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port",
                             "sample": f"{sample} rows per step of the same workload; float32 "
                                       f"NumPy restatement of the reference's fp32 path (the "
                                       f"reference runs only on Metal; BLAS on {cores} "
                                       f"threads){', ' + note if note else ''}; steps capped "
                                       f"at 120 s"},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
