"""Benchmark of the fused KAN forward on B200: rows/s at N GPUs, roofline, CPU baseline, e2e.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl engine|reference]

Default workload (N=1): BASELINE config 2 -- FastKAN RBF layer fp16, B=4096, 256 -> 256,
8 Gaussian centres on [-2, 2], sigma = 4/7 (inv_denominator = 1/sigma^2), input LayerNorm,
SiLU base branch; x ~ N(0,1), W_rbf ~ N(0, 0.1^2), W_base ~ N(0, 1/256); synthetic, seeded.
Other configs print their own line: c1 (ChebyKAN fp32), c3 (BSpline 784-512-512-10 net fp16),
c4 (GatedKAN bf16, INT4 weights), c5:<ternary|int2>:<B> (4096x4096 Cheby, 2-bit weights, bf16).

Timing: W untimed warm-up steps; then K steps, each preceded (outside the timed interval) by a
256 MiB write that flushes the 126 MB L2, timed with CUDA events on the engine's stream;
barrier + synchronize before and after; the max over ranks is reported.  `value` is whole-job
rows/s.  Multi-GPU (torchrun): batch sharding -- every rank runs the full per-GPU batch with the
weights replicated (weak scaling, no data-path collective); for c5 with B <= 16 the layer is
output-sharded instead (each rank 1/N of the output columns, NCCL all-gather inside the timed
step; strong scaling).  `e2e` times the public API (`layer(x)` on a NumPy array in pinned host
memory: host->device copy, kernels, device->host copy) with the wall clock.
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

# ncu dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel, from the
# `ncu --set full` captures summarised under profiles/ (one summary per kernel and workload);
# None when the config was not captured at its own size (c4 is captured on 2048 tokens); c3: the
# first (largest) of its three launches
TRAFFIC = {"c2": 3386368, "c1": 453632, "c5:ternary:4096": 470647552 + 23311616,
           "c5:ternary:16": 53773568 + 152064, "c3": 20276992}


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
# workloads: fp32 weights from seed 0 (replicated on every rank), inputs from seed 100 + rank
# --------------------------------------------------------------------------------------------
class Workload:
    """One BASELINE config: weights/inputs, the engine objects, the algorithmic work and the CPU
    restatement of the reference path (for the timed CPU baseline)."""

    bound = "tensor"
    bytes = 0.0


def _rng(rank):
    return np.random.default_rng(0), np.random.default_rng(100 + rank)


def spec_c1(rank=0):
    rw, rx = _rng(rank)
    w = Workload()
    w.key, w.B, w.dtype, w.d_out = "c1", 1024, "f32", 64
    w.name = "ChebyKAN fp32 64->64, T_0..T_8 of tanh(x) (BASELINE config 1)"
    w.W = {"w_cheby": rw.normal(0, np.sqrt(1 / 576), (64, 576)).astype(np.float32)}
    w.x = rx.uniform(-1, 1, (w.B, 64)).astype(np.float32)
    w.flops = 2.0 * w.B * 64 * 64 * 9
    w.cfg = {"B": w.B, "D_in": 64, "D_out": 64, "K": 9, "basis": "cheby", "input_map": "tanh",
             "note": "fp32 runs on CUDA cores (SIMT); roofline shown against the bf16 tensor peak"}
    W = w.W["w_cheby"]
    from oracle import kan_oracle as O

    w.cpu = lambda xs: O.kan_layer_cpu_f32(xs, "cheby", W, K=9, input_map="tanh")
    return w


def engine_c1(mk, w):
    l = mk.ChebyKAN(64, 64, degree=9, bias=False, use_base=False, input_map="tanh")
    l.w_cheby = w.W["w_cheby"]
    return l, [l]


def spec_c2(rank=0):
    rw, rx = _rng(rank)
    w = Workload()
    w.key, w.B, w.dtype, w.d_out = "c2", 4096, "f16", 256
    w.name = "FastKAN RBF fp16 256->256, 8 centres, LayerNorm input (BASELINE config 2)"
    w.W = {"w_rbf": rw.normal(0.0, 0.1, (256, 256 * 8)).astype(np.float32),
           "w_base": rw.normal(0.0, 1.0 / 16.0, (256, 256)).astype(np.float32),
           "bias": np.zeros(256, np.float32)}
    w.x = rx.normal(0.0, 1.0, (w.B, 256)).astype(np.float16)
    w.flops = 2.0 * w.B * 256 * 256 * (8 + 1)
    w.cfg = {"B": w.B, "D_in": 256, "D_out": 256, "K": 8, "basis": "rbf",
             "input_map": "layernorm", "sigma": 4 / 7, "grid": [-2.0, 2.0], "has_base": True}
    Wf, Wbf, bf = w.W["w_rbf"], w.W["w_base"], w.W["bias"]
    g = np.linspace(-2.0, 2.0, 8).astype(np.float32)
    from oracle import kan_oracle as O

    w.cpu = lambda xs: O.kan_layer_cpu_f32(xs.astype(np.float32), "rbf", Wf, Wbf, bf, K=8,
                                           grid=g, inv_den=3.0625, input_map="layernorm")
    return w


def engine_c2(mk, w):
    l = mk.FastKAN(256, 256, num_centers=8, grid_range=(-2.0, 2.0), bias=True, use_base=True,
                   input_map="layernorm")
    l.inv_denominator = 1.0 / (4.0 / 7.0) ** 2  # 3.0625: exp(-((x-c)/sigma)^2)
    l.w_rbf, l.w_base, l.bias = w.W["w_rbf"], w.W["w_base"], w.W["bias"]
    l.half()
    return l, [l]


C3_DIMS = [784, 512, 512, 10]


def spec_c3(rank=0):
    rw, rx = _rng(rank)
    w = Workload()
    w.key, w.B, w.dtype, w.d_out = "c3", 8192, "f16", 10
    w.name = "BSplineKAN net 784-512-512-10 fp16, cubic, grid 5 on [-1,1] (BASELINE config 3)"
    w.W = []
    for di, do in zip(C3_DIMS, C3_DIMS[1:]):
        w.W.append({"w_spline": rw.normal(0, 0.1, (do, di * 8)).astype(np.float32),
                    "w_base": rw.normal(0, 1.0 / np.sqrt(di), (do, di)).astype(np.float32),
                    "bias": np.zeros(do, np.float32)})
    w.x = rx.uniform(-1, 1, (w.B, 784)).astype(np.float16)
    w.flops = 2.0 * w.B * sum(a * b for a, b in zip(C3_DIMS, C3_DIMS[1:])) * 9
    w.cfg = {"B": w.B, "dims": C3_DIMS, "K": 8, "basis": "bspline", "grid_size": 5,
             "has_base": True}
    from oracle import kan_oracle as O

    def cpu(xs):
        h = xs.astype(np.float32)
        for p in w.W:
            h = O.kan_layer_cpu_f32(h, "bspline", p["w_spline"], p["w_base"], p["bias"],
                                    grid_size=5, grid_min=-1.0, inv_h=2.5)
        return h
    w.cpu = cpu
    return w


def engine_c3(mk, w):
    # MetalKAN passes `degree` as the B-spline grid size (metal_kan.py:76-77): 5 -> 8 bases
    net = mk.MetalKAN(C3_DIMS, basis_type="bspline", degree=5, bias=True, use_base=True)
    for l, p in zip(net.layers, w.W):
        l.w_spline, l.w_base, l.bias = p["w_spline"], p["w_base"], p["bias"]
    net.half()
    return net, list(net.layers)


C4_D, C4_H, C4_K = 2048, 5632, 5


def spec_c4(rank=0):
    rw, rx = _rng(rank)
    w = Workload()
    w.key, w.B, w.dtype, w.d_out = "c4", 16384, "bf16", C4_D
    w.name = ("GatedKAN FFN bf16, INT4 block-affine weights (group 64), Cheby T_0..T_4 "
              "(BASELINE config 4)")
    w.W = {}
    for nm, (do, di) in (("gate", (C4_H, C4_D)), ("up", (C4_H, C4_D)), ("down", (C4_D, C4_H))):
        w.W[nm] = (rw.normal(0, 0.02, (do, di * C4_K)).astype(np.float32),
                   rw.normal(0, 0.02, (do, di)).astype(np.float32))
    from metal_kans._engine import BFLOAT16

    w.x = rx.normal(0, 1, (w.B, C4_D)).astype(np.float32).astype(BFLOAT16)
    w.flops = 2.0 * w.B * 3 * C4_H * C4_D * (C4_K + 1)
    w.cfg = {"tokens": w.B, "d_model": C4_D, "d_ffn": C4_H, "K": C4_K, "basis": "cheby",
             "has_base": True, "weights": "int4 g64, fp32 scale/min (reference layout)"}
    from oracle import kan_oracle as O

    def cpu(xs):
        x = xs.astype(np.float32)
        g = O.kan_layer_cpu_f32(x, "cheby", *w.W["gate"], K=C4_K)
        u = O.kan_layer_cpu_f32(x, "cheby", *w.W["up"], K=C4_K)
        h = (g / (1.0 + np.exp(-np.clip(g, -20, 20))) * u).astype(np.float32)
        return O.kan_layer_cpu_f32(h, "cheby", *w.W["down"], K=C4_K)
    w.cpu = cpu
    w.cpu_note = "fp32 weights before INT4 quantisation (same shapes and work)"
    return w


def engine_c4(mk, w):
    blk = mk.GatedKAN(C4_D, C4_H, degree=C4_K, has_base=True, has_bias=False)
    for nm, l in zip(("gate", "up", "down"), blk._layers()):
        l.w_cheby, l.w_base = w.W[nm]
    blk.to_int4(group_size=64)
    blk.bfloat16()
    return blk, list(blk._layers())


C5_D, C5_K, C5_GS = 4096, 9, 64


def spec_c5(rank=0, B=4096, kind="ternary"):
    rw, rx = _rng(rank)
    from oracle import kan_oracle as O

    w = Workload()
    w.key, w.B, w.dtype, w.d_out, w.kind = f"c5:{kind}:{B}", B, "bf16", C5_D, kind
    w.name = (f"ChebyKAN 4096->4096 T_0..T_8, {kind} 2-bit weights (group 64), bf16 "
              f"(BASELINE config 5)")
    w.W = {}
    for nm, cols in (("w_cheby", C5_D * C5_K), ("w_base", C5_D)):
        groups = (cols + C5_GS - 1) // C5_GS
        if kind == "ternary":
            codes = rw.integers(0, 3, (C5_D, cols)).astype(np.uint32)
            scales = rw.uniform(0.01, 0.05, (C5_D, groups)).astype(np.float16).astype(np.float32)
            cb = None
        else:
            codes = rw.integers(0, 4, (C5_D, cols)).astype(np.uint32)
            scales = np.ones((C5_D, groups), np.float32)
            cb = rw.normal(0, 0.03, 4).astype(np.float16).astype(np.float32)
        w.W[nm] = (O._pack2(codes), scales, (C5_D, cols), cb)
    from metal_kans._engine import BFLOAT16

    w.x = rx.uniform(-1, 1, (B, C5_D)).astype(np.float32).astype(BFLOAT16)
    w.flops = 2.0 * B * C5_D * C5_D * (C5_K + 1)
    packed = sum(p.nbytes + s.nbytes for p, s, _, _ in w.W.values())
    w.bytes = packed + w.x.nbytes + B * C5_D * 2
    w.bound = "hbm" if B <= 16 else "tensor"
    w.cfg = {"B": B, "D_in": C5_D, "D_out": C5_D, "K": C5_K, "basis": "cheby", "has_base": True,
             "weights": f"{kind} 2-bit g{C5_GS}", "packed_weight_bytes": int(packed)}

    def dense(nm):
        p, s, shape, cb = w.W[nm]
        if kind == "ternary":
            return O.dequantize_ternary(p, s, shape[1], C5_GS)
        return O.dequantize_int2(p, s, cb, shape[1], C5_GS)

    cache = {}

    def cpu(xs):
        if not cache:
            cache["W"], cache["Wb"] = dense("w_cheby"), dense("w_base")
        return O.kan_layer_cpu_f32(xs.astype(np.float32), "cheby", cache["W"], cache["Wb"],
                                   K=C5_K)
    w.cpu = cpu
    return w


def engine_c5(mk, w):
    from metal_kans.quantization import attach_packed, packed_from_codes

    l = mk.ChebyKAN(C5_D, C5_D, degree=C5_K, bias=False, use_base=True)
    for nm in ("w_cheby", "w_base"):
        p, s, shape, cb = w.W[nm]
        attach_packed(l, nm, packed_from_codes(w.kind, p, s, shape, C5_GS, cb))
    l.bfloat16()
    return l, [l]


def get_spec(config, rank=0, rows=0):
    """(Workload, engine builder) for "c1".."c4" or "c5:<ternary|int2>:<B>"; rows > 0 keeps the
    config's weights and takes the first `rows` input rows (a smaller case of the same layer)."""
    parts = config.split(":")
    if parts[0] == "c5":
        kind = parts[1] if len(parts) > 1 else "ternary"
        B = int(parts[2]) if len(parts) > 2 else 4096
        w, eng = spec_c5(rank, B=rows or B, kind=kind), engine_c5
    else:
        spec, eng = {"c1": (spec_c1, engine_c1), "c2": (spec_c2, engine_c2),
                     "c3": (spec_c3, engine_c3), "c4": (spec_c4, engine_c4)}[parts[0]]
        w = spec(rank)
        if rows:
            scale = rows / w.B
            w.x = np.ascontiguousarray(w.x[:rows]) if rows <= w.B else \
                np.ascontiguousarray(np.resize(w.x, (rows, w.x.shape[1])))
            w.flops *= scale
            w.B = rows
            w.cfg = {**w.cfg, "rows_override": rows}
    return w, eng


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


def cpu_baseline(w, budget_s=10.0):
    """Time the CPU restatement of the reference path on a bounded row sample."""
    cores = len(os.sched_getaffinity(0))
    sample = min(w.B, 512)
    xs = np.ascontiguousarray(w.x[:sample])
    w.cpu(xs)  # warm-up
    n, t0 = 0, time.perf_counter()
    while n < 1 or time.perf_counter() - t0 < budget_s:
        w.cpu(xs)
        n += 1
    dt = time.perf_counter() - t0
    note = getattr(w, "cpu_note", "")
    return {"value": n * sample / dt, "unit": "rows/s", "cores": cores, "kind": "port",
            "sample": f"{n} calls x {sample} rows of the same workload, float32 NumPy "
                      f"(BLAS on {cores} threads){', ' + note if note else ''}, {dt:.1f} s"}


def device_step(mk, obj, layers, B, x_ptr, y_ptr, keep):
    """A closure that enqueues the workload on device buffers; descriptors are built once."""
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
        return lambda: lib.kan_gated_forward_pair(*args)
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
    return run


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="c2")
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--rows", type=int, default=0,
                    help="override the per-GPU batch (smaller cases of a config for profiling)")
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

    lib = mk.get_metal_bridge()
    lib.kan_set_device(local)
    w, engine = get_spec(args.config, rank, args.rows)
    obj, layers = engine(mk, w)
    oshard = world > 1 and args.config.startswith("c5") and w.B <= 16
    stream = torch.cuda.ExternalStream(lib.kan_default_stream())
    keep = []
    B = w.B
    esz = w.x.dtype.itemsize
    dx = DeviceBuffer.from_array(w.x)
    dy = DeviceBuffer(B * w.d_out * esz)
    if oshard:
        # each rank computes its column block into a torch tensor on the engine's stream; the
        # NCCL all-gather (ordered after it by torch's stream semantics) assembles Y[B, D_out]
        from metal_kans.parallel import OutputShardedLayer

        sharded = OutputShardedLayer(obj)
        tdt = torch.bfloat16 if w.dtype == "bf16" else torch.float16
        y_loc = torch.empty((B, sharded.local.out_features), dtype=tdt, device="cuda")
        gathered = torch.empty((world, B, sharded.width), dtype=tdt, device="cuda")
        y_full = torch.empty((B, w.d_out), dtype=tdt, device="cuda")
        run_local = device_step(mk, sharded.local, [sharded.local], B, dx.ptr, y_loc.data_ptr(),
                                keep)

        def step():
            run_local()
            sharded.gather_into(y_loc, gathered, y_full)
    else:
        step = device_step(mk, obj, layers, B, dx.ptr, dy.ptr, keep)

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    lib.kan_stream_synchronize(None)

    def barrier():
        torch.cuda.synchronize()
        lib.kan_stream_synchronize(None)
        if dist is not None:
            dist.barrier()
            torch.cuda.synchronize()

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier()
    clocks = Clocks(local)
    n0 = lib.kan_launch_count()
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush.zero_()  # L2 flush, outside the timed interval
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
    barrier()
    clk = clocks.stop()
    launches = lib.kan_launch_count() - n0
    times = [a.elapsed_time(b) for a, b in ev]  # ms per step
    total_ms = sum(times)
    if dist is not None:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_step = total_ms / args.steps
    rows_per_step = B if oshard else world * B
    value = rows_per_step * args.steps / (total_ms / 1e3)
    pk = peaks()
    kern_s = statistics.mean(times) / 1e3
    if w.bound == "tensor":
        achieved = w.flops / kern_s / 1e12
        # a run held at the power cap (sw_power_cap seen during the timed region) is compared
        # with the measured sustained GEMM rate, a run at full clocks with the burst rate
        capped = "sw_power_cap" in clk.get("reasons", [])
        peak = pk["tensor_sustained"] if capped else pk["tensor"]
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_src": pk["src"] + " bf16 dense (" + ("sustained, power-capped run"
                                                          if capped else "burst") + ")",
                "traffic": TRAFFIC.get(args.config), "algorithmic_flops_per_step": w.flops}
    else:
        per_rank_bytes = w.bytes / (world if oshard else 1)
        achieved = per_rank_bytes / kern_s / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s",
                "frac": achieved / pk["hbm"], "peak_src": pk["src"] + " copy",
                "traffic": TRAFFIC.get(args.config), "algorithmic_bytes_per_step": per_rank_bytes}

    e2e = (e2e_measure(sharded if oshard else obj, w, args, barrier, dist, rows_per_step)
           if args.e2e_steps > 0 else None)
    cpu = (cpu_baseline(w, args.cpu_seconds)
           if (rank == 0 and world == 1 and args.cpu_seconds > 0) else None)
    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong" if oshard else "weak",
            "vs_baseline": None, "dtype": w.dtype,
            "data": "synthetic (seeded; BASELINE shapes and distributions)",
            "config": {"workload": w.name, **w.cfg, "per_gpu_rows": B,
                       "parallelism": (f"output-shard x{world} + NCCL all-gather" if oshard else
                                       (f"batch-shard x{world}" if world > 1 else "single GPU")),
                       "l2": "flushed (256 MiB write) before every timed step"},
            "roofline": roof, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del keep
    if dist is not None:
        dist.destroy_process_group()


def e2e_measure(obj, w, args, barrier, dist, rows_per_step):
    """Public-API throughput: obj(x) on host x in pinned memory, returning host y."""
    from metal_kans._engine import _Pinned

    pin = _Pinned(w.x.nbytes)
    xh = np.frombuffer((ctypes.c_char * w.x.nbytes).from_address(pin.ptr),
                       dtype=w.x.dtype).reshape(w.x.shape)
    xh[...] = w.x
    for _ in range(args.warmup):
        y = obj(xh)
    barrier()
    n = max(3, args.e2e_steps if w.B * w.d_out <= (1 << 24) else args.e2e_steps // 10)
    t0 = time.perf_counter()
    for _ in range(n):
        y = obj(xh)
    barrier()
    dt = time.perf_counter() - t0
    if dist is not None:
        import torch

        t = torch.tensor([dt], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    return {"value": rows_per_step * n / dt, "unit": "rows/s", "steps": n,
            "h2d_bytes_per_step": int(w.x.nbytes), "d2h_bytes_per_step": int(y.nbytes),
            "api": f"{type(obj).__name__}.forward(numpy in pinned host memory), wall clock"}


def reference_arm(args, rank, world):
    """The reference path on host cores (its CPU restatement; the reference itself runs only on
    Metal): same config, metric and unit; rank 0 runs, other ranks exit."""
    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0))
    w, _ = get_spec(args.config, 0, args.rows)
    sample = min(w.B, 512)
    xs = np.ascontiguousarray(w.x[:sample])
    for _ in range(min(args.warmup, 3)):
        w.cpu(xs)
    steps, t0 = 0, time.perf_counter()
    while steps < args.steps and (steps < 1 or time.perf_counter() - t0 < 60.0):
        w.cpu(xs)
        steps += 1
    dt = time.perf_counter() - t0
    value = steps * sample / dt
    note = getattr(w, "cpu_note", "")
    line = {"metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": steps, "warmup": min(args.warmup, 3), "ms_per_step": dt * 1e3 / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE shapes and distributions)",
            "config": {"workload": w.name, **w.cfg, "per_step_rows": sample},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port",
                             "sample": f"{sample} rows per step of the same workload; float32 "
                                       f"NumPy restatement of the reference fp32 path (the "
                                       f"reference runs only on Metal){', ' + note if note else ''}"
                                       f"; steps capped at 60 s"},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
