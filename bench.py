"""Benchmark of the fused KAN forward on B200: rows/s at N GPUs, roofline, CPU baseline, e2e.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl engine|reference]

Default workload (N=1): BASELINE config 2 -- FastKAN RBF layer fp16, B=4096, 256 -> 256,
8 Gaussian centres on [-2, 2], sigma = 4/7 (inv_denominator = 1/sigma^2), input LayerNorm,
SiLU base branch; x ~ N(0,1), W_rbf ~ N(0, 0.1^2), W_base ~ N(0, 1/256); synthetic, seeded.
Other configs (--config c1|c3|c4|c5[:B]) print their own lines.

Timing: W untimed warm-up steps; then K steps, each preceded (outside the timed region) by a
write of a 256 MiB buffer that flushes the 126 MB L2, each timed with CUDA events on the engine's
stream; barrier + synchronize before and after; the max over ranks is reported.  `value` is
whole-job rows/s (all ranks).  `e2e` runs the public NumPy API (`layer(x)`) from pinned host
memory: host->device copy of x, the kernel, device->host copy of y, every step, wall clock.
Multi-GPU (torchrun): the batch is sharded by rank with weights replicated (weak scaling, no
data-path collective); ranks synchronise through torch.distributed (NCCL) only for barriers and
the max-over-ranks reduction.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(REPO, "metal-kans_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "fused KAN layer rows/sec at 1/2/4/8 B200; % tensor-pipe or HBM roofline"


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": p["hbm_gbs"], "tensor": p["bf16_tflops"], "src": "measured"}
    except Exception:
        return {"hbm": 6650.0, "tensor": 1590.0, "src": "fallback"}


# --------------------------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------------------------
class Workload:
    """One BASELINE config: builds the engine object, its synthetic input and the CPU port."""

    def __init__(self, name, B):
        self.name, self.B = name, B


def build_c2(mk, B=4096, seed=0):
    rng = np.random.default_rng(seed)
    np.random.seed(seed)
    l = mk.FastKAN(256, 256, num_centers=8, grid_range=(-2.0, 2.0), bias=True, use_base=True,
                   input_map="layernorm")
    l.inv_denominator = 1.0 / (4.0 / 7.0) ** 2  # 3.0625: exp(-((x-c)/sigma)^2)
    l.w_rbf = rng.normal(0.0, 0.1, (256, 256 * 8)).astype(np.float32)
    l.w_base = rng.normal(0.0, 1.0 / 16.0, (256, 256)).astype(np.float32)
    l.half()
    x = rng.normal(0.0, 1.0, (B, 256)).astype(np.float16)
    w = Workload("FastKAN RBF fp16 256->256, 8 centres, LayerNorm input (BASELINE config 2)", B)
    w.obj, w.x, w.d_out, w.dtype = l, x, 256, "f16"
    w.flops = 2.0 * B * 256 * 256 * (8 + 1)
    w.bytes = x.nbytes + B * 256 * 2 + l.w_rbf.nbytes + l.w_base.nbytes
    w.bound = "tensor"
    w.cfg = {"B": B, "D_in": 256, "D_out": 256, "K": 8, "basis": "rbf", "input_map": "layernorm",
             "sigma": 4 / 7, "grid": [-2.0, 2.0], "has_base": True}

    def cpu(xs):
        from oracle import kan_oracle as O
        return O.kan_layer_cpu_f32(xs.astype(np.float32), "rbf", np.asarray(l.w_rbf, np.float32),
                                   np.asarray(l.w_base, np.float32), np.asarray(l.bias, np.float32),
                                   K=8, grid=np.asarray(l.grid, np.float32),
                                   inv_den=l.inv_denominator, input_map="layernorm")
    w.cpu = cpu
    return w


def build_c1(mk, B=1024, seed=0):
    rng = np.random.default_rng(seed)
    l = mk.ChebyKAN(64, 64, degree=9, bias=False, use_base=False, input_map="tanh")
    l.w_cheby = rng.normal(0, np.sqrt(1 / 576), (64, 576)).astype(np.float32)
    x = rng.uniform(-1, 1, (B, 64)).astype(np.float32)
    w = Workload("ChebyKAN fp32 64->64, T_0..T_8 of tanh(x) (BASELINE config 1)", B)
    w.obj, w.x, w.d_out, w.dtype = l, x, 64, "f32"
    w.flops = 2.0 * B * 64 * 64 * 9
    w.bytes = x.nbytes + B * 64 * 4 + l.w_cheby.nbytes
    w.bound = "tensor"
    w.cfg = {"B": B, "D_in": 64, "D_out": 64, "K": 9, "basis": "cheby", "input_map": "tanh"}

    def cpu(xs):
        from oracle import kan_oracle as O
        return O.kan_layer_cpu_f32(xs, "cheby", np.asarray(l.w_cheby), K=9, input_map="tanh")
    w.cpu = cpu
    return w


BUILDERS = {"c1": build_c1, "c2": build_c2}


# --------------------------------------------------------------------------------------------
# measurement helpers
# --------------------------------------------------------------------------------------------
class Clocks:
    """nvidia-smi sampling during the timed region (200 ms period)."""

    def __init__(self, index):
        self.path = tempfile.mktemp(prefix="kan_clocks_", suffix=".csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [s.strip() for s in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def cpu_baseline(w, budget_s=10.0):
    """Time the CPU port (the reference's fp32 path restated) on a bounded row sample."""
    import threadpoolctl  # noqa: F401  (makes the BLAS thread count explicit)

    cores = len(os.sched_getaffinity(0))
    sample = min(w.B, 512)
    xs = np.ascontiguousarray(w.x[:sample])
    w.cpu(xs)  # warm-up
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        w.cpu(xs)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n * sample / dt, "unit": "rows/s", "cores": cores, "kind": "port",
            "sample": f"{n} calls x {sample} rows of the same workload, float32 NumPy "
                      f"(BLAS on {cores} threads), {dt:.1f} s"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2")
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
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

    lib = mk.get_metal_bridge()
    lib.kan_set_device(local)
    w = BUILDERS[args.config](mk, seed=rank)
    layer = w.obj
    B = w.B
    esz = w.x.dtype.itemsize
    from metal_kans._engine import DeviceBuffer

    dx = DeviceBuffer.from_array(w.x)
    dy = DeviceBuffer(B * w.d_out * esz)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.ExternalStream(lib.kan_default_stream())

    import ctypes

    keep = []
    desc = layer._descriptor(keep)  # weights resident and packed once, outside the timed loop
    pdesc, px, py = ctypes.byref(desc), ctypes.c_void_p(dx.ptr), ctypes.c_void_p(dy.ptr)

    def step():
        lib.kan_forward(pdesc, px, py, B, None)

    for _ in range(args.warmup):
        step()
    lib.kan_stream_synchronize(None)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        lib.kan_stream_synchronize(None)

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    clocks = Clocks(local)
    barrier()
    n0 = lib.kan_launch_count()
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush.zero_()  # L2 flush, outside the timed interval
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
    barrier()
    launches = lib.kan_launch_count() - n0
    clk = clocks.stop()
    times = [a.elapsed_time(b) for a, b in ev]  # ms per step
    total_ms = sum(times)
    if dist is not None:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_step = total_ms / args.steps
    value = world * B * args.steps / (total_ms / 1e3)
    pk = peaks()
    kern_ms = statistics.mean(times)
    if w.bound == "tensor":
        achieved = w.flops / (kern_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": pk["tensor"], "unit": "TFLOP/s",
                "frac": achieved / pk["tensor"], "peak_src": pk["src"],
                "traffic": TRAFFIC.get(args.config), "algorithmic_flops": w.flops}
    else:
        achieved = w.bytes / (kern_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s",
                "frac": achieved / pk["hbm"], "peak_src": pk["src"],
                "traffic": TRAFFIC.get(args.config), "algorithmic_bytes": w.bytes}

    # e2e through the public NumPy API from pinned host memory
    e2e = e2e_measure(mk, w, args, barrier, dist)

    cpu = cpu_baseline(w, args.cpu_seconds) if (rank == 0 and world == 1) else None
    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": w.dtype, "data": "synthetic (seeded; BASELINE distributions)",
            "config": {"workload": w.name, **w.cfg, "per_gpu_rows": B,
                       "parallelism": f"batch-shard x{world}" if world > 1 else "single GPU",
                       "l2": "flushed (256 MiB write) before every timed step"},
            "roofline": roof, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk, "cpu_baseline": cpu,
        }
        print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()


# ncu dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel
# (profiles/*.md), or None when not yet captured for the config.
TRAFFIC = {}


def e2e_measure(mk, w, args, barrier, dist):
    from metal_kans._engine import _Pinned

    lib = mk.get_metal_bridge()
    pin = _Pinned(w.x.nbytes)
    xh = np.frombuffer((np.ctypeslib.ctypes.c_char * w.x.nbytes).from_address(pin.ptr),
                       dtype=w.x.dtype).reshape(w.x.shape)
    xh[...] = w.x
    for _ in range(args.warmup):
        w.obj(xh)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        y = w.obj(xh)
    barrier()
    dt = time.perf_counter() - t0
    if dist is not None:
        import torch

        t = torch.tensor([dt], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    world = dist.get_world_size() if dist is not None else 1
    return {"value": world * w.B * args.steps / dt, "unit": "rows/s",
            "h2d_bytes_per_step": int(w.x.nbytes), "d2h_bytes_per_step": int(y.nbytes),
            "api": f"{type(w.obj).__name__}.forward(numpy, pinned host memory)"}


def reference_arm(args, rank, world):
    """Time the reference's CPU path (oracle port) on this config; rank 0 only."""
    if rank != 0:
        return
    os.environ.setdefault("OPENBLAS_NUM_THREADS", str(len(os.sched_getaffinity(0))))

    class _MK:  # the CPU port needs no GPU: build the weights with NumPy only
        pass

    w = build_cpu_only(args.config)
    cores = len(os.sched_getaffinity(0))
    sample = min(w.B, 512)
    xs = np.ascontiguousarray(w.x[:sample])
    for _ in range(args.warmup):
        w.cpu(xs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        w.cpu(xs)
    dt = time.perf_counter() - t0
    value = args.steps * sample / dt
    line = {"metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {"workload": w.name, **w.cfg, "per_step_rows": sample},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port",
                             "sample": f"{sample} rows per step of the same workload, float32 "
                                       f"NumPy restatement of the reference fp32 path"},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def build_cpu_only(config):
    """Same synthetic weights as the engine arm, without touching a GPU."""
    rng = np.random.default_rng(0)
    from oracle import kan_oracle as O

    if config == "c1":
        W = rng.normal(0, np.sqrt(1 / 576), (64, 576)).astype(np.float32)
        x = rng.uniform(-1, 1, (1024, 64)).astype(np.float32)
        w = Workload("ChebyKAN fp32 64->64, T_0..T_8 of tanh(x) (BASELINE config 1)", 1024)
        w.x, w.cfg = x, {"B": 1024, "D_in": 64, "D_out": 64, "K": 9}
        w.cpu = lambda xs: O.kan_layer_cpu_f32(xs, "cheby", W, K=9, input_map="tanh")
        return w
    W = rng.normal(0.0, 0.1, (256, 2048)).astype(np.float16).astype(np.float32)
    Wb = rng.normal(0.0, 1.0 / 16.0, (256, 256)).astype(np.float16).astype(np.float32)
    x = rng.normal(0.0, 1.0, (4096, 256)).astype(np.float16)
    grid = np.linspace(-2, 2, 8).astype(np.float16).astype(np.float32)
    w = Workload("FastKAN RBF fp16 256->256, 8 centres, LayerNorm input (BASELINE config 2)", 4096)
    w.x = x
    w.cfg = {"B": 4096, "D_in": 256, "D_out": 256, "K": 8, "basis": "rbf",
             "input_map": "layernorm"}
    w.cpu = lambda xs: O.kan_layer_cpu_f32(xs.astype(np.float32), "rbf", W, Wb,
                                           np.zeros(256, np.float32), K=8, grid=grid,
                                           inv_den=3.0625, input_map="layernorm")
    return w


if __name__ == "__main__":
    main()
