"""CPU: multi-GPU host logic -- shard ranges, row slicing of dense and packed weights, the real
OutputShardedLayer / BatchShardedLayer / gather_into on engine layer objects, and the
batch / output sharded forwards assembled over a world-size-2 gloo process group (the per-rank
compute is the CPU oracle here; on GPUs it is the engine and the collective runs on NCCL)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import kan_oracle as O


def test_shard_range_covers_once():
    from metal_kans.parallel import shard_range

    for n in (0, 1, 7, 16, 4096, 4099):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s, e = shard_range(n, world, r)
                seen.extend(range(s, e))
            assert seen == list(range(n))


def test_packed_row_slices_dequantise_to_row_slices():
    from metal_kans.parallel import slice_2bit_rows, slice_affine_rows

    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.03, (10, 9 * 7)).astype(np.float32)  # rows padded for gs=64
    for bits in (8, 4):
        qw, s, b, pin = O.quantize_affine(w, bits, 64)
        full = O.dequantize_affine_matrix(qw, s, b, bits, 64, w.shape, pin)
        q2, s2, b2 = slice_affine_rows(qw, s, b, 10, pin, 64, 3, 7)
        part = O.dequantize_affine_matrix(q2, s2, b2, bits, 64, (4, w.shape[1]), pin)
        np.testing.assert_array_equal(part, full[3:7])
    p, s = O.quantize_ternary(w, 32)
    p2, s2 = slice_2bit_rows(p, s, 2, 9)
    np.testing.assert_array_equal(O.dequantize_ternary(p2, s2, w.shape[1], 32),
                                  O.dequantize_ternary(p, s, w.shape[1], 32)[2:9])


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from metal_kans.parallel import all_gather_columns, shard_range, slice_dense_rows

        rng = np.random.default_rng(1)
        B, D_in, D_out, K = 6, 8, 13, 5
        x = rng.uniform(-1, 1, (B, D_in)).astype(np.float32)
        W = rng.normal(0, 0.2, (D_out, D_in * K)).astype(np.float32)
        Wb = rng.normal(0, 0.2, (D_out, D_in)).astype(np.float32)
        bias = rng.normal(0, 0.1, D_out).astype(np.float32)
        full = O.kan_layer(x, "cheby", "f32", W, Wb, bias, K=K)
        # output sharding: this rank's weight rows -> its columns -> all-gather
        ranges = [shard_range(D_out, world, r) for r in range(world)]
        s, e = ranges[rank]
        y_loc = O.kan_layer(x, "cheby", "f32", slice_dense_rows(W, s, e),
                            slice_dense_rows(Wb, s, e), bias[s:e], K=K)
        y = all_gather_columns(torch.from_numpy(np.ascontiguousarray(y_loc)), ranges)
        ok_cols = bool(np.array_equal(y.numpy(), full))
        # batch sharding: this rank's rows, gathered back in rank order
        rs, re_ = shard_range(B, world, rank)
        y_rows = torch.from_numpy(np.ascontiguousarray(O.kan_layer(x[rs:re_], "cheby", "f32", W, Wb,
                                                                   bias, K=K)))
        sizes = [shard_range(B, world, r) for r in range(world)]
        width = max(b - a for a, b in sizes)
        pad = torch.zeros((width, D_out))
        pad[: re_ - rs] = y_rows
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
        y_b = torch.cat([p[: b - a] for p, (a, b) in zip(parts, sizes)])
        ok_rows = bool(np.array_equal(y_b.numpy(), full))
        q.put((rank, ok_cols, ok_rows))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_sharded_forwards_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert [r[0] for r in res] == [0, 1]
    assert all(r[1] for r in res), "output-sharded forward differs from the full layer"
    assert all(r[2] for r in res), "batch-sharded forward differs from the full layer"


# ---------------------------------------------------------------------------------------------
# The real sharding classes on engine layer objects.  Layer construction, quantisation (host C++
# in libkan_cuda.so) and row slicing need no GPU: the bridge is bound without initialising a
# device.  Each rank's column block is computed by the oracle from the SLICED layer's own
# (packed) weights, so the test checks what OutputShardedLayer hands to the engine.
# ---------------------------------------------------------------------------------------------

def _deq(q):
    """The oracle's dequantisation of a packed weight object (host NumPy, no device)."""
    if hasattr(q, "qweight"):
        return O.dequantize_affine_matrix(q.qweight, q.scales, q.biases, q.bits, q.group_size,
                                          q.shape, q.padded_in_features)
    if hasattr(q, "codebook"):
        return O.dequantize_int2(q.w_packed, q.scales, q.codebook, q.shape[1], q.group_size)
    return O.dequantize_ternary(q.w_packed, q.scales, q.shape[1], q.group_size)


def _layer_oracle(layer, x):
    """fp32 oracle of an engine layer, its main and base weights from the packed objects."""
    W, Wb = layer.w_cheby, layer.w_base
    if layer._packed("w_cheby") is not None:
        W, Wb = _deq(layer._packed("w_cheby")), _deq(layer._packed("w_base"))
    return O.kan_layer(x, "cheby", "f32", W, Wb, layer.bias, K=layer._terms())


def _real_layers_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import metal_kans as mk
        from metal_kans import device as Dv
        from metal_kans.parallel import BatchShardedLayer, OutputShardedLayer

        Dv.get_metal_bridge = Dv.load_library  # host-only entry points, no device
        # 2-bit dequantisation runs on the GPU in the engine: the oracle's stands in here
        from metal_kans import quantization as Q

        Q.TernaryQuantizedWeight.dequantize = _deq
        Q.Int2QuantizedWeight.dequantize = _deq

        results = []
        for fmt in ("dense", "int8", "int4", "ternary", "int2"):
            np.random.seed(7)
            layer = mk.ChebyKAN(40, 23, degree=5)  # 23 outputs: ragged shards at world 2 and 3
            layer.bias = np.random.default_rng(2).normal(0, 0.1, 23).astype(np.float32)
            if fmt != "dense":
                getattr(mk, "to_" + fmt)(layer, group_size=32 if fmt != "int2" else 16)
            x = np.random.default_rng(3).uniform(-1, 1, (6, 40)).astype(np.float32)
            full = _layer_oracle(layer, x)
            osl = OutputShardedLayer(layer)
            s, e = osl.ranges[rank]
            loc = osl.local
            ok_shape = loc.out_features == e - s and loc.w_cheby.shape[0] == e - s
            if fmt != "dense":  # the packed rows travel with the slice
                for name in ("w_cheby", "w_base"):
                    ok_shape &= bool(np.array_equal(_deq(loc._packed(name)),
                                                    _deq(layer._packed(name))[s:e]))
            y_loc = _layer_oracle(loc, x)
            yt = torch.from_numpy(np.ascontiguousarray(y_loc))
            gathered = torch.empty((world, 6, osl.width), dtype=yt.dtype)
            out = torch.empty((6, 23), dtype=yt.dtype)
            osl.gather_into(yt, gathered, out)
            y_gather = osl.gather(yt)
            ok_out = bool(np.array_equal(out.numpy(), full) and np.array_equal(y_gather.numpy(), full))

            class _Oracle:  # the engine's call signature, oracle arithmetic
                def __call__(self, xs):
                    return _layer_oracle(layer, xs)

            bsl = BatchShardedLayer(_Oracle())
            rs, re_ = bsl.local_rows(6)
            ok_rows = bool(np.array_equal(bsl.forward_local(x), full[rs:re_]))
            results.append((fmt, bool(ok_shape), ok_out, ok_rows))
        q.put((rank, results))
    except Exception as exc:  # report instead of leaving the parent waiting
        q.put((rank, [("error", False, False, repr(exc))]))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 3])
def test_sharding_classes_on_engine_layers_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_real_layers_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(60)
    assert [r[0] for r in res] == list(range(world))
    for rank, results in res:
        for fmt, ok_shape, ok_out, ok_rows in results:
            assert ok_shape, f"rank {rank} {fmt}: sliced layer has the wrong rows"
            assert ok_out, f"rank {rank} {fmt}: gathered output differs from the full layer"
            assert ok_rows, f"rank {rank} {fmt}: batch shard differs from the full layer's rows"
