"""CPU: multi-GPU host logic -- shard ranges, row slicing of dense and packed weights, and the
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
