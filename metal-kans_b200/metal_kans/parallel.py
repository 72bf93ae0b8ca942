"""Multi-GPU execution of KAN layers: one process per GPU (torch.distributed, NCCL over NVLink).

Two strategies, chosen by batch size (the reference is single-device; both are new):

* batch sharding -- rows are split contiguously over the ranks and every rank holds the whole
  layer; no collective touches the data path (large batches: every row is independent);
* output sharding -- rank r owns output columns [r*D_out/n, (r+1)*D_out/n): the rows of W, W_base,
  bias and of the packed quantised arrays (quantisation groups never cross a weight row, so packed
  data split cleanly by row); each rank computes Y[:, its columns] and an all-gather over NVLink
  assembles Y (small, wide batches whose cost is streaming the weights: each GPU streams 1/n).

The slicing helpers below are plain array functions (no device needed); the layer wrappers run
the engine on the rank's GPU.
"""
from __future__ import annotations

import copy
from typing import Dict, Optional, Tuple

import numpy as np


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of n items for `rank` of `world` (first n % world ranks get one
    extra)."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


# ---------------------------------------------------------------------------------------------
# row slicing of weights (dense and packed), device-free
# ---------------------------------------------------------------------------------------------

def slice_dense_rows(w: np.ndarray, start: int, stop: int) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(w)[start:stop])


def slice_affine_rows(qweight, scales, biases, rows: int, padded_cols: int, group_size: int,
                      start: int, stop: int):
    """INT8/INT4 QuantizedWeight arrays of rows [start, stop): groups are consecutive `group_size`
    elements of the row-padded matrix, so a row owns groups [row*gpr, (row+1)*gpr)."""
    gpr = padded_cols // group_size
    sl = slice(start * gpr, stop * gpr)
    return (np.ascontiguousarray(qweight[sl]), np.ascontiguousarray(scales[sl]),
            np.ascontiguousarray(biases[sl]))


def slice_2bit_rows(w_packed, scales, start: int, stop: int):
    """Ternary/INT2 arrays of rows [start, stop) (both are [rows][...] already)."""
    return np.ascontiguousarray(w_packed[start:stop]), np.ascontiguousarray(scales[start:stop])


def slice_packed(q, start: int, stop: int):
    """A packed weight object restricted to rows [start, stop) (same class, same layout)."""
    from .quantization import QuantizedWeight

    r = copy.copy(q)
    r.__dict__.pop("_dev_bufs", None)
    rows = stop - start
    if isinstance(q, QuantizedWeight):
        r.qweight, r.scales, r.biases = slice_affine_rows(
            q.qweight, q.scales, q.biases, q.shape[0], q.padded_in_features, q.group_size,
            start, stop)
    else:
        r.w_packed, r.scales = slice_2bit_rows(q.w_packed, q.scales, start, stop)
    r.shape = (rows, q.shape[1])
    return r


def slice_layer_outputs(layer, start: int, stop: int):
    """A copy of `layer` computing only outputs [start, stop): weight rows, bias entries and
    packed weights sliced; basis parameters (grid, translations, scales) shared."""
    from ._layer import PACKED_SUFFIXES

    new = copy.copy(layer)
    d = new.__dict__
    for k in ("_dev_cache", "_tc_cache", "_scratch_bufs", "_keepalive", "_desc_cache"):
        d.pop(k, None)
    d["_versions"] = dict(layer.__dict__.get("_versions", {}))
    new.out_features = stop - start
    for name in (layer.MAIN, "w_base"):
        if name == "w_base" and not layer.has_base:
            continue
        q = layer._packed(name)
        object.__setattr__(new, name, slice_dense_rows(getattr(layer, name), start, stop))
        getattr(new, name).flags.writeable = False
        for suf in PACKED_SUFFIXES:
            d.pop(f"_{name}{suf}", None)
        if q is not None:
            qs = slice_packed(q, start, stop)
            qs._source_version = d["_versions"].get(name, 0)
            suffix = next(s for s in PACKED_SUFFIXES if layer.__dict__.get(f"_{name}{s}") is q)
            d[f"_{name}{suffix}"] = qs
    if layer.has_bias:
        object.__setattr__(new, "bias", slice_dense_rows(layer.bias, start, stop))
        new.bias.flags.writeable = False
    return new


def assemble_columns(parts, widths) -> np.ndarray:
    """Y[B, sum(widths)] from per-rank column blocks Y_r[B, widths[r]]."""
    return np.concatenate([np.asarray(p)[:, :w] for p, w in zip(parts, widths)], axis=1)


# ---------------------------------------------------------------------------------------------
# layer wrappers (one process per GPU)
# ---------------------------------------------------------------------------------------------

class BatchShardedLayer:
    """Each rank runs the full layer on its contiguous share of the batch (no collective)."""

    def __init__(self, layer, group=None):
        import torch.distributed as dist

        self.layer = layer
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def local_rows(self, B: int) -> Tuple[int, int]:
        return shard_range(B, self.world, self.rank)

    def forward_local(self, x_full: np.ndarray) -> np.ndarray:
        s, e = self.local_rows(x_full.shape[0])
        return self.layer(x_full[s:e])


class OutputShardedLayer:
    """Rank r owns output columns shard_range(D_out, world, r); Y is assembled by an all-gather
    over the process group (NCCL over NVLink on GPUs, gloo in the CPU tests)."""

    def __init__(self, layer, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.d_out = layer.out_features
        self.ranges = [shard_range(self.d_out, self.world, r) for r in range(self.world)]
        s, e = self.ranges[self.rank]
        self.local = slice_layer_outputs(layer, s, e)
        self.width = max(b - a for a, b in self.ranges)

    def gather(self, y_local):
        """Y[B, D_out] (torch tensor on y_local's device) from this rank's column block."""
        return all_gather_columns(y_local, self.ranges, self.group)

    def gather_into(self, y_local, gathered, out):
        """Allocation-free gather for a steady-state loop: ``gathered`` [world, B, width] and
        ``out`` [B, D_out] are preallocated; one all-gather, then one strided copy (equal
        shards) or one copy per rank (ragged shards) puts the column blocks in place."""
        import torch.distributed as dist

        B, w = y_local.shape
        src = y_local
        if w != self.width:
            pad = self.__dict__.get("_pad")
            if pad is None or pad.shape[0] != B:
                import torch

                pad = torch.zeros((B, self.width), dtype=y_local.dtype, device=y_local.device)
                self._pad = pad
            pad[:, :w] = y_local
            src = pad
        # the output as [world * B, width]: NCCL takes any shape of the right size, gloo splits
        # dim 0 into per-rank blocks of the input's shape
        dist.all_gather_into_tensor(gathered.view(self.world * B, self.width), src,
                                    group=self.group)
        if all(b - a == self.width for a, b in self.ranges):
            out.view(B, self.world, self.width).copy_(gathered.permute(1, 0, 2))
        else:
            for r, (a, b) in enumerate(self.ranges):
                out[:, a:b].copy_(gathered[r, :, : b - a])
        return out

    def forward(self, x: np.ndarray) -> np.ndarray:
        """Full-width Y for host input x (every rank passes the same x and gets the same Y):
        upload, this rank's column block on the engine's kernels (on torch's current stream),
        all-gather over the process group, download."""
        import torch

        from . import _engine as E

        act = self.local.dtype
        x2, orig = E.as_activation(x, act, self.local.in_features)
        B = x2.shape[0]
        tdt = _TORCH_DT[np.dtype(act).name]
        xt = torch.from_numpy(x2.view(np.int16) if tdt == torch.bfloat16 else x2)
        if tdt == torch.bfloat16:
            xt = xt.view(torch.bfloat16)
        dev = torch.device("cuda", torch.cuda.current_device())
        dx = xt.to(dev, non_blocking=True)
        y_loc = torch.empty((B, self.local.out_features), dtype=tdt, device=dev)
        self.local.forward_device(dx.data_ptr(), y_loc.data_ptr(), B,
                                  torch.cuda.current_stream().cuda_stream)
        y = self.gather(y_loc).cpu()
        out = (y.view(torch.int16).numpy().view(act) if tdt == torch.bfloat16 else y.numpy())
        return E.restore_shape(out, orig, self.d_out)

    __call__ = forward


def _torch_dtypes():
    import torch

    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


class _LazyDt(dict):
    def __missing__(self, k):
        self.update(_torch_dtypes())
        return dict.__getitem__(self, k)


_TORCH_DT = _LazyDt()


def all_gather_columns(y_local, ranges, group=None):
    """All-gather per-rank column blocks Y_r[B, b_r - a_r] (torch tensors) into Y[B, D_out]:
    blocks are padded to a common width for the collective and cut back after it."""
    import torch
    import torch.distributed as dist

    B = y_local.shape[0]
    width = max(b - a for a, b in ranges)
    pad = torch.zeros((B, width), dtype=y_local.dtype, device=y_local.device)
    pad[:, : y_local.shape[1]] = y_local
    parts = [torch.empty_like(pad) for _ in ranges]
    dist.all_gather(parts, pad.contiguous(), group=group)
    return torch.cat([p[:, : b - a] for p, (a, b) in zip(parts, ranges)], dim=1)
