"""Sharding the vq4 path across GPUs: one process per GPU, `torch.distributed`.

The reference has no multi-GPU layer (one device per process, chosen by
ACK_DEVICE). The path shards three ways:

* encode / decode: contiguous ranges of whole code words (8 * group values);
  each rank's image is a word-aligned slice of the one-GPU image, so the
  concatenation is bit-for-bit the same. No collective.
* products with coded weights stored N x K: rows of W (output columns of Y)
  split across ranks, activations replicated; each rank computes its Y
  columns and, when a replicated Y is wanted, one NCCL all-gather assembles
  it. A row split is word-aligned when (rows * K / group) % 8 == 0.
* VQAdamW: whole experts per rank. No collective (the clip is per expert).

Row results do not depend on how rows are split, so a sharded product is
bitwise equal to the one-GPU product.
"""
from __future__ import annotations

import math


def word_aligned_ranges(count: int, group: int, world: int) -> list[tuple[int, int]]:
    """Split `count` values into `world` ranges on whole-word boundaries
    (multiples of 8 * group values); the last range takes the tail."""
    if world < 1 or count < 0:
        raise ValueError("world must be positive and count non-negative")
    unit = 8 * group
    words = math.ceil(count / unit)
    per = math.ceil(words / world) if words else 0
    out = []
    for r in range(world):
        w0, w1 = min(words, r * per), min(words, (r + 1) * per)
        out.append((min(count, w0 * unit), min(count, w1 * unit)))
    return out


def row_ranges(rows: int, cols: int, group: int, world: int) -> list[tuple[int, int]]:
    """Split `rows` rows of a coded (rows x cols) matrix into `world` ranges
    whose code slices start on whole words."""
    step = 8 // math.gcd(8, (cols // group) % 8 or 8) if cols % group == 0 else None
    if step is None:
        raise ValueError("row sharding needs cols to be a multiple of the group")
    per = math.ceil(rows / world / step) * step
    return [(min(rows, r * per), min(rows, (r + 1) * per)) for r in range(world)]


def code_slice(start_value: int, stop_value: int, group: int) -> tuple[int, int]:
    """Word range [w0, w1) of the packed image that holds values [start, stop);
    `start_value` must be word-aligned."""
    unit = 8 * group
    if start_value % unit:
        raise ValueError("a code slice must start on a whole word")
    return start_value // unit, math.ceil(math.ceil(stop_value / group) / 8)


def expert_range(experts: int, rank: int, world: int) -> tuple[int, int]:
    """Experts [e0, e1) owned by `rank`."""
    per = math.ceil(experts / world)
    return min(experts, rank * per), min(experts, (rank + 1) * per)


def gather_columns(y_local, n_total: int, ranges, group=None):
    """All-gather the column shards Y_r (..., M, n_r) of every rank into the
    full (..., M, n_total) on every rank (one NCCL all-gather of padded
    shards; works with gloo on CPU tensors too)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    width = max(b - a for a, b in ranges)
    lead = y_local.shape[:-1]
    padded = y_local.new_zeros(lead + (width,))
    padded[..., : y_local.shape[-1]] = y_local
    flat = y_local.new_empty(world * padded.numel())
    dist.all_gather_into_tensor(flat, padded.contiguous().view(-1), group=group)
    out = flat.view((world,) + lead + (width,))
    parts = [out[r][..., : b - a] for r, (a, b) in enumerate(ranges)]
    full = torch.cat(parts, dim=-1)
    assert full.shape[-1] == n_total
    return full


def dense_sharded(x, codes, book, n_total: int, k: int, group: int, *, gather: bool = True, status=None):
    """Y = X @ decode(W).T with W (n_total x k) row-sharded over the ranks:
    `codes` is this rank's word slice (from `row_ranges` + `code_slice`),
    `book` the shared codebook, `x` (M, k) replicated. Returns the full Y
    (gather=True) or this rank's columns."""
    import torch.distributed as dist

    from . import cuda
    world, rank = dist.get_world_size(), dist.get_rank()
    ranges = row_ranges(n_total, k, group, world)
    a, b = ranges[rank]
    y, status = cuda.dense(x.unsqueeze(0), codes.unsqueeze(0), book.unsqueeze(0), b - a, group, status=status)
    y = y[0]
    if not gather:
        return y, status
    return gather_columns(y, n_total, ranges), status


def coded_sharded(a_codes, a_book, b_codes, b_book, m: int, n_total: int, k: int, group: int, *,
                  gather: bool = True, status=None):
    """C = decode(A) @ decode(B).T with B (n_total x k) row-sharded: `b_codes`
    is this rank's word slice; A and both books replicated."""
    import torch.distributed as dist

    from . import cuda
    world, rank = dist.get_world_size(), dist.get_rank()
    ranges = row_ranges(n_total, k, group, world)
    lo, hi = ranges[rank]
    y, status = cuda.coded(a_codes, a_book, b_codes, b_book, m, hi - lo, k, group, flags=2, status=status)
    if not gather:
        return y, status
    return gather_columns(y, n_total, ranges), status
