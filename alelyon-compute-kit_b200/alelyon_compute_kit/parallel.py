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


def gather_columns(y_local, n_total: int, ranges, group=None, *, layout: str = "columns", out=None):
    """All-gather the column shards Y_r (..., M, n_r) of every rank with one
    NCCL all-gather (gloo on CPU tensors too).

    layout="rank-major": the collective lands in place in a (world, ...,
    M, width) buffer (`out` when given), each rank's slice padded to the
    widest range; nothing is copied after the collective.
    layout="columns": the usual (..., M, n_total), made from the rank-major
    buffer by one strided copy."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    width = max(b - a for a, b in ranges)
    lead = tuple(y_local.shape[:-1])
    if y_local.shape[-1] == width and y_local.is_contiguous():
        send = y_local.view(-1)
    else:
        padded = y_local.new_zeros(lead + (width,))
        padded[..., : y_local.shape[-1]] = y_local
        send = padded.view(-1)
    if out is None:
        out = y_local.new_empty((world,) + lead + (width,))
    dist.all_gather_into_tensor(out.view(-1), send, group=group)
    if layout == "rank-major":
        return out
    if layout != "columns":
        raise ValueError(f"unknown gather layout {layout!r}")
    if all(b - a == width for a, b in ranges):
        # (world, ..., width) -> (..., world, width): one copy, columns in rank order
        order = tuple(range(1, len(lead) + 1)) + (0, len(lead) + 1)
        full = out.permute(order).reshape(lead + (world * width,))
    else:
        full = y_local.new_empty(lead + (n_total,))
        for r, (a, b) in enumerate(ranges):
            full[..., a:b] = out[r][..., : b - a]
    assert full.shape[-1] == n_total
    return full


def dense_sharded(x, codes, book, n_total: int, k: int, group: int, *, gather: bool = True, status=None,
                  layout: str = "columns"):
    """Y = X @ decode(W).T with W (n_total x k) row-sharded over the ranks:
    `codes` is this rank's word slice (from `row_ranges` + `code_slice`),
    `book` the shared codebook, `x` (M, k) replicated. Returns the full Y
    (gather=True; `layout` as in `gather_columns`) or this rank's columns."""
    import torch.distributed as dist

    from . import cuda
    world, rank = dist.get_world_size(), dist.get_rank()
    ranges = row_ranges(n_total, k, group, world)
    a, b = ranges[rank]
    y, status = cuda.dense(x.unsqueeze(0), codes.unsqueeze(0), book.unsqueeze(0), b - a, group, status=status)
    y = y[0]
    if not gather:
        return y, status
    return gather_columns(y, n_total, ranges, layout=layout), status


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
