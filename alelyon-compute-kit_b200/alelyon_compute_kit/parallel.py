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

`PeerSlots` replaces the all-gather of the M = 1 dense product by peer
stores: every rank's byte-pair GEMV writes its Y shard into its slot of
every rank's rank-major buffer (CUDA IPC mappings over NVLink, no multicast
object), then a step flag is published to every rank and awaited (bounded).
The result is the all-gathered buffer, bit for bit, without a separate
collective after the product.
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


class _CudaBuffer:
    """A device allocation of the library's, seen by PyTorch without a copy."""

    def __init__(self, ptr: int, shape, device):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.device = device


class PeerSlots:
    """A rank-major (world, E, width) float32 buffer on every rank, each
    rank's slot written by that rank's product straight into every other
    rank's buffer, and one u32 step flag per (receiver, sender).

    `dense(x, codes, books, n, group)` runs this rank's op-16 product (M = 1,
    W stored n x K, the byte-pair kernel's shapes) with peer stores, then
    publishes the step and waits (bounded; a wait that runs out sets the
    stalled bit of `status`) until every rank has published it. After the
    wait, `tensor()` holds every rank's rows. Slots are rewritten by the next
    call on any rank: read them before the next call, or `torch.distributed`
    barrier first. `close()` unmaps and frees (call it on every rank)."""

    def __init__(self, experts: int, width: int, group=None, device=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import ack
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > 8:
            raise ack.AckError("peer slots hold at most 8 ranks")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.experts, self.width = experts, width
        self.slot = experts * width * 4
        self.flags_off = self.world * self.slot
        self._lib = ack._lib()
        c = self._lib.cdll
        for name, args in (("ack_peer_alloc", [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
                           ("ack_peer_open", [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
                           ("ack_peer_close", [ctypes.c_void_p]), ("ack_peer_free", [ctypes.c_void_p]),
                           ("ack_vq_dense_peers", [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                                   ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]),
                           ("ack_peer_signal", [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                                ctypes.c_void_p]),
                           ("ack_peer_wait", [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                              ctypes.c_uint32, ctypes.c_void_p])):
            getattr(c, name).argtypes = args
            getattr(c, name).restype = ctypes.c_int32
        # every rank reaches every collective below, and all give up together
        # if any rank's allocation or mapping fails (no rank is left waiting)
        ptr, handle = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
        with torch.cuda.device(self.device):
            rc = c.ack_peer_alloc(self.flags_off + 256, ctypes.byref(ptr), handle)
        mine = bytes(handle) if rc == ack.ACK_OK else None
        error = None if rc == ack.ACK_OK else self._lib.last_error()
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        self.base = [0] * self.world
        self._opened = []
        if mine is not None:
            self.base[self.rank] = ptr.value
        if all(h is not None for h in handles):
            with torch.cuda.device(self.device):
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    peer = ctypes.c_void_p()
                    h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                    if c.ack_peer_open(h, ctypes.byref(peer)) != ack.ACK_OK:
                        error = error or self._lib.last_error()
                        break
                    self.base[r] = peer.value
                    self._opened.append(peer.value)
        else:
            error = error or "a peer rank could not allocate its buffer"
        ok = torch.tensor([0 if error else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            self.close()
            raise ack.AckError(f"peer slots unavailable: {error or 'another rank failed'}")
        others = [self.base[r] + self.rank * self.slot for r in range(self.world) if r != self.rank]
        self._peers = (ctypes.c_void_p * max(1, len(others)))(*others)
        self._flags = (ctypes.c_void_p * self.world)(*[b + self.flags_off for b in self.base])
        self._view = _CudaBuffer(ptr.value, (self.world, experts, width), self.device)
        self._tensor = torch.as_tensor(self._view, device=self.device)
        self.epoch = 0

    def tensor(self):
        """The rank-major (world, E, width) buffer (valid after `dense`)."""
        return self._tensor

    def dense(self, x, codes, books, n: int, group: int, status):
        import ctypes

        import torch

        from . import ack, cuda
        e, m, k = x.shape
        if m != 1 or n != self.width or e != self.experts:
            raise ack.AckError("peer slots hold (experts, width) rows of an M = 1 product")
        out = self._tensor[self.rank].view(e, 1, n)
        plan = cuda.plan2(cuda.OP_DENSE, 1, n, k, group, flags=2, batch=e)
        ops = ack.AckVqOperands()
        ops.size = ctypes.sizeof(ops)
        ops.nslots = 8
        for i, t in enumerate((x, codes, books, None, None, out, None, status)):
            if t is not None:
                ops.ptr[i] = t.data_ptr()
                ops.bytes[i] = t.numel() * t.element_size()
        c = self._lib.cdll
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        self.epoch += 1
        rc = c.ack_vq_dense_peers(plan, len(plan), ctypes.byref(ops), self._peers, self.world - 1, stream)
        if rc == ack.ACK_OK:
            rc = c.ack_peer_signal(self._flags, self.world, self.rank, self.epoch, stream)
        if rc == ack.ACK_OK:
            rc = c.ack_peer_wait(ctypes.c_void_p(self.base[self.rank] + self.flags_off), self.world, self.epoch,
                                 ctypes.c_void_p(status.data_ptr()), 0, stream)
        if rc != ack.ACK_OK:
            raise ack._kit_error("vq2-dense-peers", rc, self._lib.last_error())
        return self._tensor

    def close(self):
        import torch
        c = self._lib.cdll
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                c.ack_peer_close(p)
            self._opened = []
            if self.base[self.rank]:
                c.ack_peer_free(self.base[self.rank])
                self.base[self.rank] = 0
