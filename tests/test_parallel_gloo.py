"""The sharding logic of the multi-GPU path, run as world_size-2 gloo
ranks on the CPU: word-aligned ranges, code slices, column gathers and
expert ranges. Each rank's arithmetic here is the package's CPU encoder or
a numpy product, so what is tested is the partitioning and the assembly,
which the GPU path shares."""
import os
import socket

import numpy as np
import pytest

from alelyon_compute_kit import parallel, vq


def test_word_aligned_ranges_cover_exactly():
    for count, group, world in ((1, 8, 2), (1000, 16, 3), (8 * 32 * 5 + 7, 32, 4), (0, 8, 2), (2 ** 20, 8, 8)):
        ranges = parallel.word_aligned_ranges(count, group, world)
        assert len(ranges) == world and ranges[0][0] == 0 and ranges[-1][1] == count
        for (a, b), (c, _) in zip(ranges, ranges[1:]):
            assert b == c and a % (8 * group) == 0


def test_row_ranges_are_word_aligned():
    for rows, cols, group, world in ((11008, 4096, 16, 8), (14336, 4096, 32, 8), (37, 24, 8, 2), (100, 40, 8, 3)):
        ranges = parallel.row_ranges(rows, cols, group, world)
        assert ranges[0][0] == 0 and ranges[-1][1] == rows
        for a, b in ranges:
            assert (a * cols // group) % 8 == 0


def test_expert_ranges_partition():
    for experts, world in ((64, 8), (5, 2), (1, 4)):
        got = [parallel.expert_range(experts, r, world) for r in range(world)]
        assert sum(b - a for a, b in got) == experts


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        group = 8
        values = rng.standard_normal(8 * group * 9 + 5).astype(np.float32)
        book = rng.standard_normal((16, group)).astype(np.float32)
        a, b = parallel.word_aligned_ranges(values.size, group, world)[rank]
        local = vq.encode(values[a:b], book, group=group).codes if b > a else np.zeros(0, np.uint32)
        pieces = [None] * world
        dist.all_gather_object(pieces, local.tolist())
        joined = np.array([w for p in pieces for w in p], dtype=np.uint32)
        full = vq.encode(values, book, group=group).codes
        ok_encode = bool(np.array_equal(joined, full))
        # column-sharded product assembled by gather_columns
        n, k, m = 37, 24, 3
        w = vq.encode(rng.standard_normal((n, k)).astype(np.float32), book, group=group)
        x = rng.standard_normal((m, k)).astype(np.float32)
        ranges = parallel.row_ranges(n, k, group, world)
        lo, hi = ranges[rank]
        w0, w1 = parallel.code_slice(lo * k, hi * k, group)
        shard = vq.VQArray((hi - lo, k), group, w.codes[w0:w1].copy(), w.codebook) if hi > lo else None
        y_local = torch.from_numpy(x @ shard.decode().T if shard else np.zeros((m, 0), np.float32))
        full_y = parallel.gather_columns(y_local, n, ranges).numpy()
        ok_gather = bool(np.allclose(full_y, x @ w.decode().T, rtol=1e-6, atol=1e-6))
        # in place, rank-major: rank r's padded slice holds its columns
        rm = parallel.gather_columns(y_local, n, ranges, layout="rank-major").numpy()
        want = x @ w.decode().T
        ok_gather &= rm.shape[0] == world and all(
            np.allclose(rm[r][:, : b - a], want[:, a:b], rtol=1e-6, atol=1e-6) for r, (a, b) in enumerate(ranges))
        # equal ranges: the one-copy column layout of (E, M, width) shards
        even = [(r * 5, (r + 1) * 5) for r in range(world)]
        y_even = torch.from_numpy(np.full((2, m, 5), rank, np.float32) + np.arange(5, dtype=np.float32))
        full_even = parallel.gather_columns(y_even, 5 * world, even).numpy()
        expect = np.concatenate([np.full((2, m, 5), r, np.float32) + np.arange(5, dtype=np.float32)
                                 for r in range(world)], axis=-1)
        ok_gather &= bool(np.array_equal(full_even, expect))
        queue.put((rank, ok_encode, ok_gather))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_assemble():
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(results) == [(0, True, True), (1, True, True)]


def test_a_rank_that_dies_is_seen_by_the_other_as_an_error():
    """Failure detection on the host: rank 1 exits before the collective;
    rank 0's collective ends with an error within the process-group timeout."""
    pytest.importorskip("torch")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    outcome = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert outcome == (0, "error")


def _dying_worker(rank, port, queue):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)   # leaves between steps, with nothing in flight
    try:
        dist.all_reduce(torch.ones(1))
        queue.put((0, "completed"))
    except Exception:
        queue.put((0, "error"))
