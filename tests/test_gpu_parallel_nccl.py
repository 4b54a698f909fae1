"""Row-sharded products over NCCL on two GPUs: each rank runs the dense and
the both-coded product on its rows of W and one all-gather assembles Y; the
result must equal the one-GPU product bit for bit (the same kernels and the
same per-row summation order). The M = 1 product with peer stores
(`PeerSlots`: each rank's GEMV writes its rows into every rank's buffer over
NVLink, then step flags) must equal the all-gathered rows bit for bit. Skipped with fewer than two GPUs; the
sharding arithmetic itself is covered on CPU by the gloo tests."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime
    import sys
    from pathlib import Path

    import torch.distributed as dist
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "alelyon-compute-kit_b200"))
    sys.path.insert(0, str(root / "oracle"))
    import vq_oracle as o
    from alelyon_compute_kit import cuda, parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cuda", rank)
        rng = np.random.default_rng(5)
        n, k, group, m = 1000, 512, 16, 3
        codes = o.pack(rng.integers(0, 16, n * k // group))
        book = (rng.standard_normal((16, group)) * 0.1).astype(np.float32)
        x = rng.standard_normal((m, k)).astype(np.float32)
        tcodes = torch.from_numpy(codes.view(np.int32)).to(dev)
        tbook = torch.from_numpy(book).to(dev)
        tx = torch.from_numpy(x).to(dev)
        # the whole product on this GPU
        full, st = cuda.dense(tx.unsqueeze(0), tcodes.unsqueeze(0), tbook.unsqueeze(0), n, group)
        cuda.check(st)
        # this rank's rows, then one all-gather
        lo, hi = parallel.row_ranges(n, k, group, world)[rank]
        w0, w1 = parallel.code_slice(lo * k, hi * k, group)
        y, st = parallel.dense_sharded(tx, tcodes[w0:w1].contiguous(), tbook, n, k, group)
        cuda.check(st)
        same_dense = bool(torch.equal(y.view(torch.int32), full[0].view(torch.int32)))
        # both operands coded: A replicated (m x k), B row-sharded
        a_codes = torch.from_numpy(o.pack(rng.integers(0, 16, m * k // group)).view(np.int32)).to(dev)
        cfull, st = cuda.coded(a_codes, tbook, tcodes, tbook, m, n, k, group, flags=2)
        cuda.check(st)
        c, st = parallel.coded_sharded(a_codes, tbook, tcodes[w0:w1].contiguous(), tbook, m, n, k, group)
        cuda.check(st)
        same_coded = bool(torch.equal(c.view(torch.int32), cfull.view(torch.int32)))
        # M = 1 over many experts (the byte-pair kernel) with peer stores instead of the all-gather
        e, n1, k1 = 64, 1024, 4096
        pcodes = torch.from_numpy(o.pack(rng.integers(0, 16, e * n1 * k1 // group)).view(np.int32)).to(dev)
        pcodes = pcodes.view(e, -1)
        pbooks = tbook.unsqueeze(0).repeat(e, 1, 1).contiguous()
        px = torch.from_numpy(rng.standard_normal((e, 1, k1)).astype(np.float32)).to(dev)
        lo1, hi1 = parallel.row_ranges(n1, k1, group, world)[rank]
        rw = k1 // group // 8
        shard = pcodes.view(e, n1, rw)[:, lo1:hi1].contiguous().view(e, -1)
        st = cuda.status_word(dev)
        yl, _ = cuda.dense(px, shard, pbooks, hi1 - lo1, group, status=st)
        gathered = torch.empty((world, e, hi1 - lo1), device=dev)
        dist.all_gather_into_tensor(gathered.view(-1), yl.contiguous().view(-1))
        slots = parallel.PeerSlots(e, hi1 - lo1)
        try:
            for _ in range(3):   # repeated steps: the flags move by epoch
                got = slots.dense(px, shard, pbooks, hi1 - lo1, group, st)
                torch.cuda.synchronize()
                cuda.check(st)
                same_peer = bool(torch.equal(got.view(torch.int32), gathered.view(torch.int32)))
                dist.barrier()
                if not same_peer:
                    break
        finally:
            slots.close()
            dist.barrier()
        Path(out_dir, f"rank{rank}").write_text(f"{int(same_dense)} {int(same_coded)} {int(same_peer)}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_row_sharded_products_over_nccl_equal_the_single_gpu_product(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "1 1 1"
