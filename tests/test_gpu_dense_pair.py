"""The M = 1 dense product through the byte-pair table (k_dense_pair:
Q[p][b] = P[2p][b & 15] + P[2p+1][b >> 4], one shared-memory lookup per code
byte) against the float64 oracle. The canonical layout with one activation
row, K a multiple of 256 g and enough (expert, 32-row) units to fill one
block per SM takes this kernel; the bound is the normwise 1e-5 of every
dense product here."""
import numpy as np
import pytest

import vq_oracle as o

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from alelyon_compute_kit import ack, cuda  # noqa: E402


def normwise(y, x, codes, book, n, k, group):
    y64 = o.dense_nt_f64(x, codes, book, n, k, group)
    wd = o.decode(codes, book, n * k, group).reshape(n, k).astype(np.float64)
    return np.max(np.abs(y - y64) / (np.abs(x).astype(np.float64) @ np.abs(wd).T))


@pytest.mark.parametrize("group", [8, 16, 32])
@pytest.mark.parametrize("chunks,n,e", [(1, 1000, 20), (2, 777, 26), (3, 4096, 5)])
def test_pair_table_product_within_the_normwise_bound(group, chunks, n, e):
    rng = np.random.default_rng(group * 10 + chunks)
    k = 256 * group * chunks
    assert e * ((n + 31) // 32) >= 4 * torch.cuda.get_device_properties(0).multi_processor_count
    codes = np.stack([o.pack(rng.integers(0, 16, n * k // group)) for _ in range(e)])
    books = (rng.standard_normal((e, 16, group)) * 0.02).astype(np.float32)
    x = rng.standard_normal((e, 1, k)).astype(np.float32)
    y, status = cuda.dense(torch.from_numpy(x).cuda(), torch.from_numpy(codes.view(np.int32)).cuda(),
                           torch.from_numpy(books).cuda(), n, group)
    cuda.check(status)
    y = y.cpu().numpy()
    for i in (0, e // 2, e - 1):
        assert normwise(y[i], x[i], codes[i], books[i], n, k, group) <= 1e-5


def test_pair_table_flags_a_nonfinite_book():
    rng = np.random.default_rng(7)
    e, n, group = 20, 1024, 16
    k = 256 * group
    codes = np.stack([o.pack(rng.integers(0, 16, n * k // group)) for _ in range(e)])
    books = rng.standard_normal((e, 16, group)).astype(np.float32)
    books[13, 4, 2] = np.inf
    x = rng.standard_normal((e, 1, k)).astype(np.float32)
    y, status = cuda.dense(torch.from_numpy(x).cuda(), torch.from_numpy(codes.view(np.int32)).cuda(),
                           torch.from_numpy(books).cuda(), n, group)
    with pytest.raises(ack.AckError, match="nonfinite"):
        cuda.check(status)
    y = y.cpu().numpy()
    assert normwise(y[0], x[0], codes[0], books[0], n, k, group) <= 1e-5


def test_pair_table_agrees_with_the_tile32_kernel_at_cfg2_shape():
    """768 experts of 11008 x 4096 (g16) would be 1 GB; 96 experts keep the
    shape per expert. The two kernels sum in different orders, so they agree
    to the FP32 rounding of a 4096-term dot product."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    e, n, k, group = 96, 11008, 4096, 16
    words = n * k // group // 8
    codes = torch.randint(-2**31, 2**31 - 1, (e, words), generator=gen, device="cuda", dtype=torch.int32)
    books = torch.randn((e, 16, group), generator=gen, device="cuda") * 0.02
    x = torch.randn((e, 1, k), generator=gen, device="cuda")
    y_pair, st = cuda.dense(x, codes, books, n, group)
    packed, st2 = cuda.repack_tile32(codes, n, k, group)
    y_t32, _ = cuda.dense(x, packed, books, n, group, layout="tile32", status=st2)
    cuda.check(st)
    cuda.check(st2)
    scale = (x.abs() @ torch.ones(k, 1, device="cuda")).max().item() * books.abs().max().item()
    assert (y_pair - y_t32).abs().max().item() <= 1e-5 * scale
    i = 7
    c = codes[i].cpu().numpy().view(np.uint32)
    assert normwise(y_pair[i].cpu().numpy(), x[i].cpu().numpy(), c, books[i].cpu().numpy(), n, k, group) <= 1e-5
