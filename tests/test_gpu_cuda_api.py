"""The device-pointer entry (`ack_vq_launch`) on PyTorch CUDA tensors:
the same kernels as the handle API, enqueued on the caller's stream.
Sizes here exceed L2 where it matters (2^26 values = 256 MiB)."""
import numpy as np
import pytest

import vq_oracle as o
import vq_oracle_c as oc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from alelyon_compute_kit import ack, cuda  # noqa: E402


def u32(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("group", [8, 16, 32])
def test_large_decode_and_encode_bit_exact(group):
    n = (1 << 26) + 5  # a tail
    rng = np.random.default_rng(group)
    book = rng.standard_normal((16, group)).astype(np.float32)
    vectors = (n + group - 1) // group
    codes = o.pack(rng.integers(0, 16, vectors))
    dev = torch.device("cuda:0")
    tc = torch.from_numpy(codes.view(np.int32)).to(dev)
    tb = torch.from_numpy(book).to(dev)
    values, status = cuda.decode(tc, tb, n, group)
    cuda.check(status)
    want = oc.decode(codes, book, n, group)
    np.testing.assert_array_equal(values.cpu().numpy().view(np.uint32), want.view(np.uint32))
    again, status = cuda.encode(values, tb, group)
    cuda.check(status)
    np.testing.assert_array_equal(u32(again), codes)


def test_encode_of_gaussian_data_matches_c_oracle():
    n, group = 1 << 22, 16
    x = o.block_normalised(o.gaussian(n, 1.0, 10), group)
    from alelyon_compute_kit import vq
    book = vq.fit_codebook(x, group=group, sample_vectors=65536)
    codes, status = cuda.encode(torch.from_numpy(x).cuda(), torch.from_numpy(book).cuda(), group)
    cuda.check(status)
    np.testing.assert_array_equal(u32(codes), oc.encode(x, book, group))


def test_grouped_dense_on_a_side_stream():
    rng = np.random.default_rng(1)
    e, m, n, k, group = 4, 2, 640, 512, 16
    codes = np.stack([o.pack(rng.integers(0, 16, n * k // group)) for _ in range(e)])
    books = rng.standard_normal((e, 16, group)).astype(np.float32)
    x = rng.standard_normal((e, m, k)).astype(np.float32)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        tx = torch.from_numpy(x).cuda()
        tc = torch.from_numpy(codes.view(np.int32)).cuda()
        tb = torch.from_numpy(books).cuda()
        y, status = cuda.dense(tx, tc, tb, n, group)
    side.synchronize()
    cuda.check(status)
    y = y.cpu().numpy()
    for i in range(e):
        y64 = o.dense_nt_f64(x[i], codes[i], books[i], n, k, group)
        wd = o.decode(codes[i], books[i], n * k, group).reshape(n, k).astype(np.float64)
        err = np.max(np.abs(y[i] - y64) / (np.abs(x[i]).astype(np.float64) @ np.abs(wd).T))
        assert err <= 1e-5


def test_launch_refuses_host_tensors_and_mixed_devices():
    with pytest.raises(ack.AckError, match="not a CUDA tensor"):
        cuda.decode(torch.zeros(1, dtype=torch.int32), torch.zeros(16, 8), 8, 8)


def test_concurrent_encodes_with_different_books_on_many_streams():
    """16 encodes with 16 different codebooks, interleaved over 4 streams,
    wrap the constant-bank book slots twice; every result must still be the
    oracle's (a slot is reused only after its previous kernel finished)."""
    from alelyon_compute_kit import vq
    rng = np.random.default_rng(11)
    group, n = 16, 1 << 20
    streams = [torch.cuda.Stream() for _ in range(4)]
    jobs = []
    for i in range(16):
        x = rng.standard_normal(n).astype(np.float32)
        book = rng.standard_normal((16, group)).astype(np.float32)
        jobs.append((x, book))
    outs = []
    for i, (x, book) in enumerate(jobs):
        s = streams[i % 4]
        with torch.cuda.stream(s):
            tx = torch.from_numpy(x).cuda()
            tb = torch.from_numpy(book).cuda()
            codes, status = cuda.encode(tx, tb, group)
            outs.append((codes, status, tx, tb))
    torch.cuda.synchronize()
    for (x, book), (codes, status, _, _) in zip(jobs, outs):
        cuda.check(status)
        np.testing.assert_array_equal(u32(codes), oc.encode(x, book, group))


@pytest.mark.parametrize("group", [8, 16, 32])
def test_tile32_layout_is_bitwise_the_canonical_product(group):
    rng = np.random.default_rng(group + 3)
    for (e, m, n, k) in ((3, 1, 1000, 32 * group), (2, 3, 517, 256 * group), (2, 8, 64, 128 * group),
                         (1, 16, 333, 32 * group), (2, 1, 300, 128 * group), (2, 2, 77, 384 * group),
                         (1, 5, 129, 64 * group)):
        codes = np.stack([o.pack(rng.integers(0, 16, n * k // group)) for _ in range(e)])
        books = rng.standard_normal((e, 16, group)).astype(np.float32)
        x = rng.standard_normal((e, m, k)).astype(np.float32)
        tc = torch.from_numpy(codes.view(np.int32)).cuda()
        tb = torch.from_numpy(books).cuda()
        tx = torch.from_numpy(x).cuda()
        packed, status = cuda.repack_tile32(tc, n, k, group)
        y_t32, _ = cuda.dense(tx, packed, tb, n, group, layout="tile32", status=status)
        y_can, _ = cuda.dense(tx, tc, tb, n, group, status=status)
        cuda.check(status)
        np.testing.assert_array_equal(y_t32.cpu().numpy().view(np.uint32), y_can.cpu().numpy().view(np.uint32))
        wd = o.decode(codes[0], books[0], n * k, group).reshape(n, k).astype(np.float64)
        y64 = x[0].astype(np.float64) @ wd.T
        err = np.max(np.abs(y_t32[0].cpu().numpy() - y64) / (np.abs(x[0]).astype(np.float64) @ np.abs(wd).T))
        assert err <= 1e-5
