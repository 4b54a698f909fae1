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


@pytest.mark.parametrize("m,engine,layout", [(1, "lut", "canonical"), (2, "lut", "canonical"),
                                             (4, "lut", "tile32"), (16, "lut", "tile32"),
                                             (64, "tensor", "canonical")])
def test_dense_flags_nonfinite_activations(m, engine, layout):
    """Every dense engine reports a NaN or infinity in X (or an overflowed
    sum) in the status word, as the wire API refuses nonfinite input: the
    byte-pair GEMV (M = 1, K a multiple of 256 g), the LUT kernels and the
    tensor-core product. A finite X leaves the word clear."""
    group, n, k, e = 16, 11008, 4096, 2   # M = 1: 688 row batches, enough for the byte-pair kernel
    rng = np.random.default_rng(70 + m)
    dev = torch.device("cuda:0")
    codes = torch.from_numpy(o.pack(rng.integers(0, 16, e * n * k // group)).view(np.int32)).to(dev).view(e, -1)
    books = torch.from_numpy(rng.standard_normal((e, 16, group)).astype(np.float32) * 0.05).to(dev)
    run = codes if layout == "canonical" else cuda.repack_tile32(codes, n, k, group)[0]
    ws = (torch.empty(cuda.dense_tc_workspace_bytes(m, k, group, e), dtype=torch.uint8, device=dev)
          if engine == "tensor" else None)
    x = torch.from_numpy(rng.standard_normal((e, m, k)).astype(np.float32)).to(dev)
    _, status = cuda.dense(x, run, books, n, group, layout=layout, engine=engine, workspace=ws)
    assert int(status.item()) == 0
    for bad in (float("nan"), float("inf")):
        xb = x.clone()
        xb[e - 1, m - 1, k // 2 + 3] = bad
        _, status = cuda.dense(xb, run, books, n, group, layout=layout, engine=engine, workspace=ws)
        assert int(status.item()) & 1, (bad, m, engine)


def test_resident_product_refuses_nonfinite_activations():
    """The resident-weights product checks X on the device, not by a host
    pass, and refuses a nonfinite X with the wire API's error type."""
    from alelyon_compute_kit import vq
    group, n, k, e = 16, 512, 4096, 2
    rng = np.random.default_rng(9)
    ws = [vq.VQArray((n, k), group, o.pack(rng.integers(0, 16, n * k // group)),
                     rng.standard_normal((16, group)).astype(np.float32) * 0.05) for _ in range(e)]
    x = rng.standard_normal((e, 1, k)).astype(np.float32)
    with ack.Device() as d:
        backend = vq.VQDevice(d)
        with backend.resident(vq.VQStack.from_arrays(ws), layout="canonical") as weights:
            backend.matmul_dense_grouped(x, weights)
            x[1, 0, 7] = np.nan
            with pytest.raises(ValueError, match="finite"):
                backend.matmul_dense_grouped(x, weights)
            with pytest.raises(ValueError, match="finite"):
                backend.matmul_dense_grouped(x.astype(np.float64), weights)
