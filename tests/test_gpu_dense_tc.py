"""The dense product on the tensor cores (op 16 with the tensor-core flag:
one-hot codes in tensor memory times the projections of X on the codebook
entries, bf16 hi + lo), through `alelyon_compute_kit.cuda` (the C ABI's
device-pointer entry), against float64 with the products' normwise bound
|y - y64| <= 1e-5 * sum_k |x_k w_k|; and against the lookup-table kernels on
the same inputs."""
import numpy as np
import pytest

import vq_oracle as o

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
TOL = 1e-5


def _case(rng, e, m, n, k, group, scale=0.05):
    codes = np.stack([o.pack(rng.integers(0, 16, n * k // group)) for _ in range(e)])
    books = (rng.standard_normal((e, 16, group)) * scale).astype(np.float32)
    x = rng.standard_normal((e, m, k)).astype(np.float32)
    return x, codes, books


def _check(y, x, codes, books, n, k, group):
    for i in range(x.shape[0]):
        wd = o.decode(codes[i], books[i], n * k, group).reshape(n, k).astype(np.float64)
        y64 = x[i].astype(np.float64) @ wd.T
        bound = np.abs(x[i]).astype(np.float64) @ np.abs(wd).T
        err = float(np.max(np.abs(y[i].astype(np.float64) - y64) / np.maximum(bound, 1e-300)))
        assert err <= TOL, (i, err)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("group", [8, 16, 32])
def test_tensor_core_dense_product_within_tolerance(group):
    from alelyon_compute_kit import cuda
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(500 + group)
    # ragged N (a partial 128-row item), M below, at and above one 128-row
    # pass, several experts, K of one and of several code rows
    for (e, m, n, k) in ((2, 8, 300, 32 * group), (3, 16, 129, 64 * group), (1, 64, 517, 32 * group),
                         (2, 37, 256, 96 * group), (1, 130, 200, 32 * group), (1, 1, 128, 32 * group)):
        x, codes, books = _case(rng, e, m, n, k, group)
        tx, tc, tb = (torch.from_numpy(a).to(dev) for a in (x, codes.view(np.int32), books))
        y, st = cuda.dense(tx, tc, tb, n, group, engine="tensor")
        cuda.check(st)
        _check(y.cpu().numpy(), x, codes, books, n, k, group)
        assert cuda.dense_engine(m, k, group) == ("tensor" if m >= cuda.DENSE_TC_MIN_ROWS else "lut")
        y2, st = cuda.dense(tx, tc, tb, n, group, engine="lut")
        cuda.check(st)
        assert float((y - y2).abs().max()) <= 1e-4 * float(y2.abs().max() + 1)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_tensor_core_dense_product_at_the_cfg2_shape():
    """One 11008 x 4096 g16 matrix, M in {8, 16, 64}: every output against
    float64, and the nonfinite flag on a NaN codebook entry."""
    from alelyon_compute_kit import cuda
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(7)
    n, k, group = 11008, 4096, 16
    codes = o.pack(rng.integers(0, 16, n * k // group))[None]
    books = (rng.standard_normal((1, 16, group)) * 0.25).astype(np.float32)
    wd = o.decode(codes[0], books[0], n * k, group).reshape(n, k).astype(np.float64)
    tc_, tb = torch.from_numpy(codes.view(np.int32)).to(dev), torch.from_numpy(books).to(dev)
    for m in (8, 16, 64):
        x = rng.standard_normal((1, m, k)).astype(np.float32)
        y, st = cuda.dense(torch.from_numpy(x).to(dev), tc_, tb, n, group, engine="tensor")
        cuda.check(st)
        y64 = x[0].astype(np.float64) @ wd.T
        bound = np.abs(x[0]).astype(np.float64) @ np.abs(wd).T
        err = float(np.max(np.abs(y.cpu().numpy()[0] - y64) / bound))
        assert err <= TOL, (m, err)
    bad = books.copy()
    bad[0, 3, 5] = np.nan
    _, st = cuda.dense(torch.from_numpy(x).to(dev), tc_, torch.from_numpy(bad).to(dev), n, group, engine="tensor")
    assert int(st.item()) & 1
