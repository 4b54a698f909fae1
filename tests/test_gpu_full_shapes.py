"""Products at the workloads' full shapes, through `alelyon_compute_kit.cuda`
(the C ABI's device-pointer entry), checked against float64 on sampled
outputs: the whole float64 product would take minutes on the host, a sample
of rows x columns takes seconds and sees every code path of the launch.

Tolerance (normwise, the products' bound in every test here):
|y - y64| <= 1e-5 * sum_k |a_k b_k| for each sampled output.
"""
import numpy as np
import pytest

import vq_oracle as o

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
TOL = 1e-5


def _fit(vq, values, group, sample=4096):
    complete = values.numel() // group
    pos = np.linspace(0, complete - 1, min(complete, sample), dtype=np.int64)
    rows = values[: complete * group].view(complete, group)[torch.from_numpy(pos).to(values.device)]
    return vq.fit_codebook(rows.cpu().numpy().reshape(-1), group=group, sample_vectors=sample)


def _decoded_rows(codes, book, rows, k, group):
    """Rows `rows` of a coded (R x k) matrix, decoded on the host in float64."""
    words_per_row = k // group // 8
    c = codes.view(-1, words_per_row)[torch.from_numpy(rows).to(codes.device)].cpu().numpy().view(np.uint32)
    out = np.empty((len(rows), k), np.float64)
    for i in range(len(rows)):
        out[i] = o.decode(c[i], book, k, group)
    return out


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_both_coded_product_at_the_full_cfg3_shape():
    """X 4096 x 4096 (N(0,1), its own g32 book) times W 14336 x 4096
    (N(0, 0.02^2), g32) transposed: 4,096 x 14,336 outputs, 128 group lookups
    each. 4,096 outputs (64 random rows x 64 random columns) against float64."""
    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", 0)
    m, n, k, group = 4096, 14336, 4096, 32
    gen = torch.Generator(device=device)
    gen.manual_seed(8)
    x = torch.randn(m * k, generator=gen, device=device)
    gen.manual_seed(7)
    w = torch.randn(n * k, generator=gen, device=device) * 0.02
    xb, wb = _fit(vq, x, group), _fit(vq, w, group)
    xc, status = cuda.encode(x, torch.from_numpy(xb).to(device), group)
    wc, _ = cuda.encode(w, torch.from_numpy(wb).to(device), group, status=status)
    del x, w
    y, _ = cuda.coded(xc, torch.from_numpy(xb).to(device), wc, torch.from_numpy(wb).to(device), m, n, k, group,
                      flags=2, status=status)
    cuda.check(status)
    rng = np.random.default_rng(33)
    rows = np.sort(rng.choice(m, 64, replace=False))
    cols = np.sort(rng.choice(n, 64, replace=False))
    # the first and last rows and columns too: tile edges of the launch
    rows[0], rows[-1], cols[0], cols[-1] = 0, m - 1, 0, n - 1
    a = _decoded_rows(xc, xb, rows, k, group)
    b = _decoded_rows(wc, wb, cols, k, group)
    got = y[torch.from_numpy(rows).to(device)][:, torch.from_numpy(cols).to(device)].cpu().numpy()
    want = a @ b.T
    bound = np.abs(a) @ np.abs(b).T
    err = np.abs(got.astype(np.float64) - want) / np.maximum(bound, 1e-300)
    assert float(err.max()) <= TOL, float(err.max())
