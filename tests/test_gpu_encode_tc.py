"""Edge cases of the tensor-core encode (k_encode_tc: TMA tiles of 128 H
vectors, tcgen05 tf32 filter, per-warp queue of near ties refined in FP32,
float64 pass for what stays tied) against the C oracle, the reference CPU
encoder's float64 arithmetic (vq.py:154-179). 16-byte aligned inputs with at
least one complete vector take this path; the unaligned case checks the
CUDA-core kernel it falls back to."""
import numpy as np
import pytest

import vq_oracle as o
import vq_oracle_c as oc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from alelyon_compute_kit import ack, cuda, vq  # noqa: E402

# vectors per tile (128 H) for groups 8, 16, 32
TILE = {8: 512, 16: 256, 32: 128}


def u32(t):
    return t.cpu().numpy().view(np.uint32)


def encode(x, book, group):
    codes, status = cuda.encode(torch.from_numpy(x).cuda(), torch.from_numpy(book).cuda(), group)
    return u32(codes), int(status.item())


@pytest.mark.parametrize("group", [8, 16, 32])
def test_tile_and_tail_boundaries(group):
    """Lengths around one vector, one warp, one sub-tile, one tile and one
    full persistent sweep, each with and without a partial last vector."""
    rng = np.random.default_rng(100 + group)
    book = rng.standard_normal((16, group)).astype(np.float32)
    t = TILE[group]
    for vectors in (1, 2, 31, 32, 33, 127, 128, 129, t - 1, t, t + 1, 3 * t + 7, 148 * 2 * t + 5):
        for tail in (0, 1, group - 1):
            n = vectors * group + tail
            x = rng.standard_normal(n).astype(np.float32)
            got, status = encode(x, book, group)
            assert status == 0
            np.testing.assert_array_equal(got, oc.encode(x, book, group), err_msg=f"n={n}")


@pytest.mark.parametrize("group", [8, 16, 32])
def test_every_vector_a_near_tie(group):
    """Midpoints of entry pairs (plus a few ulps of noise): every vector is
    deferred, most reach the float64 pass, and every warp's queue fills
    in every tile."""
    rng = np.random.default_rng(200 + group)
    book = rng.standard_normal((16, group)).astype(np.float32)
    vectors = 40 * TILE[group] + 3
    a = rng.integers(0, 16, vectors)
    b = (a + 1 + rng.integers(0, 15, vectors)) % 16
    mid = (book[a].astype(np.float64) + book[b].astype(np.float64)) / 2
    x = mid.astype(np.float32)
    jitter = rng.random(vectors) < 0.5
    x[jitter] = np.nextafter(x[jitter], np.float32(np.inf))
    x = x.reshape(-1)
    got, status = encode(x, book, group)
    assert status == 0
    np.testing.assert_array_equal(got, oc.encode(x, book, group))


@pytest.mark.parametrize("group", [8, 16, 32])
def test_unaligned_input_takes_the_cuda_core_kernel_and_agrees(group):
    rng = np.random.default_rng(300 + group)
    n = 5000 * group + 3
    x = rng.standard_normal(n).astype(np.float32)
    book = rng.standard_normal((16, group)).astype(np.float32)
    buf = torch.zeros(n + 1, dtype=torch.float32, device="cuda")
    buf[1:] = torch.from_numpy(x).cuda()
    shifted = buf[1:]
    assert shifted.data_ptr() % 16 != 0
    tb = torch.from_numpy(book).cuda()
    c_unaligned, s1 = cuda.encode(shifted, tb, group)
    c_aligned, s2 = cuda.encode(buf[1:].clone(), tb, group)
    cuda.check(s1)
    cuda.check(s2)
    want = oc.encode(x, book, group)
    np.testing.assert_array_equal(u32(c_unaligned), want)
    np.testing.assert_array_equal(u32(c_aligned), want)


@pytest.mark.parametrize("group", [8, 16, 32])
def test_nonfinite_values_are_flagged_and_encoded_like_the_reference(group):
    rng = np.random.default_rng(400 + group)
    n = 3 * TILE[group] * group + 5
    x = rng.standard_normal(n).astype(np.float32)
    book = rng.standard_normal((16, group)).astype(np.float32)
    pos = rng.choice(n, 40, replace=False)
    x[pos[:15]] = np.nan
    x[pos[15:30]] = np.inf
    x[pos[30:]] = -np.inf
    got, status = encode(x, book, group)
    assert status & 1
    np.testing.assert_array_equal(got, oc.encode(x, book, group))


@pytest.mark.parametrize("group", [8, 16, 32])
def test_duplicate_book_rows_and_zero_vectors(group):
    """Duplicate entries tie exactly; the lowest index wins (np.argmin)."""
    rng = np.random.default_rng(500 + group)
    book = rng.standard_normal((16, group)).astype(np.float32)
    book[9] = book[2]
    book[15] = book[2]
    book[4] = 0.0
    vectors = 6 * TILE[group]
    idx = rng.integers(0, 16, vectors)
    x = book[idx].copy()
    x[::7] = 0.0
    x = x.reshape(-1)
    got, status = encode(x, book, group)
    assert status == 0
    np.testing.assert_array_equal(got, oc.encode(x, book, group))


@pytest.mark.parametrize("group", [8, 16, 32])
@pytest.mark.parametrize("scale", [1e-30, 1e-19, 1e17, 3e18])
def test_extreme_magnitudes(group, scale):
    """Subnormal products (the absolute floor of the bound) and squared
    norms near or past FP32 overflow (the float64 pass decides)."""
    rng = np.random.default_rng(600 + group)
    n = 4 * TILE[group] * group
    x = (rng.standard_normal(n) * scale).astype(np.float32)
    book = (rng.standard_normal((16, group)) * scale).astype(np.float32)
    got, status = encode(x, book, group)
    want = oc.encode(x, book, group)
    np.testing.assert_array_equal(got, want)
    assert status in (0, 1)


@pytest.mark.parametrize("group", [8, 16, 32])
def test_fitted_book_on_smooth_data_at_scale(group):
    """2^24 block-normalised Gaussian values with a fitted book: a few per
    cent of the vectors go through the deferred refinement."""
    x = o.block_normalised(o.gaussian(1 << 24, 1.0, 20 + group), group)
    x = np.concatenate([x, o.gaussian(3, 1.0, 1)])
    book = vq.fit_codebook(x, group=group, sample_vectors=65536)
    got, status = encode(x, book, group)
    assert status == 0
    np.testing.assert_array_equal(got, oc.encode(x, book, group))


def test_stalled_status_bit_is_reported():
    """The bounded-wait bit has its own name and makes `check` raise."""
    status = torch.tensor([8], dtype=torch.int32, device="cuda")
    with pytest.raises(ack.AckError, match="stalled"):
        cuda.check(status)
