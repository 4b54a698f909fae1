"""The encode entry that allocates nothing (`ack_vq_encode_noalloc`), called
through the C ABI with device pointers, against the library's regular
device-pointer encode (`ack_vq_launch`, op 21) on the same inputs, and
against the reference's float64 encoder restated in C (`oracle/`).

It exists for callers that cannot allocate device memory at the point of
the call (a host whose own allocator owns all device memory, or code where an
allocation would stall or be refused); its only scratch is a fixed array
inside the library. Encode output is compared bit for bit, as every encode
test here is. This file is collected last so that a run stopping at the
first failure has run every other test; it passes alone as well.
"""
import ctypes

import numpy as np
import pytest

import vq_oracle_c as oc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _entry():
    from alelyon_compute_kit import ack
    lib = ack._lib()
    fn = lib.cdll.ack_vq_encode_noalloc
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return lib, fn


def _words(count, group):
    return ((count + group - 1) // group + 7) // 8


def _inputs(seed, batch, count, group, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((batch, count), generator=g, device=device)
    books = torch.randn((batch, 16, group), generator=g, device=device) * 0.5
    # some vectors equal to book rows, so exact ties and the float64 pass occur
    full = count // group
    for b in range(batch):
        rows = x[b, : full * group].view(full, group)
        rows[: min(full, 64)] = books[b, torch.arange(min(full, 64), device=device) % 16]
    return x, books


def _run_noalloc(fn, x, books, group, stream):
    batch, count = x.shape
    codes = torch.full((batch, _words(count, group)), -1, dtype=torch.int32, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    rc = fn(x.data_ptr(), count, batch, books.data_ptr(), group, codes.data_ptr(), status.data_ptr(),
            stream.cuda_stream)
    return rc, codes, status


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("group", [8, 16, 32])
def test_noalloc_encode_equals_the_regular_entry_on_two_calls_in_a_row(group):
    from alelyon_compute_kit import ack, cuda
    lib, fn = _entry()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    # two calls in a row on different data, books and batch sizes: the second
    # must not see anything the first left in the shared scratch
    for seed, batch, count in ((11, 5, 4099 * group // 8 + 3), (12, 3, 1 << 16)):
        x, books = _inputs(seed + group, batch, count, group, device)
        rc, codes, status = _run_noalloc(fn, x, books, group, stream)
        assert rc == ack.ACK_OK, lib.last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        for b in range(batch):
            want, st = cuda.encode(x[b].contiguous(), books[b].contiguous(), group)
            cuda.check(st)
            np.testing.assert_array_equal(codes[b].cpu().numpy(), want.cpu().numpy())
            # and the reference's float64 encoder, restated in C on the host
            host = oc.encode(x[b].cpu().numpy(), books[b].cpu().numpy(), group)
            np.testing.assert_array_equal(codes[b].cpu().numpy().view(np.uint32), host)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("group", [8, 16, 32])
def test_noalloc_encode_flags_nonfinite_values_and_books_like_the_regular_entry(group):
    """A NaN in a complete vector, an infinity in the partial last vector and
    a NaN in one tensor's book: per tensor, the codes and the status word
    equal the regular entry's; a batch call's status is their OR."""
    from alelyon_compute_kit import ack, cuda
    lib, fn = _entry()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    batch, count = 4, 37 * group + 5
    x, books = _inputs(90 + group, batch, count, group, device)
    x[0, 3 * group + 1] = float("nan")      # a complete vector
    x[1, count - 2] = float("inf")          # the partial last vector
    books[2, 7, group - 1] = float("nan")   # a book entry
    want_all = 0
    for b in range(batch):
        rc, codes, status = _run_noalloc(fn, x[b:b + 1].contiguous(), books[b:b + 1].contiguous(), group, stream)
        assert rc == ack.ACK_OK, lib.last_error()
        want, st = cuda.encode(x[b].contiguous(), books[b].contiguous(), group)
        torch.cuda.synchronize()
        assert int(status.item()) == int(st.item()), b
        want_all |= int(st.item())
        np.testing.assert_array_equal(codes[0].cpu().numpy(), want.cpu().numpy())
    assert want_all == 1
    rc, codes, status = _run_noalloc(fn, x, books, group, stream)
    assert rc == ack.ACK_OK, lib.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == want_all
    for b in range(batch):
        want, _ = cuda.encode(x[b].contiguous(), books[b].contiguous(), group)
        np.testing.assert_array_equal(codes[b].cpu().numpy(), want.cpu().numpy())


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_noalloc_encode_refuses_what_its_scratch_cannot_hold():
    from alelyon_compute_kit import ack
    lib, fn = _entry()
    device = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(device)
    x, books = _inputs(3, 65, 64, 16, device)
    rc, _, _ = _run_noalloc(fn, x, books, 16, stream)
    assert rc == ack.ACK_ERR_SIZE
    assert "exceeds the 64 books" in lib.last_error()
    rc, _, _ = _run_noalloc(fn, x[:2], books[:2], 12, stream)
    assert rc == ack.ACK_ERR_SHAPE
    assert fn(None, 64, 1, books.data_ptr(), 16, None, None, stream.cuda_stream) == ack.ACK_ERR_NULL
