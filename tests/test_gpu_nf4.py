"""The NF4 comparator on the GPU, bit for bit against the restatement of
the reference's law (oracle/nf4_oracle.py, itself pinned to the shaders in
test_nf4_oracle.py), on the reference's own test shapes
(src/alelyon_compute_kit/_kit/tests/nf4_gemv_abi.rs:485-595,
nf4_decode_abi.rs): whole-source and selected decodes in FP32, bf16 and fp16;
the grouped GEMV with 0 to 16 rows a group, a pitch wider than K, columns
straddling members, more columns than one grid dimension, and fp16
subnormals."""
import numpy as np
import pytest

import nf4_cases as nc
import nf4_oracle as no

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from alelyon_compute_kit import ack, nf4  # noqa: E402

DEV = "cuda:0"


def _t(a, dtype=None):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a.copy()).to(DEV)


def _src(g):
    return (_t(g["packed"]), _t(g["absmax_q"]), _t(g["absmax2"]), _t(g["tables"]), _t(g["starts"]),
            _t(g["offsets"]))


def _host(g):
    return (g["packed"], g["absmax_q"], g["absmax2"], g["tables"], g["starts"], g["offsets"])


def _bits(x):
    return x.cpu().numpy().view(np.uint16 if x.dtype == torch.int16 else np.uint32)


@pytest.mark.parametrize("storage", ["f32", "bf16", "f16"])
def test_decode_is_the_law(storage):
    code = nf4.STORAGE[storage]
    g = nc.source(21, 4, 2 * no.NESTED_VALUES, base_blocks=1)
    n = 4 * 2 * no.NESTED_VALUES - 3
    got = nf4.decode(*_src(g), n, src_base=g["base"], storage=storage)
    want = no.decode(*_host(g), n, src_base=g["base"], storage=code)
    np.testing.assert_array_equal(_bits(got), want.view(np.uint32 if code == 0 else np.uint16))
    ids = np.array([3, 1, 1, 9, -2, 0], np.int64)
    got = nf4.decode(*_src(g), 6 * 8192, ids=_t(ids), member_values=8192, src_base=g["base"], storage=storage)
    want = no.decode(*_host(g), 6 * 8192, ids=ids, member_values=8192, src_base=g["base"], storage=code)
    np.testing.assert_array_equal(_bits(got), want.view(np.uint32 if code == 0 else np.uint16))


def _gemv_case(g, experts, per_expert, n, k, lda, elem, scale=1.0, seed=0):
    table, rows = nc.weight_groups(experts, per_expert)
    rows = max(rows, 1)
    a16 = nc.activations(seed, rows, lda, elem, scale)
    got = nf4.gemv(_t(a16), *_src(g), _t(table), rows=rows, n=n, k=k, lda=lda, src_base=g["base"],
                   elem="bf16" if elem == 0 else "f16")
    want = no.gemv(a16, *_host(g), table, rows=rows, n=n, k=k, lda=lda, src_base=g["base"], elem=elem)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
    return want


@pytest.mark.parametrize("elem", [0, 1])
def test_gemv_follows_the_documented_order(elem):
    nv = no.NESTED_VALUES
    # four routed experts of 2 members each (W 128 x 256), rows 5, 0, 16, 1, one nested block of filler
    gu = nc.source(22, 8, nv, base_blocks=1)
    _gemv_case(gu, [(2, 5), (1, 0), (0, 16), (3, 1)], 2 * nv, 128, 256, 256, elem, seed=1)
    # an attention-sized weight 512 x 2048 at 1, 3 and 16 rows, the 16 with a pitch wider than K
    attn = nc.source(23, 1, 64 * nv)
    for rows, lda in ((1, 2048), (3, 2048), (16, 2056)):
        _gemv_case(attn, [(0, rows)], 0, 512, 2048, lda, elem, seed=rows)
    # columns of 24,576 values over members of 16,384: every column straddles a member boundary
    st = nc.source(24, 3, nv)
    _gemv_case(st, [(0, 2)], 0, 2, 3 * nv // 2, 3 * nv // 2, elem, seed=9)


def test_gemv_more_columns_than_one_grid_dimension():
    wide = nc.source(25, 1, 274 * no.NESTED_VALUES)
    _gemv_case(wide, [(0, 2)], 0, 70_000, 64, 64, 1, seed=3)


def test_gemv_fp16_subnormals():
    tiny = nc.source(26, 1, 64 * no.NESTED_VALUES)
    tiny["absmax2"] = (2.0e-6 + (np.arange(len(tiny["absmax2"])) % 7) * 7.0e-6).astype(np.float32)
    tiny["offsets"][:] = 0
    for rows in (1, 3, 16):
        want = _gemv_case(tiny, [(0, rows)], 0, 512, 2048, 2048, 1, scale=1.0e-5, seed=rows)
        assert np.abs(want).max() > 0


def test_gemv_groups_the_call_does_not_cover_write_nothing():
    """The kernel's own guards: a group with no rows, past the rows, or a
    weight base off a word leaves its rows of C as they were."""
    g = nc.source(27, 2, no.NESTED_VALUES)
    table = np.array([[0, 2, 0], [2, 0, 0], [2, 3, 4], [5, 2, 8192]], np.uint32)   # base 4: not whole words
    a16 = nc.activations(4, 7, 256, 0)
    c = torch.full((7, 64), 7.0, device=DEV)
    nf4.gemv(_t(a16), *_src(g), _t(table), rows=7, n=64, k=256, out=c)
    want = no.gemv(a16, *_host(g), table, rows=7, n=64, k=256, c=np.full((7, 64), 7.0, np.float32))
    np.testing.assert_array_equal(c.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert (c[2:5].cpu().numpy() == 7.0).all()


def test_handle_entries_bind_as_the_reference():
    """ack_nf4_decode and ack_gemv_nf4 on device buffers (the reference's
    entries), same words as the tensor API; ms_out reads NaN."""
    import ctypes
    g = nc.source(28, 2, no.NESTED_VALUES)
    n = 2 * no.NESTED_VALUES
    with ack.Device() as dev:
        lib = dev._lib.cdll

        def up(arr):
            raw = np.ascontiguousarray(arr).view(np.uint8)
            b = dev.buffer(max(raw.size, 4))
            b.upload(raw)
            return b
        bufs = [up(x) for x in _host(g)]
        out = dev.buffer(2 * n)
        ms = ctypes.c_double(0.0)
        rc = lib.ack_nf4_decode(dev._handle, *[b._handle for b in bufs], None, out._handle, n, 2, 0, 0, 0, 1,
                                ctypes.byref(ms))
        assert rc == ack.ACK_OK, dev._lib.last_error()
        assert np.isnan(ms.value)
        np.testing.assert_array_equal(out.download(np.uint16), no.decode(*_host(g), n, storage=1))
        table = np.array([[0, 3, 0], [3, 1, no.NESTED_VALUES]], np.uint32)
        a16 = nc.activations(8, 4, 512, 0)
        abuf, tbuf, cbuf = up(a16), up(table), dev.buffer(4 * 4 * 32)
        rc = lib.ack_gemv_nf4(dev._handle, abuf._handle, *[b._handle for b in bufs], tbuf._handle, cbuf._handle,
                              4, 3, 32, 512, 0, 2, 2, 0, 0, None)
        assert rc == ack.ACK_OK, dev._lib.last_error()
        np.testing.assert_array_equal(cbuf.download(np.uint32),
                                      no.gemv(a16, *_host(g), table, rows=4, n=32, k=512).view(np.uint32).reshape(-1))
        rc = lib.ack_gemv_nf4(dev._handle, abuf._handle, *[b._handle for b in bufs], tbuf._handle, abuf._handle,
                              4, 3, 32, 512, 0, 2, 2, 0, 0, None)
        assert rc == ack.ACK_ERR_SHAPE and "aliases" in dev._lib.last_error()
        for b in bufs + [out, abuf, tbuf, cbuf]:
            b.free()
