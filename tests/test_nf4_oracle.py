"""The NF4 comparator's CPU side: the numpy restatement (oracle/nf4_oracle.py)
against the reference's nf4_decode.comp and nf4_gemv.comp compiled for the
host (oracle/_ref, built from a reference checkout), and the refusals by
name of the library's admission (which runs before any CUDA call)."""
import ctypes

import numpy as np
import pytest

import nf4_cases as nc
import nf4_oracle as no
import nf4_ref as nr
from alelyon_compute_kit import ack

needs_ref = pytest.mark.skipif(not nr.available(), reason="oracle/_ref NF4 shaders not built (needs a reference "
                                                          "checkout: make -C oracle ref REFERENCE=...)")


def _same(x, y):
    x, y = np.asarray(x), np.asarray(y)
    return x.shape == y.shape and x.tobytes() == y.tobytes()


@needs_ref
@pytest.mark.parametrize("storage", [0, 1, 2])
def test_decode_restatement_is_the_shader(storage):
    g = nc.source(11, 3, no.NESTED_VALUES, base_blocks=1)
    args = (g["packed"], g["absmax_q"], g["absmax2"], g["tables"], g["starts"], g["offsets"])
    n = 3 * no.NESTED_VALUES - 5   # a partial last word
    assert _same(no.decode(*args, n, src_base=g["base"], storage=storage),
                 nr.decode(*args, n, src_base=g["base"], storage=storage))
    # a selection: repeated, out-of-range and negative ids (their values read NaN)
    ids = np.array([2, 0, 2, 7, -1], np.int64)
    kw = dict(ids=ids, member_values=4096, src_base=g["base"], storage=storage)
    want = nr.decode(*args, 5 * 4096, **kw)
    got = no.decode(*args, 5 * 4096, **kw)
    assert _same(got, want)
    if storage == 0:
        assert np.isnan(got[3 * 4096:]).all() and not np.isnan(got[: 3 * 4096]).any()


@needs_ref
@pytest.mark.parametrize("elem", [0, 1])
def test_gemv_restatement_is_the_shader(elem):
    """Four experts of two members (128 x 256 weights), grouped with 5, 0,
    16 and 1 rows; then a column straddling members with their own offsets."""
    g = nc.source(12, 8, no.NESTED_VALUES, base_blocks=1)
    table, rows = nc.weight_groups([(2, 5), (1, 0), (0, 16), (3, 1)], 2 * no.NESTED_VALUES)
    a16 = nc.activations(5, rows, 256, elem)
    args = (a16, g["packed"], g["absmax_q"], g["absmax2"], g["tables"], g["starts"], g["offsets"], table)
    kw = dict(rows=rows, n=128, k=256, src_base=g["base"], elem=elem)
    assert _same(no.gemv(*args, **kw), nr.gemv(*args, **kw))
    s = nc.source(13, 3, no.NESTED_VALUES)
    k = 3 * no.NESTED_VALUES // 2
    a16 = nc.activations(6, 2, k, elem)
    args = (a16, s["packed"], s["absmax_q"], s["absmax2"], s["tables"], s["starts"], s["offsets"],
            np.array([[0, 2, 0]], np.uint32))
    assert _same(no.gemv(*args, rows=2, n=2, k=k, elem=elem), nr.gemv(*args, rows=2, n=2, k=k, elem=elem))


@needs_ref
def test_gemv_fp16_subnormals_follow_the_shader():
    """Every absmax below fp16's smallest normal, activations scaled into the
    subnormals too (nf4_gemv_abi.rs's subnormal case, smaller)."""
    g = nc.source(14, 1, 4 * no.NESTED_VALUES)
    g["absmax2"] = (2.0e-6 + (np.arange(len(g["absmax2"])) % 7) * 7.0e-6).astype(np.float32)
    g["offsets"][:] = 0
    a16 = nc.activations(7, 3, 512, 1, scale=1.0e-5)
    args = (a16, g["packed"], g["absmax_q"], g["absmax2"], g["tables"], g["starts"], g["offsets"],
            np.array([[0, 3, 0]], np.uint32))
    kw = dict(rows=3, n=64, k=512, elem=1)
    got = no.gemv(*args, **kw)
    assert _same(got, nr.gemv(*args, **kw)) and np.abs(got).max() > 0


def test_plan_refusals_by_name():
    cov = no.values_covered(1 << 20, 1 << 15, 64)
    cases = [
        (lambda: no.decode_plan(0, 1, 0, 0, 0, cov, 0), "nf4-zero-values"),
        (lambda: no.decode_plan(64, 0, 0, 0, 0, cov, 0), "nf4-members-out-of-range"),
        (lambda: no.decode_plan(64, 1, 1, 65, 0, cov, 0), "nf4-selection-out-of-range"),
        (lambda: no.decode_plan(64, 1, 0, 0, 100, cov, 0), "nf4-base-out-of-range"),
        (lambda: no.decode_plan(cov + 8, 1, 0, 0, 0, cov, 0), "nf4-source-too-small"),
        (lambda: no.decode_plan(64, 1, 0, 0, 0, cov, 3), "nf4-storage-out-of-range"),
        (lambda: no.gemv_plan(1, 17, 8, 64, 0, 1, 1, 0, cov, 0), "nf4-matmul-rows-out-of-range"),
        (lambda: no.gemv_plan(32, 17, 8, 64, 0, 1, 1, 0, cov, 0), "nf4-gemv-rows-above-16"),
        (lambda: no.gemv_plan(1, 1, 8, 60, 0, 1, 1, 0, cov, 0), "nf4-matmul-row-not-whole-words"),
        (lambda: no.gemv_plan(1, 1, 8, 64, 60, 1, 1, 0, cov, 0), "nf4-matmul-pitch-below-width"),
        (lambda: no.gemv_plan(1, 1, 8, 64, 68, 1, 1, 0, cov, 0), "nf4-gemv-pitch-not-whole-words"),
        (lambda: no.gemv_plan(1, 1, 8, 64, 0, 0, 1, 0, cov, 0), "nf4-matmul-groups-out-of-range"),
        (lambda: no.gemv_plan(1, 1, 8, 64, 0, 1, 1, 0, cov, 2), "nf4-matmul-elem-out-of-range"),
    ]
    for fn, name in cases:
        with pytest.raises(no.Nf4PlanError, match=name):
            fn()


def _launch_decode(lib, n, members, selected, member_values, src_base, storage, sizes):
    ptrs = (ctypes.c_void_p * 8)(*[0x10000 * (i + 1) for i in range(8)])
    byts = (ctypes.c_uint64 * 8)(*sizes)
    return lib.cdll.ack_nf4_decode_launch(ptrs, byts, n, members, selected, member_values, src_base, storage, None)


def _launch_gemv(lib, rows, max_rows, n, k, lda, groups, members, src_base, elem, sizes):
    ptrs = (ctypes.c_void_p * 9)(*[0x10000 * (i + 1) for i in range(9)])
    byts = (ctypes.c_uint64 * 9)(*sizes)
    return lib.cdll.ack_gemv_nf4_launch(ptrs, byts, rows, max_rows, n, k, lda, groups, members, src_base, elem,
                                        None)


def test_library_refuses_what_the_planner_refuses():
    """The device-pointer entries admit before any CUDA call: refusals need
    no GPU. Sizes: packed 512 KB, absmax_q 16 KB, absmax2 64 B (2^20 values
    covered), tables, starts and offsets for one member, a big output."""
    lib = ack._lib()
    src = [1 << 19, 1 << 14, 64, 272 * 4, 8, 4]
    cases = [
        (dict(n=0, members=1, selected=0, member_values=0, src_base=0, storage=0), ack.ACK_ERR_SHAPE, "nf4-zero-values"),
        (dict(n=64, members=1, selected=0, member_values=0, src_base=0, storage=5), ack.ACK_ERR_SHAPE,
         "nf4-storage-out-of-range"),
        (dict(n=(1 << 20) + 8, members=1, selected=0, member_values=0, src_base=0, storage=0), ack.ACK_ERR_SIZE,
         "nf4-source-too-small"),
        (dict(n=64, members=1, selected=0, member_values=0, src_base=16, storage=0), ack.ACK_ERR_SHAPE,
         "nf4-base-out-of-range"),
    ]
    for kw, rc, name in cases:
        assert _launch_decode(lib, sizes=src + [0, 1 << 30], **kw) == rc
        assert name in lib.last_error()
    # an output too small for the values, by name
    assert _launch_decode(lib, 64, 1, 0, 0, 0, 0, src + [0, 100]) == ack.ACK_ERR_SIZE
    assert "nf4-output-too-small" in lib.last_error()
    gsrc = [1 << 20] + src + [12, 1 << 20]
    for args, rc, name in [
        ((20, 17, 8, 64, 0, 1, 1, 0, 0), ack.ACK_ERR_SHAPE, "nf4-gemv-rows-above-16"),
        ((1, 1, 8, 60, 0, 1, 1, 0, 0), ack.ACK_ERR_SHAPE, "nf4-matmul-row-not-whole-words"),
        ((2, 1, 8, 64, 68, 1, 1, 0, 0), ack.ACK_ERR_SHAPE, "nf4-gemv-pitch-not-whole-words"),
        ((1, 1, 8, 64, 0, 1, 1, 0, 7), ack.ACK_ERR_SHAPE, "nf4-matmul-elem-out-of-range"),
        ((1, 1, 1 << 15, 64, 0, 1, 1, 0, 0), ack.ACK_ERR_SIZE, "nf4-source-too-small"),
    ]:
        assert _launch_gemv(lib, *args, sizes=gsrc) == rc
        assert name in lib.last_error()
