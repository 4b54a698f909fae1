"""Pin the CPU oracle to the reference: its restated format, encode, decode
and fit must reproduce, byte for byte, what the reference's own Python code
produced for the same seeded inputs (`tests/golden/gen_golden.py`)."""
import hashlib

import numpy as np
import pytest

import vq_oracle as o


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_cfg1_three_thousand_one_hundred_twenty_eight_bytes(golden):
    g = golden("cfg1")
    w = o.gaussian((256, 256), 0.02, 7)
    assert sha(w) == str(g["w_sha256"])
    book = o.fit_codebook(w, group=16)
    np.testing.assert_array_equal(book, g["book"])
    codes = o.encode(w, book, 16)
    np.testing.assert_array_equal(codes, g["codes"])
    wire = o.to_bytes((256, 256), 16, codes, book)
    assert len(wire) == 3128 == o.layout((256, 256), 16)["serialized_bytes"]
    assert wire == g["wire"].tobytes()
    assert sha(o.decode(codes, book, 256 * 256, 16).reshape(256, 256)) == str(g["decoded_sha256"])
    x = np.random.default_rng(8).standard_normal((1, 256)).astype(np.float32)
    np.testing.assert_array_equal(x, g["x"])
    xb = o.fit_codebook(x, group=16)
    np.testing.assert_array_equal(xb, g["x_book"])
    np.testing.assert_array_equal(o.encode(x, xb, 16), g["x_codes"])


@pytest.mark.parametrize("group", [8, 16, 32])
def test_encode_decode_with_tails(golden, group):
    g = golden("encode_decode")
    for n in (1, group, 8 * group, 8 * group + 1, 1000, 4097, 3 * group - 5):
        key = f"g{group}_n{n}"
        values, book = g[key + "_values"], g[key + "_book"]
        fit_input = values if n >= group else np.pad(values, (0, group - n))
        np.testing.assert_array_equal(o.fit_codebook(fit_input, group=group), book)
        codes = o.encode(values, book, group)
        np.testing.assert_array_equal(codes, g[key + "_codes"], err_msg=key)
        np.testing.assert_array_equal(o.decode(codes, book, n, group), g[key + "_decoded"])
        assert o.to_bytes((n,), group, codes, book) == g[key + "_wire"].tobytes()
        shape, grp, c2, b2 = o.from_bytes(g[key + "_wire"].tobytes())
        assert shape == (n,) and grp == group
        np.testing.assert_array_equal(c2, codes)


@pytest.mark.parametrize("group", [8, 16, 32])
def test_ties_keep_the_lowest_index(golden, group):
    t = golden("ties")
    codes = o.encode(t[f"g{group}_values"], t[f"g{group}_book"], group)
    np.testing.assert_array_equal(codes, t[f"g{group}_codes"])
    idx = o.unpack(codes, t[f"g{group}_values"].size // group)
    assert not np.isin(idx, [7, 12]).any(), "a duplicate row was selected"
    np.testing.assert_array_equal(
        o.encode(t[f"g{group}_zero_values"], np.zeros((16, group), np.float32), group),
        t[f"g{group}_zero_codes"])
    heavy = t[f"g{group}_heavy_values"]
    np.testing.assert_array_equal(heavy, o.duplicate_heavy(heavy.size // group, group))
    book = o.fit_codebook(heavy, group=group, sample_vectors=65536)
    np.testing.assert_array_equal(book, t[f"g{group}_heavy_book"])
    np.testing.assert_array_equal(o.encode(heavy, book, group), t[f"g{group}_heavy_codes"])


def test_fit_codebook_occupancy_and_warm_start(golden):
    f = golden("fit")
    for name in ("even", "common_rare", "geometric", "dominant"):
        np.testing.assert_array_equal(
            o.fit_codebook(f[f"occ_{name}_values"], group=16), f[f"occ_{name}_book"], err_msg=name)
    for group, rare in ((8, 8191), (8, 1), (16, 4095), (32, 2047)):
        key = f"warm_g{group}_r{rare}"
        values = f[key + "_atoms"][f[key + "_index"].astype(np.int64)].reshape(-1)
        assert sha(values) == str(f[key + "_values_sha256"])
        np.testing.assert_array_equal(
            o.fit_codebook(values, group=group, init=f[key + "_atoms"]), f[key + "_book"], err_msg=key)
    gauss = o.gaussian(200_000, 0.02, 11)
    assert sha(gauss) == str(f["gauss_values_sha256"])
    for group in (8, 16, 32):
        cold = o.fit_codebook(gauss, group=group)
        np.testing.assert_array_equal(cold, f[f"gauss_g{group}_cold"])
        np.testing.assert_array_equal(
            o.fit_codebook(gauss * np.float32(1.01), group=group, init=cold), f[f"gauss_g{group}_warm"])
        np.testing.assert_array_equal(
            o.fit_codebook(gauss, group=group, sample_vectors=65536, iterations=2),
            f[f"gauss_g{group}_big"])


def test_wire_images_of_every_rank(golden):
    w = golden("wire")
    names = sorted({k.rsplit("_", 1)[0] for k in w.files})
    assert len(names) == 15
    for key in names:
        shape = tuple(int(d) for d in key.split("_g")[0].split("x"))
        group = int(key.split("_g")[1])
        codes = o.encode(w[key + "_values"], w[key + "_book"], group)
        assert o.to_bytes(shape, group, codes, w[key + "_book"]) == w[key + "_wire"].tobytes(), key
        lay = o.layout(shape, group)
        assert [lay[k] for k in ("elements", "vectors", "code_bytes", "codebook_bytes", "metadata_bytes",
                                 "serialized_bytes", "payload_bytes")] == w[key + "_layout"].tolist()


def test_shader_restatements_agree_with_float64_on_easy_data():
    """The unpinned shader restatements are at least consistent with the
    float64 references on well-conditioned inputs."""
    rng = np.random.default_rng(3)
    m, n, k, g = 5, 7, 24, 8
    ab = rng.standard_normal((16, g)).astype(np.float32)
    bb = rng.standard_normal((16, g)).astype(np.float32)
    ac = o.pack(rng.integers(0, 16, (m * k + g - 1) // g))
    bc = o.pack(rng.integers(0, 16, (k * n + g - 1) // g))
    for flags in range(4):
        y = o.matmul_shader(ac, ab, bc, bb, m, n, k, g, flags)
        y64 = o.coded_f64(ac, ab, bc, bb, m, n, k, g, flags)
        assert np.allclose(y, y64, rtol=1e-5, atol=1e-5)
    x = rng.standard_normal(4096).astype(np.float32)
    fp32 = o.nearest_fp32_shader(x, ab, g)
    fp64 = o.nearest(x, ab, g)
    mism = np.nonzero(fp32 != fp64)[0]
    assert set(mism.tolist()) <= set(o.near_ties(x, ab, g, rel=1e-5).tolist())
