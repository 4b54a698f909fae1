"""Pin the CPU oracle to the reference.

* The restated format, encode, decode and fit must reproduce, byte for byte,
  what the reference's own Python code produced for the same seeded inputs
  (`tests/golden/gen_golden.py`).
* The restated shader arithmetic (op 0 FP32 encode, op 2 packed-pair matmul,
  op 3 AdamW, and the status bits) must equal, bit for bit, the reference's
  own `vq4.comp` compiled for the host (`oracle/vq4_ref.py`), on every case
  the GPU parity tests use (`tests/shader_cases.py`)."""
import hashlib
import os

import numpy as np
import pytest

import shader_cases as sc
import vq4_ref
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
    """The shader restatements are also consistent with the float64
    references on well-conditioned inputs."""
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


# ------------------------------------------- the shader compiled for the host ----

REFERENCE_ROOTS = (os.environ.get("ACK_REFERENCE_ROOT"), "/root/reference")


@pytest.fixture(scope="module")
def shader():
    """The reference shader library, built here if a reference checkout is
    present and the library is not yet built."""
    if not vq4_ref.available():
        for root in REFERENCE_ROOTS:
            if root and os.path.isdir(root) and vq4_ref.build(root):
                break
    if not vq4_ref.available():
        pytest.skip("the reference shader library is not built and no reference checkout is present")
    return vq4_ref


@pytest.mark.parametrize("flags", [0, 1, 2, 3])
def test_matmul_restatement_is_the_shader(shader, flags):
    for (m, n, k, group, ac, ab, bc, bb) in sc.matmul_cases(flags):
        ref, status = shader.matmul(ac, ab, bc, bb, m, n, k, group, flags)
        assert status == 0
        mine = o.matmul_shader(ac, ab, bc, bb, m, n, k, group, flags)
        np.testing.assert_array_equal(mine.view(np.uint32), ref.view(np.uint32), err_msg=str((m, n, k, group)))


def test_adamw_restatement_is_the_shader(shader):
    for (n, group, codes, books, step) in sc.adamw_cases():
        coefs = sc.adamw_coefficients(step)
        ref, status = shader.adamw(codes, books, coefs, n, group)
        assert status == 0
        mine = o.adamw_shader(*(o.decode(c, b, n, group) for c, b in zip(codes, books)), coefs)
        for a, b in zip(mine, ref):
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32), err_msg=str((n, group, step)))


def test_adamw_restatement_is_the_shader_at_the_bank_shape(shader):
    """One 4096 x 1024 g8 expert (the fused-VQAdamW workload's tensor): W
    from N(0, 0.02^2) fitted, moments after one step, a 1e-3 gradient."""
    n, group = 4096 * 1024, 8
    rng = np.random.default_rng(9)
    codes, books = [], []
    for std in (0.02, 1e-4, 1e-6, 1e-3):
        values = (rng.standard_normal(n) * std).astype(np.float32)
        if std == 1e-6:
            values = values * values
        book = o.fit_codebook(values, group=group)
        codes.append(o.encode(values, book, group))
        books.append(book)
    for step in (2, 1000):
        coefs = o.adamw_coefficients(1e-3, 0.9, 0.999, 1e-8, 0.01, step)
        ref, status = shader.adamw(codes, books, coefs, n, group)
        assert status == 0
        mine = o.adamw_shader(*(o.decode(c, b, n, group) for c, b in zip(codes, books)), coefs)
        for a, b in zip(mine, ref):
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


def test_status_words_are_the_shaders(shader):
    for name, plan, bindings, out_values, status in sc.status_cases():
        padded = list(bindings) + [None] * (4 - len(bindings))
        _, got = shader.run(plan, *padded, out_words=out_values)
        assert got == status, name


@pytest.mark.parametrize("group", [8, 16, 32])
def test_fp32_encode_restatement_is_the_shader(shader, group):
    for name, values, book, head in sc.fp32_encode_cases(group):
        words, status = shader.encode(values[:head], book, group)
        assert status == 0
        np.testing.assert_array_equal(o.nearest_fp32_shader(values[:head], book, group),
                                      o.unpack(words, head // group), err_msg=name)


def test_fp32_encode_restatement_is_the_shader_on_tails_and_ties(shader, golden):
    """Ragged tails (the partial final vector compares its valid values
    only) and exact ties (the lowest index wins), from the golden inputs."""
    g = golden("encode_decode")
    t = golden("ties")
    for group in (8, 16, 32):
        cases = [(g[f"g{group}_n{n}_values"], g[f"g{group}_n{n}_book"])
                 for n in (1, group, 8 * group, 8 * group + 1, 1000, 4097, 3 * group - 5)]
        cases += [(t[f"g{group}_values"], t[f"g{group}_book"]),
                  (t[f"g{group}_zero_values"], np.zeros((16, group), np.float32)),
                  (t[f"g{group}_heavy_values"], t[f"g{group}_heavy_book"])]
        for values, book in cases:
            words, status = shader.encode(values, book, group)
            assert status == 0
            vectors = (values.size + group - 1) // group
            np.testing.assert_array_equal(o.nearest_fp32_shader(values, book, group), o.unpack(words, vectors))


def test_decode_restatement_is_the_shader(shader):
    rng = np.random.default_rng(12)
    for group in (8, 16, 32):
        for n in (1, group - 1, 8 * group + 3, 5000):
            book = sc.rand_book(rng, group)
            codes = o.pack(rng.integers(0, 16, (n + group - 1) // group))
            ref, status = shader.decode(codes, book, n, group)
            assert status == 0
            np.testing.assert_array_equal(o.decode(codes, book, n, group).view(np.uint32), ref.view(np.uint32))
