"""The package's CPU side (format, `encode`, `fit_codebook`, `VQAdamW` with a
host backend) against the reference's golden vectors and the reference's
own property tests (`tests/test_fit_codebook_keeps_every_entry.py`)."""
import hashlib

import numpy as np
import pytest

import vq_oracle as o
from alelyon_compute_kit import vq
from alelyon_compute_kit.vq import ENTRIES, VQAdamW, VQArray, encode, fit_codebook


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---- pinned to the reference's outputs ----

def test_cfg1_image_matches_the_reference(golden):
    g = golden("cfg1")
    w = o.gaussian((256, 256), 0.02, 7)
    book = fit_codebook(w, group=16)
    np.testing.assert_array_equal(book, g["book"])
    image = encode(w, book, group=16)
    assert image.to_bytes() == g["wire"].tobytes()
    assert image.layout["serialized_bytes"] == 3128
    assert VQArray.from_bytes(g["wire"].tobytes()).to_bytes() == image.to_bytes()


@pytest.mark.parametrize("group", [8, 16, 32])
def test_encode_decode_fit_match_the_reference(golden, group):
    g = golden("encode_decode")
    for n in (1, group, 8 * group, 8 * group + 1, 1000, 4097, 3 * group - 5):
        key = f"g{group}_n{n}"
        values = g[key + "_values"]
        fit_input = values if n >= group else np.pad(values, (0, group - n))
        np.testing.assert_array_equal(fit_codebook(fit_input, group=group), g[key + "_book"])
        arr = encode(values, g[key + "_book"], group=group)
        assert arr.to_bytes() == g[key + "_wire"].tobytes(), key
        np.testing.assert_array_equal(arr.decode(), g[key + "_decoded"])


def test_fit_codebook_warm_starts_match_the_reference(golden):
    f = golden("fit")
    for group, rare in ((8, 8191), (8, 1), (16, 4095), (32, 2047)):
        key = f"warm_g{group}_r{rare}"
        values = f[key + "_atoms"][f[key + "_index"].astype(np.int64)].reshape(-1)
        np.testing.assert_array_equal(fit_codebook(values, group=group, init=f[key + "_atoms"]), f[key + "_book"])
    gauss = o.gaussian(200_000, 0.02, 11)
    for group in (8, 16, 32):
        cold = fit_codebook(gauss, group=group)
        np.testing.assert_array_equal(cold, f[f"gauss_g{group}_cold"])
        np.testing.assert_array_equal(fit_codebook(gauss * np.float32(1.01), group=group, init=cold),
                                      f[f"gauss_g{group}_warm"])


@pytest.mark.parametrize("group", [8, 16, 32])
def test_ties_match_the_reference(golden, group):
    t = golden("ties")
    assert encode(t[f"g{group}_values"], t[f"g{group}_book"], group=group).codes.tobytes() == \
        t[f"g{group}_codes"].tobytes()


def test_wire_refusals():
    good = encode(np.arange(20, dtype=np.float32), np.zeros((16, 8), np.float32), group=8)
    data = good.to_bytes()
    with pytest.raises(ValueError, match="header"):
        VQArray.from_bytes(b"XXXXXXXX" + data[8:])
    with pytest.raises(ValueError, match="length"):
        VQArray.from_bytes(data + b"\0")
    with pytest.raises(ValueError, match="truncated"):
        VQArray.from_bytes(data[:20])
    codes = good.codes.copy()
    codes[-1] |= np.uint32(1 << 31)
    with pytest.raises(ValueError, match="unused codeword bits"):
        VQArray(good.shape, 8, codes, good.codebook)
    with pytest.raises(ValueError, match="finite"):
        encode(np.array([np.nan] * 8, np.float32), np.zeros((16, 8), np.float32), group=8)
    with pytest.raises(ValueError, match="group"):
        vq.storage_layout((4,), 12)


# ---- the reference's fit properties (test_fit_codebook_keeps_every_entry.py) ----

DIMS, SEED = 16, 1
OCCUPANCY = {
    "even": [64] * ENTRIES,
    "eight common, eight rare": [120] * 8 + [8] * 8,
    "skewed geometric": [max(1, int(512 * 0.55 ** i)) for i in range(ENTRIES)],
    "one dominant, fifteen rare": [900] + [4] * (ENTRIES - 1),
}


def indices(sample, book):
    codes = encode(sample, book, group=DIMS).codes
    pos = np.arange(len(sample))
    return (codes[pos // 8] >> ((pos % 8) * 4).astype(np.uint32)) & 15


def sample_of(counts):
    atoms = np.random.default_rng(SEED).standard_normal((ENTRIES, DIMS))
    return np.repeat(atoms, counts, axis=0).astype(np.float32)


@pytest.mark.parametrize("name", list(OCCUPANCY))
def test_every_entry_is_distinct_and_reachable(name):
    sample = sample_of(OCCUPANCY[name])
    book = fit_codebook(sample.reshape(-1), group=DIMS)
    assert len(np.unique(book.round(6), axis=0)) == ENTRIES
    assert len(np.unique(indices(sample, book))) == ENTRIES


def test_identical_input_collapses_and_that_is_correct():
    book = fit_codebook(np.ones((512, DIMS), dtype=np.float32).reshape(-1), group=DIMS)
    assert len(np.unique(book.round(6), axis=0)) == 1


class HostBackend:
    """The reference shader's arithmetic on the host, restated by the
    oracle: AdamW op 3 in FP32 shader order, the CPU encoder."""

    def encode(self, values, codebook, *, group):
        return encode(values, codebook, group=group)

    def decode(self, value):
        return value.decode()

    def adamw(self, weight, momentum, variance, gradient, *, lr, beta1, beta2, eps, weight_decay, step):
        coefs = o.adamw_coefficients(lr, beta1, beta2, eps, weight_decay, step)
        w, m, v = o.adamw_shader(*(s.decode() for s in (weight, momentum, variance, gradient)), coefs)
        return w, m, v


def review_shape(group, rare_at=-1):
    vectors = 65536 // group
    atoms = np.random.default_rng(SEED).standard_normal((ENTRIES, group)).astype(np.float32)
    index = np.insert(np.arange(vectors - 1) % (ENTRIES - 1), rare_at % vectors, ENTRIES - 1)
    return atoms, index


def zero_gradient_step(backend, atoms, index, group):
    values = atoms[index].reshape(-1)
    weight = encode(values, atoms, group=group)
    zero = VQArray(weight.shape, group, np.zeros_like(weight.codes), np.zeros((ENTRIES, group), np.float32))
    optimizer = VQAdamW(backend, weight, lr=1e-3, weight_decay=0.0)
    before = optimizer.weight.decode().copy()
    report = optimizer.step(zero)
    after = optimizer.weight.decode()
    assert report["changed_weight_values"] == int((before != after).sum())
    return report["changed_weight_values"], len(np.unique(optimizer.weight.codebook.round(6), axis=0))


@pytest.mark.parametrize("group,rare_at", [(8, -1), (16, -1), (32, -1), (8, 1)])
def test_zero_gradient_moves_no_weight(group, rare_at):
    changed, rows = zero_gradient_step(HostBackend(), *review_shape(group, rare_at), group)
    assert changed == 0 and rows == ENTRIES


def test_vqadamw_refuses_without_changing_state():
    w = encode(np.ones(64, np.float32), np.eye(16, 8, dtype=np.float32), group=8)
    opt = VQAdamW(HostBackend(), w, lr=-1.0)
    with pytest.raises(ValueError):
        # the host backend is not consulted for coefficients; VQDevice checks them
        vq._adamw_coefficients((w, w, w, w), -1.0, 0.9, 0.95, 1e-8, 0.0, 1)
    assert opt.steps == 0 and opt.weight is w


def test_stack_round_trip():
    arrays = [encode(np.random.default_rng(i).standard_normal(80).astype(np.float32),
                     np.random.default_rng(9).standard_normal((16, 8)).astype(np.float32), group=8)
              for i in range(3)]
    stack = vq.VQStack.from_arrays(arrays)
    assert len(stack) == 3 and stack.codes.shape == (3, arrays[0].codes.size)
    for i in range(3):
        assert stack[i].to_bytes() == arrays[i].to_bytes()
    with pytest.raises(ValueError):
        vq.VQStack.from_arrays([arrays[0], encode(np.ones(16, np.float32), np.zeros((16, 8), np.float32), group=8)])
