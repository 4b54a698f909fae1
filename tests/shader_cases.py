"""Seeded inputs of the shader-order operations (op 0 FP32 encode, op 2
packed-pair matmul, op 3 AdamW), shared by the GPU parity tests and the CPU
tests that pin the numpy restatements to the reference shader compiled for
the host (`oracle/vq4_ref.py`). Both sides iterate the same generators, so
every case the device is checked on is also a case the restatement is
pinned on."""
from __future__ import annotations

import numpy as np

import vq_oracle as o


def rand_book(rng, group, scale=1.0):
    return (rng.standard_normal((16, group)) * scale).astype(np.float32)


MATMUL_SHAPES = ((3, 5, 7, 8), (33, 65, 129, 16), (64, 17, 96, 32), (1, 256, 256, 16))


def matmul_cases(flags):
    """Op 2 cases for one flag value: (m, n, k, group, a_codes, a_book,
    b_codes, b_book). A is stored K x M when flags bit 0 is set, B is stored
    N x K when bit 1 is set (`vq4.comp:169-170`)."""
    rng = np.random.default_rng(40 + flags)
    for (m, n, k, group) in MATMUL_SHAPES:
        ab, bb = rand_book(rng, group), rand_book(rng, group)
        ac = o.pack(rng.integers(0, 16, (m * k + group - 1) // group))
        bc = o.pack(rng.integers(0, 16, (k * n + group - 1) // group))
        yield m, n, k, group, ac, ab, bc, bb


def adamw_cases():
    """Op 3 cases: (n, group, state codes [W, M, V, G], books, step). The
    variance book is made non-negative, as a real second moment is."""
    rng = np.random.default_rng(77)
    for (n, group) in ((129, 16), (4096, 8), (50_001, 32)):
        codes, books = [], []
        for scale in (0.02, 0.01, 1e-4, 1e-3):
            book = rand_book(rng, group, scale)
            if scale == 1e-4:
                book = np.abs(book)
            books.append(book)
            codes.append(o.pack(rng.integers(0, 16, (n + group - 1) // group)))
        for step in (1, 7):
            yield n, group, codes, books, step


ADAMW_HYPER = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01)


def adamw_coefficients(step):
    h = ADAMW_HYPER
    return o.adamw_coefficients(h["lr"], h["beta1"], h["beta2"], h["eps"], h["weight_decay"], step)


def status_cases():
    """Plans whose status word is not zero: (name, plan, bindings, out
    values, expected status). Negative variance and beta1 outside [0, 1) set
    bit 2 (`vq4.comp:95-102`); a nonfinite coefficient or book value sets
    bit 0 (`vq4.comp:93, 156`)."""
    rng = np.random.default_rng(3)
    n, group = 64, 8
    codes = o.pack(rng.integers(0, 16, n // group))
    negative = -np.abs(rand_book(rng, group))
    states = np.concatenate([codes] * 4)
    books = np.concatenate([rand_book(rng, group).reshape(-1), rand_book(rng, group).reshape(-1),
                            negative.reshape(-1), rand_book(rng, group).reshape(-1)])
    coefs = o.adamw_coefficients(1e-3, 0.9, 0.999, 1e-8, 0.0, 1)
    plan3 = (3, n, 1, 1, group, 16, 0, 0)
    yield "negative-variance", plan3, (states, books, coefs), n * 3, 4
    bad = coefs.copy()
    bad[1] = 1.5
    yield "beta1-out-of-range", plan3, (states, np.abs(books), bad.copy()), n * 3, 4
    bad[1] = np.inf
    yield "infinite-coefficient", plan3, (states, np.abs(books), bad.copy()), n * 3, 1
    nan_book = rand_book(rng, group)
    nan_book[5, 2] = np.nan
    yield "nan-book", (1, n, 1, 1, group, 16, 0, 0), (codes, nan_book), n, 1


def fp32_encode_cases(group, count=1 << 20, head=1 << 16):
    """The near-tie counting inputs of the encode parity test: both cfg-5
    distributions (block-normalised Gaussian; duplicate-heavy), their books
    fitted from a 65,536-vector sample. Yields (name, values, book, head):
    the shader's FP32 encoder is compared on the first `head` values."""
    from alelyon_compute_kit import vq
    gauss = o.block_normalised(o.gaussian(count, 1.0, 10), group)
    heavy = o.duplicate_heavy(count // group, group)
    for name, values in (("gauss", gauss), ("heavy", heavy)):
        book = vq.fit_codebook(values, group=group, sample_vectors=65536)
        yield name, values, book, head
