"""NF4 comparator test data, shaped as the reference's own NF4 tests build
theirs (src/alelyon_compute_kit/_kit/tests/nf4_gemv_abi.rs:212-258): members
of whole nested blocks back to back, a few nested blocks of filler before the
source, absmax2 values in [0.004, 0.2], member offsets from a short list, and
a table of 16 code values then the 256 signed map values (i - 127.5) / 128.
The code values here are normal quantiles scaled to [-1, 1] with 0 among
them (the table is an input, so any 16 values exercise the law)."""
from statistics import NormalDist

import numpy as np

import nf4_oracle as no


def tables() -> np.ndarray:
    nd = NormalDist()
    q = [nd.inv_cdf(p) for p in np.linspace(0.03, 0.97, 15)]
    code = np.array(sorted(q + [0.0]), np.float64)
    code = (code / np.abs(code).max()).astype(np.float32)
    return np.concatenate([code, ((np.arange(256) - 127.5) / 128.0).astype(np.float32)])


def source(seed: int, members: int, member_values: int, base_blocks: int = 0) -> dict:
    assert member_values % no.NESTED_VALUES == 0
    rng = np.random.default_rng(seed)
    base = base_blocks * no.NESTED_VALUES
    values = base + members * member_values
    blocks = values // no.BLOCK
    nested = blocks // no.NESTED
    return {"packed": rng.integers(0, 256, values // 2, dtype=np.uint8),
            "absmax_q": rng.integers(0, 256, blocks, dtype=np.uint8),
            "absmax2": (0.004 + rng.integers(0, 997, nested) * 0.0002).astype(np.float32),
            "tables": tables(),
            "starts": np.arange(members, dtype=np.int64) * member_values,
            "offsets": np.array([0.011, -0.004, 0.0073, 0.0, -0.0021] * ((members + 4) // 5), np.float32)[:members],
            "base": base}


def activations(seed: int, rows: int, lda: int, elem: int, scale: float = 1.0) -> np.ndarray:
    """A's 16-bit words, rows x lda (bf16 for elem 0, fp16 for 1)."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(rows * lda) * scale).astype(np.float32)
    return no.narrow(1 + elem, x).reshape(rows, lda)


def weight_groups(experts, per_expert_values: int) -> np.ndarray:
    """The groups table for (expert, rows) in dispatch order: rows stacked in
    that order, each group's weight at its expert's first member."""
    table, row = [], 0
    for expert, rows in experts:
        table.append((row, rows, expert * per_expert_values))
        row += rows
    return np.array(table, np.uint32), row
