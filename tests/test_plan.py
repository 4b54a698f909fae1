"""Host-only vq4 admission: the reference planner's tests
(`_kit/tests/vq4_plan.rs`), run against this library's C planner through
its probe entries. Same plans, same byte counts, same refusals."""
import pytest

from abi_util import MAX_DIM, MAX_VALUES, probe, refusal, required, validate_buffers, validate_dispatch

SHAPE, SIZE = -3, -4


def vector(op, n, group):
    return [op, n, 1, 1, group, 16, 0, 0]


@pytest.mark.parametrize("group", [8, 16, 32])
def test_packed_cost_counts_padding_and_complete_codebooks(group):  # vq4_plan.rs:10
    for length, words in ((1, 1), (group, 1), (group * 8, 1), (group * 8 + 1, 2)):
        assert required(vector(0, length, group)) == [length * 4, group * 64, 0, 0, words * 4, 4]
        assert required(vector(1, length, group)) == [words * 4, group * 64, 0, 0, length * 4, 4]
        assert probe(vector(0, length, group))[2] == words
        assert probe(vector(1, length, group))[2] == length


def test_adamw_is_four_packed_states_and_three_dense_scratch_arrays():  # vq4_plan.rs:44
    rc, req, work, disp = probe(vector(3, 129, 16))
    assert rc == 0
    assert req[:6] == [32, 4096, 28, 0, 1548, 4]
    assert work == 129 and disp == [3, 1, 1]
    assert probe([3, MAX_VALUES // 3, 1, 1, 8, 16, 0, 0])[0] == 0
    rc, msg = refusal([3, MAX_VALUES // 3 + 1, 1, 1, 8, 16, 0, 0])
    assert rc == SIZE and msg.endswith("vq-address-limit-exceeded")


def test_matmul_transposes_preserve_storage_counts():  # vq4_plan.rs:58
    for flags in range(4):
        rc, req, work, disp = probe([2, 3, 5, 7, 8, 16, flags, 0])
        assert rc == 0 and req[:6] == [4, 512, 4, 512, 60, 4] and work == 15 and disp == [1, 1, 1]


def test_all_schema_words_are_closed():  # vq4_plan.rs:74
    good = [0, 64, 1, 1, 8, 16, 0, 0]
    for slot, value, name in ((0, 4, "vq-operation-out-of-range"), (4, 0, "vq-unsupported-group"),
                              (4, 4, "vq-unsupported-group"), (4, 64, "vq-unsupported-group"),
                              (5, 0, "vq-codebook-entries-not-16"), (5, 15, "vq-codebook-entries-not-16"),
                              (5, 17, "vq-codebook-entries-not-16"), (6, 1, "vq-unsupported-flags"),
                              (7, 1, "vq-nonzero-reserved-word")):
        words = list(good)
        words[slot] = value
        rc, msg = refusal(words)
        assert rc == SHAPE and msg.endswith(name), (slot, value, msg)
    assert refusal([2, 1, 1, 1, 8, 16, 4, 0])[1].endswith("vq-unsupported-flags")
    for op in (1, 3):
        assert refusal([op, 1, 1, 1, 8, 16, 1, 0])[1].endswith("vq-unsupported-flags")


def test_zero_mismatched_or_overflowing_geometry_refuses():  # vq4_plan.rs:101
    for op in range(4):
        for axis in (1, 2, 3):
            words = [op, 1, 1, 1, 8, 16, 0, 0]
            words[axis] = 0
            assert refusal(words)[1].endswith("vq-invalid-geometry")
    for op in (0, 1, 3):
        for axis in (2, 3):
            words = [op, 1, 1, 1, 8, 16, 0, 0]
            words[axis] = 2
            assert refusal(words)[1].endswith("vq-invalid-geometry")
    assert refusal([0, 0xFFFFFFFF, 1, 1, 8, 16, 0, 0]) [1].endswith("vq-address-limit-exceeded")
    assert refusal([1, MAX_VALUES + 1, 1, 1, 8, 16, 0, 0])[1].endswith("vq-address-limit-exceeded")
    assert refusal([2, MAX_DIM + 1, 1, 1, 8, 16, 0, 0])[1].endswith("vq-invalid-geometry")
    for words in ([2, MAX_DIM, MAX_DIM, 1, 8, 16, 0, 0], [2, MAX_DIM, 1, MAX_DIM, 8, 16, 0, 0],
                  [2, 1, MAX_DIM, MAX_DIM, 8, 16, 0, 0]):
        rc, msg = refusal(words)
        assert rc == SIZE and msg.endswith("vq-address-limit-exceeded")


def test_each_read_and_write_capacity_is_checked_in_bytes():  # vq4_plan.rs:138
    for op in range(4):
        words = [2, 11, 9, 7, 16, 16, 0, 0] if op == 2 else vector(op, 129, 16)
        caps = required(words)
        ids = [1, 2, 3, 4, 5, 6]
        assert validate_buffers(words, caps, ids) == 0
        for slot in range(6):
            if caps[slot] == 0:
                continue
            short = list(caps)
            short[slot] -= 1
            rc = validate_buffers(words, short, ids)
            from abi_util import last_error
            assert rc == SIZE and last_error().endswith(f"vq-binding-{slot}-too-small")


def test_every_output_alias_including_unread_inputs_refuses():  # vq4_plan.rs:160
    from abi_util import last_error
    words = vector(0, 64, 8)
    caps = [4096] * 6
    for inp in range(4):
        ids = [1, 2, 3, 4, 5, 6]
        ids[4] = ids[inp]
        assert validate_buffers(words, caps, ids) == SHAPE and last_error().endswith("vq-output-aliases-input")
    for operand in range(5):
        ids = [1, 2, 3, 4, 5, 6]
        ids[5] = ids[operand]
        assert validate_buffers(words, caps, ids) == SHAPE and last_error().endswith("vq-status-aliases-operand")
    assert validate_buffers(words, caps, [1, 1, 1, 1, 2, 3]) == 0
    for slot in range(6):
        ids = [1, 2, 3, 4, 5, 6]
        ids[slot] = 0
        assert validate_buffers(words, caps, ids) == SHAPE and last_error().endswith("vq-null-allocation-identity")


def test_maximum_tensor_uses_bounded_two_dimensional_grid():  # vq4_plan.rs:182
    from abi_util import last_error
    words = vector(1, MAX_VALUES, 32)
    _, _, _, (x, y, z) = probe(words)
    assert (x, y, z) == (65535, 65, 1)
    assert x * y * 64 >= MAX_VALUES and x * y * 64 < 2 ** 32
    assert validate_dispatch(words, [65535] * 3) == 0
    for axis in range(3):
        limits = [x, y, z]
        limits[axis] -= 1
        assert validate_dispatch(words, limits) == SHAPE and last_error().endswith("vq-dispatch-grid-unsupported")


def test_every_refusal_is_named_and_slot_specific():  # vq4_plan.rs:199
    from abi_util import last_error
    words = [2, 11, 9, 7, 16, 16, 0, 0]
    caps = required(words)
    for slot in range(6):
        short = list(caps)
        short[slot] = 0 if caps[slot] else 0
        if caps[slot]:
            validate_buffers(words, short, [1, 2, 3, 4, 5, 6])
            assert last_error() == f"vq: plan refused: vq-binding-{slot}-too-small"


def test_matmul_work_is_bounded_even_when_every_buffer_extent_fits():  # vq4_plan.rs:225
    assert probe([2, 1024, 1024, 256, 8, 16, 0, 0])[0] == 0
    for words in ([2, 1024, 1024, 257, 8, 16, 0, 0], [2, 4096, 4096, 4096, 8, 16, 0, 0]):
        rc, msg = refusal(words)
        assert rc == SIZE and msg.endswith("vq-matmul-work-limit")


# ---- schema 2 (this library's extension plan) ----

def plan2(op, m, n, k, group, flags=0, batch=1, aux0=0, aux1=0, aux2=0):
    return [op, m, n, k, group, 16, flags, 0, batch, aux0, aux1, aux2, 0, 0, 0, 0]


def test_schema2_dense_and_coded_slot_sizes():
    m, n, k, g, e = 4, 11008, 4096, 16, 3
    words = (n * k // g + 7) // 8
    assert required(plan2(16, m, n, k, g, flags=2, batch=e)) == [
        e * m * k * 4, e * words * 4, e * 64 * g, 0, 0, e * m * n * 4, 0, 4]
    assert required(plan2(17, 5, 7, 64, 8, flags=2)) == [
        (5 * 64 // 8 + 7) // 8 * 4, 512, (7 * 64 // 8 + 7) // 8 * 4, 512, 0, 140, 0, 4]
    # the schema-1 MAC bound does not apply to schema 2
    assert probe(plan2(17, 4096, 14336, 4096, 32, flags=2))[0] == 0


def test_schema2_tensor_core_dense_workspace():
    """Op 16 with flag 8 (the tensor-core kernel): the workspace in in4 holds
    bf16 hi and lo projections of one pass of at most 128 rows of X, 128 rows
    of 16 K / G values per 64-row tile, per expert; the flag needs W stored
    N x K (bit 1), the canonical layout and (K / G) % 32 == 0."""
    n, k, g, e = 11008, 4096, 16, 3
    words = (n * k // g + 7) // 8
    for m, tiles in ((1, 1), (8, 1), (37, 1), (64, 1), (65, 2), (128, 2), (300, 2)):
        assert required(plan2(16, m, n, k, g, flags=10, batch=e)) == [
            e * m * k * 4, e * words * 4, e * 64 * g, 0, e * tiles * 128 * 16 * (k // g) * 2, e * m * n * 4, 0, 4]
    for flags, k2 in ((8, k), (14, k), (10, 16 * 33), (10, 16 * 32 + 3)):
        assert refusal(plan2(16, 4, 64, k2, g, flags=flags))[1].endswith("vq2-unsupported-flags"), (flags, k2)
    # the workspace is written: it may alias no other operand
    ok = plan2(16, 8, 128, 512, 16, flags=10)
    caps = [8 * 512 * 4, 128 * 512 // 16 // 2, 1024, 0, 128 * 16 * 32 * 2, 8 * 128 * 4, 0, 4]
    assert validate_buffers(ok, caps, [1, 2, 3, 0, 4, 5, 0, 6]) == 0
    assert validate_buffers(ok, caps, [1, 2, 3, 0, 1, 5, 0, 6]) != 0
    caps[4] -= 1
    assert validate_buffers(ok, caps, [1, 2, 3, 0, 4, 5, 0, 6]) != 0


def test_schema2_adamw_and_large_slot_sizes():
    n, g, e, s = 4096 * 1024, 8, 8, 4096
    words = (n // g + 7) // 8
    assert required(plan2(18, n, 1, 1, g, batch=e, aux0=s)) == [
        e * 4 * words * 4, e * 4 * 64 * g, e * 28, s * 4, 0, e * 3 * s * g * 4, 0, 4]
    assert required(plan2(19, n, 1, 1, g, batch=e, aux0=2, aux1=7)) == [
        e * 4 * words * 4, e * 4 * 64 * g, e * 28, 64 * g, 0, 64, 0, 4]
    assert required(plan2(20, n, 1, 1, g, batch=e)) == [
        e * 4 * words * 4, e * 4 * 64 * g, e * 28, e * 3 * 64 * g, 0, e * 3 * words * 4, e * 4, 4]
    stride = (s + 15) // 16 * 16 + 160  # fit workspace per book: idx bytes, counts, usage, flag
    assert required(plan2(24, n, 1, 1, g, flags=1, batch=e, aux0=s, aux1=4)) == [
        e * 4 * words * 4, e * 4 * 64 * g, e * 28, e * 3 * s * g * 4, e * 3 * stride, e * 3 * 64 * g, 0, 4]
    # op 25: one tensor's fit, 64-bit count, sample gathered into the workspace
    big = 1 << 30
    assert required(plan2(25, big & 0xFFFFFFFF, 1, 1, 16, flags=1, aux0=65536, aux1=4, aux2=big >> 32)) == [
        big * 4, 1024, (65536 + 16) * 4, 0, 65536 * 16 * 4 + 65536 + 160, 1024, 0, 4]
    assert required(plan2(25, 1000, 1, 1, 8, aux0=100, aux1=4))[1] == 0  # cold start reads no book
    assert required(plan2(21, big & 0xFFFFFFFF, 1, 1, 16, aux0=big >> 32)) == [
        big * 4, 1024, 0, 0, 0, (big // 16 + 7) // 8 * 4, 0, 4]
    assert required(plan2(22, big & 0xFFFFFFFF, 1, 1, 16, aux0=big >> 32)) == [
        (big // 16 + 7) // 8 * 4, 1024, 0, 0, 0, big * 4, 0, 4]


def test_schema2_harness_reductions():
    """Ops 26 (residual and its float64 sum of squares) and 27 (norm and
    clip): float64 partials and their total in in4, the float64 results in
    out1; written in4 may alias nothing."""
    n, g = 1000, 16
    ws = (1024 + 1) * 8
    assert required(plan2(26, n, 1, 1, g, aux0=0x3C000000)) == [
        4 * n, ((n + g - 1) // g + 7) // 8 * 4, 64 * g, 0, ws, 4 * n, 8, 4]
    assert required(plan2(27, n, 1, 1, 8, aux0=0, aux1=0x3FF00000)) == [4 * n, 0, 0, 0, ws, 4 * n, 16, 4]
    for words, name in ((plan2(26, 0, 1, 1, g), "vq2-invalid-geometry"), (plan2(26, n, 1, 1, g, flags=1),
                        "vq2-unsupported-flags"), (plan2(27, n, 1, 1, 8, aux2=1), "vq2-invalid-aux-word"),
                        (plan2(27, n, 1, 1, 8, batch=2), "vq2-invalid-batch"), (plan2(28, n, 1, 1, 8),
                        "vq2-operation-out-of-range")):
        assert refusal(words)[1].endswith(name), name
    caps = [4 * n, 0, 0, 0, ws, 4 * n, 16, 4]
    assert validate_buffers(plan2(27, n, 1, 1, 8), caps, [1, 0, 0, 0, 2, 3, 4, 5]) == 0
    assert validate_buffers(plan2(27, n, 1, 1, 8), caps, [1, 0, 0, 0, 1, 3, 4, 5]) != 0


def test_schema2_refusals_are_named():
    cases = [
        (plan2(15, 1, 1, 1, 8), "vq2-operation-out-of-range"),
        (plan2(16, 1, 1, 1, 12), "vq2-unsupported-group"),
        (plan2(16, 1, 1, 1, 8, flags=1), "vq2-unsupported-flags"),
        (plan2(16, 0, 1, 1, 8), "vq2-invalid-geometry"),
        (plan2(16, 1, 1, 1, 8, batch=0), "vq2-invalid-batch"),
        (plan2(17, 1, 1, 1, 8, batch=2), "vq2-invalid-batch"),
        (plan2(18, 64, 1, 1, 8, aux0=0), "vq2-invalid-aux-word"),
        (plan2(18, 64, 1, 1, 8, aux0=9), "vq2-invalid-aux-word"),
        (plan2(19, 64, 1, 1, 8, aux0=3), "vq2-invalid-aux-word"),
        (plan2(19, 64, 1, 1, 8, batch=2, aux1=2), "vq2-invalid-aux-word"),
        (plan2(21, 0, 1, 1, 8), "vq2-invalid-geometry"),
        (plan2(24, 64, 1, 1, 8, aux0=8, aux1=4), "vq2-unsupported-flags"),
        (plan2(24, 64, 1, 1, 8, flags=1, aux0=9, aux1=4), "vq2-invalid-aux-word"),
        (plan2(24, 64, 1, 1, 8, flags=1, aux0=8, aux1=33), "vq2-invalid-aux-word"),
        (plan2(24, 64, 1, 1, 8, flags=1, aux0=8, aux1=4, batch=0), "vq2-invalid-batch"),
        (plan2(28, 64, 1, 1, 8), "vq2-operation-out-of-range"),
        (plan2(25, 64, 1, 1, 8, flags=2, aux0=8, aux1=4), "vq2-unsupported-flags"),
        (plan2(25, 64, 1, 1, 8, aux0=9, aux1=4), "vq2-invalid-aux-word"),
        (plan2(25, 64, 1, 1, 8, aux0=8, aux1=4, batch=2), "vq2-invalid-batch"),
        (plan2(25, 7, 1, 1, 8, aux0=1, aux1=4), "vq2-invalid-geometry"),
        (plan2(21, 1, 1, 1, 8, aux0=1 << 8), "vq2-address-limit-exceeded"),
        (plan2(16, 1 << 21, 1, 1, 8), "vq2-invalid-geometry"),
    ]
    for words, name in cases:
        rc, msg = refusal(words)
        assert rc in (SHAPE, SIZE) and msg.endswith(name), (words, msg)
    bad = plan2(16, 1, 1, 8, 8)
    bad[13] = 1
    assert refusal(bad)[1].endswith("vq2-nonzero-reserved-word")


def test_schema2_outputs_must_not_alias_and_unused_slots_may_be_null():
    from abi_util import last_error
    words = plan2(20, 1000, 1, 1, 8)
    caps = required(words)
    ids = [1, 2, 3, 4, 0, 6, 7, 8]
    assert validate_buffers(words, caps, ids) == 0
    for inp in range(4):
        bad = list(ids)
        bad[5] = bad[inp]
        assert validate_buffers(words, caps, bad) == SHAPE and last_error().endswith("vq2-output-aliases-input")
    bad = list(ids)
    bad[6] = bad[5]
    assert validate_buffers(words, caps, bad) == SHAPE and last_error().endswith("vq2-output-aliases-input")
    bad = list(ids)
    bad[7] = bad[6]
    assert validate_buffers(words, caps, bad) == SHAPE and last_error().endswith("vq2-status-aliases-operand")
    bad = list(ids)
    bad[3] = 0
    assert validate_buffers(words, caps, bad) == SHAPE and last_error().endswith("vq2-null-allocation-identity")


def test_schema2_tile32_repack_and_prepacked_dense():
    n, k, g, e = 1000, 4096, 16, 3
    tile32 = (n + 31) // 32 * 32 * (k // g) // 2
    assert required(plan2(23, n, 1, k, g, batch=e)) == [e * n * k // g // 2, 0, 0, 0, 0, e * tile32, 0, 4]
    assert required(plan2(16, 1, n, k, g, flags=6, batch=e))[1] == e * tile32
    for words, name in ((plan2(16, 1, n, k, g, flags=4), "vq2-unsupported-flags"),
                        (plan2(16, 1, n, 40 * g, g, flags=6), "vq2-unsupported-flags"),
                        (plan2(23, n, 1, 40 * g, g), "vq2-invalid-geometry"),
                        (plan2(23, n, 2, k, g), "vq2-invalid-geometry")):
        assert refusal(words)[1].endswith(name), words
