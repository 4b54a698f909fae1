"""CPU restatement of the reference's NF4 comparator: nf4-decode/v1 and
nf4-gemv/v1 (bitsandbytes' NF4 with double quantisation, read in its stored
form). TEST INFRASTRUCTURE ONLY: the parity checker of the CUDA kernels in
`alelyon_compute_kit.nf4`, used by tests/, never by the product.

Followed statement by statement (FP32 numpy operations round once each, as
the shaders' `precise` arithmetic does):
  decode   src/alelyon_compute_kit/_kit/kernels/nf4_decode.comp:108-158
           (member_of, the NaN guard, scale = fl(map[q] * absmax2),
           absmax = fl(scale + offset), value = fl(code[index] * absmax), the
           high nibble first, then the storage rounding :70-105)
  gemv     src/alelyon_compute_kit/_kit/kernels/nf4_gemv.comp:203-266 (the
           group guards, one member lookup per column when its first and
           last values share a member, the weight rounded to 16 bits and
           widened, lane l summing words l, l + 64, ... in order and the
           values of a word in order, then the tree s = 32, 16, ..., 1)
  plans    src/alelyon_compute_kit/_kit/src/nf4_ops.rs:117-191 (decode) and
           :515-569 (gemv): the refusals by name, values_covered, src_limit

Pinned against both shaders compiled for the host (oracle/nf4_ref.py) in
tests/test_oracle_golden.py.
"""
from __future__ import annotations

import numpy as np

BLOCK = 64
NESTED = 256
NESTED_VALUES = BLOCK * NESTED
TABLE_ENTRIES = 16 + 256
MAX_VALUES = 1 << 31
GEMV_MAX_ROWS = 16
GEMV_LANES = 64
GROUP_WORDS = 3
MAX_GRID = 65535
U32_MAX = (1 << 32) - 1
NAN_BITS = 0x7FC00000


class Nf4PlanError(ValueError):
    """A refused call; the message is the reference's refusal name."""


# ---------------------------------------------------------------- roundings --

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """FP32 -> bf16, round to nearest even, NaN kept quiet (nf4_decode.comp:72-79)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = ((b & 0x7F800000) == 0x7F800000) & ((b & 0x007FFFFF) != 0)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF
    return np.where(nan, (b >> 16) | 0x0040, rounded).astype(np.uint16)


def f16_bits(x: np.ndarray) -> np.ndarray:
    """FP32 -> fp16 by convert/v1's integer routine: round to nearest even,
    NaN -> sign | 0x7E00 (nf4_decode.comp:83-103)."""
    w = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.int64)
    sign = (w >> 16) & 0x8000
    e = (w >> 23) & 0xFF
    m = w & 0x7FFFFF
    out = np.zeros(w.shape, np.int64)
    special = e == 0xFF
    out[special] = sign[special] | np.where(m[special] != 0, 0x7E00, 0x7C00)
    he = e - 112
    big = ~special & (he >= 31)
    out[big] = sign[big] | 0x7C00
    sub = ~special & ~big & (he <= 0)
    tiny = sub & (he < -10)
    out[tiny] = sign[tiny]
    mid = sub & ~tiny
    if mid.any():
        mf = m[mid] | 0x800000
        shift = 14 - he[mid]
        q = mf >> shift
        rem = mf & ((np.int64(1) << shift) - 1)
        half = np.int64(1) << (shift - 1)
        q = q + ((rem > half) | ((rem == half) & ((q & 1) != 0)))
        out[mid] = sign[mid] | q
    norm = ~special & ~big & ~sub
    if norm.any():
        h = (he[norm] << 10) | (m[norm] >> 13)
        rem = m[norm] & 0x1FFF
        h = h + ((rem > 0x1000) | ((rem == 0x1000) & ((h & 1) != 0)))
        out[norm] = sign[norm] | h
    return out.astype(np.uint16)


def widen_bf16(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, np.uint32) << 16).astype(np.uint32).view(np.float32)


def widen_f16(h: np.ndarray) -> np.ndarray:
    """fp16 -> FP32, exact (nf4_gemv.comp's f16_to_f32)."""
    h = np.asarray(h, np.uint32)
    sign = (h & 0x8000) << 16
    e = (h >> 10) & 0x1F
    m = h & 0x3FF
    out = np.where(e == 0x1F, sign | 0x7F800000 | (m << 13), sign | ((e + 112) << 23) | (m << 13))
    zero = (e == 0) & (m == 0)
    out = np.where(zero, sign, out)
    subn = (e == 0) & (m != 0)
    if subn.any():
        mm = m[subn]
        t = np.floor(np.log2(mm)).astype(np.uint32)
        out[subn] = sign[subn] | ((t + 103) << 23) | ((mm << (23 - t)) & 0x7FFFFF)
    return out.astype(np.uint32).view(np.float32)


def narrow(storage: int, x: np.ndarray) -> np.ndarray:
    if storage == 0:
        return np.asarray(x, np.float32)
    return bf16_bits(x) if storage == 1 else f16_bits(x)


def widen(elem: int, h: np.ndarray) -> np.ndarray:
    return widen_bf16(h) if elem == 0 else widen_f16(h)


# ------------------------------------------------------------------- plans --

def values_covered(packed_bytes: int, absmax_q_bytes: int, absmax2_bytes: int) -> int:
    """Values the three stored buffers cover, each read in whole u32 words (nf4_ops.rs:113-122)."""
    return min(8 * (packed_bytes // 4), 4 * (absmax_q_bytes // 4) * BLOCK, (absmax2_bytes // 4) * NESTED_VALUES)


def decode_plan(n: int, members: int, selected: int, member_values: int, src_base: int, covered: int,
                storage: int) -> dict:
    """nf4_ops.rs:158-204: the push words of one decode, or Nf4PlanError."""
    if storage not in (0, 1, 2):
        raise Nf4PlanError("nf4-storage-out-of-range")
    if n == 0:
        raise Nf4PlanError("nf4-zero-values")
    if n > MAX_VALUES:
        raise Nf4PlanError("nf4-value-limit-exceeded")
    if members == 0:
        raise Nf4PlanError("nf4-members-out-of-range")
    member_values = 0 if selected == 0 else member_values
    if selected and (member_values == 0 or member_values % BLOCK or selected * member_values != n):
        raise Nf4PlanError("nf4-selection-out-of-range")
    if src_base % NESTED_VALUES or src_base >= covered:
        raise Nf4PlanError("nf4-base-out-of-range")
    src_limit = min(covered - src_base, U32_MAX)
    if selected == 0 and n > src_limit:
        raise Nf4PlanError("nf4-source-too-small")
    return {"n": n, "words": (n + 7) // 8, "members": members, "selected": selected,
            "member_values": member_values, "src_base": src_base, "src_limit": src_limit}


def gemv_plan(rows: int, max_rows: int, n: int, k: int, lda: int, groups: int, members: int, src_base: int,
              covered: int, elem: int) -> dict:
    """nf4_ops.rs:515-569: the push words of one grouped GEMV, or Nf4PlanError."""
    if elem not in (0, 1):
        raise Nf4PlanError("nf4-matmul-elem-out-of-range")
    if rows == 0 or max_rows == 0 or n == 0 or k == 0:
        raise Nf4PlanError("nf4-matmul-zero-extent")
    if groups == 0 or groups > MAX_GRID:
        raise Nf4PlanError("nf4-matmul-groups-out-of-range")
    if max_rows > rows:
        raise Nf4PlanError("nf4-matmul-rows-out-of-range")
    if max_rows > GEMV_MAX_ROWS:
        raise Nf4PlanError("nf4-gemv-rows-above-16")
    if k % 8:
        raise Nf4PlanError("nf4-matmul-row-not-whole-words")
    lda = k if lda == 0 else lda
    if lda < k:
        raise Nf4PlanError("nf4-matmul-pitch-below-width")
    if lda % 8:
        raise Nf4PlanError("nf4-gemv-pitch-not-whole-words")
    if members == 0:
        raise Nf4PlanError("nf4-members-out-of-range")
    if src_base % NESTED_VALUES or src_base >= covered:
        raise Nf4PlanError("nf4-base-out-of-range")
    weight = n * k
    past_base = covered - src_base
    if weight > past_base:
        raise Nf4PlanError("nf4-source-too-small")
    a_span = (rows - 1) * lda + k
    if a_span > U32_MAX or rows * n > U32_MAX or weight > U32_MAX:
        raise Nf4PlanError("nf4-matmul-address-limit-exceeded")
    return {"n": n, "k": k, "lda": lda, "rows": rows, "src_base": src_base,
            "src_limit": min(past_base, U32_MAX - src_base), "members": members}


# ------------------------------------------------------------------ decode --

def _member_of(starts_lo: np.ndarray, members: int, s: np.ndarray) -> np.ndarray:
    """The last start at or below s (the shader's binary search over the low
    words of the int64 starts, members entries)."""
    lo = np.zeros(s.shape, np.int64)
    hi = np.full(s.shape, members, np.int64)
    while True:
        active = hi - lo > 1
        if not active.any():
            return lo
        mid = (lo + hi) // 2
        le = starts_lo[np.minimum(mid, len(starts_lo) - 1)] <= s
        lo = np.where(active & le, mid, lo)
        hi = np.where(active & ~le, mid, hi)


def _abs_of(s: np.ndarray, absq_words: np.ndarray, absmax2: np.ndarray, tables: np.ndarray,
            offset: np.ndarray) -> np.ndarray:
    b = s // BLOCK
    q = (absq_words[b // 4] >> (8 * (b % 4)).astype(np.uint32)) & 0xFF
    scale = (tables[16 + q].astype(np.float32) * absmax2[b // NESTED]).astype(np.float32)
    return (scale + offset).astype(np.float32)


def _values(word: np.ndarray, absmax: np.ndarray, tables: np.ndarray) -> np.ndarray:
    """The 8 values of packed words: byte k // 2, the high nibble first."""
    k = np.arange(8, dtype=np.uint32)
    byte = (word[:, None] >> (8 * (k >> 1))) & 0xFF
    index = np.where((k & 1) == 0, byte >> 4, byte & 0xF)
    return (tables[index].astype(np.float32) * absmax[:, None]).astype(np.float32)


def decode(packed: np.ndarray, absmax_q: np.ndarray, absmax2: np.ndarray, tables: np.ndarray,
           starts: np.ndarray, offsets: np.ndarray, n: int, *, ids: np.ndarray | None = None,
           member_values: int = 0, src_base: int = 0, storage: int = 0) -> np.ndarray:
    """nf4-decode/v1 of `n` values: FP32 (storage 0) or the 16-bit words of
    bf16 (1) or fp16 (2). `packed`, `absmax_q` are byte arrays, `starts` and
    `ids` int64."""
    pw = np.frombuffer(np.ascontiguousarray(packed, np.uint8).tobytes() + b"\0" * (-len(packed) % 4), np.uint32)
    qw = np.frombuffer(np.ascontiguousarray(absmax_q, np.uint8).tobytes() + b"\0" * (-len(absmax_q) % 4),
                       np.uint32)
    a2 = np.ascontiguousarray(absmax2, np.float32)
    tb = np.ascontiguousarray(tables, np.float32)
    st = np.ascontiguousarray(starts, np.int64)
    of = np.ascontiguousarray(offsets, np.float32)
    members = len(st)
    selected = 0 if ids is None else len(ids)
    plan = decode_plan(n, members, selected, member_values, src_base,
                       values_covered(len(packed), len(absmax_q), 4 * len(a2)), storage)
    st_lo = (st.view(np.uint64) & U32_MAX).astype(np.int64)
    words = plan["words"]
    i0 = np.arange(words, dtype=np.int64) * 8
    if selected == 0:
        m = _member_of(st_lo, members, i0)
        s0 = i0
        bad = np.zeros(words, bool)
    else:
        iv = np.ascontiguousarray(ids, np.int64).view(np.uint64)
        j = i0 // plan["member_values"]
        raw = iv[j]
        m = (raw & U32_MAX).astype(np.int64)
        bad = ((raw >> 32) != 0) | (m >= members)
        s0 = np.where(bad, 0, st_lo[np.minimum(m, members - 1)]) + (i0 - j * plan["member_values"])
        s0 = s0 & U32_MAX   # u32 arithmetic
    count = np.minimum(8, n - i0)
    limit = plan["src_limit"]
    bad = bad | (s0 >= limit) | (count > limit - s0)
    s = (src_base + s0) & U32_MAX
    good = ~bad
    vals = np.full((words, 8), np.uint32(NAN_BITS).view(np.float32), np.float32)
    if good.any():
        sg = s[good]
        absmax = _abs_of(sg, qw, a2, tb, of[np.minimum(m[good], members - 1)])
        vals[good] = _values(pw[sg // 8], absmax, tb)
    flat = vals.reshape(-1)[:n]
    return narrow(storage, flat)


# -------------------------------------------------------------------- gemv --

def gemv(a16: np.ndarray, packed: np.ndarray, absmax_q: np.ndarray, absmax2: np.ndarray, tables: np.ndarray,
         starts: np.ndarray, offsets: np.ndarray, groups: np.ndarray, *, rows: int, n: int, k: int, lda: int = 0,
         src_base: int = 0, elem: int = 0, c: np.ndarray | None = None) -> np.ndarray:
    """nf4-gemv/v1: C[rowStart + m, col] for every group (rowStart, mRows,
    wBase) of `groups` (G x 3 u32) that passes the shader's guards; `a16` is
    A's 16-bit words (rows x lda). Entries of C that no group writes keep
    `c`'s values (zeros if None)."""
    pw = np.frombuffer(np.ascontiguousarray(packed, np.uint8).tobytes() + b"\0" * (-len(packed) % 4), np.uint32)
    qw = np.frombuffer(np.ascontiguousarray(absmax_q, np.uint8).tobytes() + b"\0" * (-len(absmax_q) % 4),
                       np.uint32)
    a2 = np.ascontiguousarray(absmax2, np.float32)
    tb = np.ascontiguousarray(tables, np.float32)
    st = np.ascontiguousarray(starts, np.int64)
    of = np.ascontiguousarray(offsets, np.float32)
    gt = np.ascontiguousarray(groups, np.uint32).reshape(-1, GROUP_WORDS)
    members = len(st)
    max_rows = int(gt[:, 1].max()) if len(gt) else 0
    plan = gemv_plan(rows, max_rows, n, k, lda, len(gt), members, src_base,
                     values_covered(len(packed), len(absmax_q), 4 * len(a2)), elem)
    lda, limit = plan["lda"], plan["src_limit"]
    st_lo = (st.view(np.uint64) & U32_MAX).astype(np.int64)
    a_flat = np.ascontiguousarray(a16, np.uint16).reshape(-1)
    out = np.zeros(rows * n, np.float32) if c is None else np.array(c, np.float32).reshape(-1)
    words = k // 8
    cols = np.arange(n, dtype=np.int64)
    for row_start, m_rows, w_base in gt.astype(np.int64):
        if (m_rows == 0 or m_rows > GEMV_MAX_ROWS or row_start + m_rows > U32_MAX or row_start + m_rows > rows
                or (w_base & 7) or w_base > limit or (n * k) & U32_MAX > limit - w_base):
            continue
        col0 = w_base + cols * k
        first = _member_of(st_lo, members, col0)
        one = first == _member_of(st_lo, members, col0 + k - 1)
        # weights: (n, words, 8) decoded, rounded to 16 bits, widened
        v0 = col0[:, None] + 8 * np.arange(words, dtype=np.int64)[None, :]
        off = np.where(one[:, None], of[first][:, None], of[_member_of(st_lo, members, v0)])
        s = (src_base + v0) & U32_MAX
        absmax = _abs_of(s.reshape(-1), qw, a2, tb, off.reshape(-1).astype(np.float32))
        w16 = narrow(1 + elem, _values(pw[(s // 8).reshape(-1)], absmax, tb))
        wf = widen(elem, w16).reshape(n, words, 8)
        for mm in range(int(m_rows)):
            base = (row_start + mm) * lda
            af = widen(elem, a_flat[base: base + k]).reshape(words, 8)
            acc = np.zeros((n, GEMV_LANES), np.float32)
            for t in range((words + GEMV_LANES - 1) // GEMV_LANES):
                j = np.arange(GEMV_LANES) + GEMV_LANES * t
                valid = j < words
                jj = np.minimum(j, words - 1)
                for e in range(8):
                    prod = (af[jj, e][None, :] * wf[:, jj, e]).astype(np.float32)
                    acc = np.where(valid[None, :], (acc + prod).astype(np.float32), acc)
            half = GEMV_LANES // 2
            while half:
                acc[:, :half] = (acc[:, :half] + acc[:, half: 2 * half]).astype(np.float32)
                half //= 2
            out[(row_start + mm) * n + cols] = acc[:, 0]
    return out.reshape(rows, n)
