"""CPU oracle for the vq4/v1 hot path -- TEST INFRASTRUCTURE ONLY.

This module is a checker. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it. The
product (`alelyon-compute-kit_b200/`) never imports, links or runs anything
under `oracle/`; its device path fails loudly when the CUDA library is missing.

It restates, in plain numpy, the reference's algorithms for the path:

* the wire format, `storage_layout` and nibble packing
  (reference `src/alelyon_compute_kit/_kit/python/vq.py:70-151`);
* `encode`, float64 squared-L2 argmin with lowest-index ties
  (`vq.py:154-179`);
* `VQArray.decode` (`vq.py:117-121`);
* `fit_codebook` and `_reseed` (`vq.py:182-257`);
* the vq4 shader's packed-pair matmul, op 2 (`_kit/kernels/vq4.comp:165-176`):
  FP32, sequential k order, product and sum rounded separately (`precise`);
* the vq4 shader's AdamW, op 3 (`vq4.comp:87-116`), FP32 in shader order;
* the shader's FP32 encode, op 0 (`vq4.comp:118-144`), used only to count how
  often the reference's two encoders disagree;
* float64 references for the north-star products (dense X times coded W, and
  both operands coded), `Y = X @ decode(W).T` and `decode(A) @ decode(B)`.

Pinning: the format, `encode`, `decode` and `fit_codebook` restatements are
checked against golden vectors produced by the reference's own Python code
(`tests/golden/gen_golden.py`, run in a container that has the reference).
The shader restatements (matmul op 2, AdamW op 3, FP32 encode op 0, decode
op 1, the status bits) are checked bit for bit against the reference's own
`vq4.comp` source compiled for the host CPU (`oracle/vq4_ref.py`,
`oracle/vq4_shim.h`) on every case the GPU tests use. That build performs
each FP32 operation once, IEEE-rounded, in the shader's source order.
"""
from __future__ import annotations

import math
import struct

import numpy as np

ENTRIES = 16
GROUPS = (8, 16, 32)
SCHEMA = 1
HEADER = struct.Struct("<8sIIIIQQ")          # vq.py:26
MAGIC = b"ACKVQ4\0\0"                        # vq.py:27


# ---------------------------------------------------------------- format ----

def layout(shape, group: int) -> dict:
    """Byte accounting of one coded tensor (vq.py:70-82)."""
    elements = int(np.prod(shape, dtype=np.int64))
    vectors = (elements + group - 1) // group
    code_bytes = ((vectors + 7) // 8) * 4
    book = ENTRIES * group * 4
    meta = HEADER.size + 8 * len(shape)
    total = code_bytes + book + meta
    return {"elements": elements, "vectors": vectors, "code_bytes": code_bytes,
            "codebook_bytes": book, "metadata_bytes": meta, "serialized_bytes": total,
            "payload_bytes": code_bytes + book, "bits_per_value": 8 * total / elements,
            "sub_bit": 8 * total < elements}


def pack(indices: np.ndarray) -> np.ndarray:
    """Eight 4-bit indices per little-endian u32, vector 8w+j at bits 4j (vq.py:175-178)."""
    idx = np.asarray(indices, dtype=np.uint32).reshape(-1)
    words = np.zeros((idx.size + 7) // 8, dtype=np.uint32)
    for lane in range(8):
        part = idx[lane::8]
        words[:part.size] |= part << np.uint32(4 * lane)
    return words


def unpack(words: np.ndarray, vectors: int) -> np.ndarray:
    """Inverse of `pack` for the first `vectors` indices (vq.py:119-120)."""
    pos = np.arange(vectors, dtype=np.int64)
    return ((np.asarray(words, dtype=np.uint32)[pos // 8] >> ((pos % 8) * 4).astype(np.uint32))
            & np.uint32(15)).astype(np.uint32)


def to_bytes(shape, group: int, codes: np.ndarray, book: np.ndarray) -> bytes:
    """Wire image: header, dims, LE f32 codebook, LE u32 codes (vq.py:123-128)."""
    lay = layout(shape, group)
    head = HEADER.pack(MAGIC, SCHEMA, group, len(shape), 0, lay["elements"], lay["code_bytes"])
    dims = struct.pack("<" + "Q" * len(shape), *shape)
    return head + dims + np.asarray(book, "<f4").tobytes() + np.asarray(codes, "<u4").tobytes()


def from_bytes(data: bytes):
    """Parse a wire image into (shape, group, codes, book) (vq.py:130-151)."""
    magic, schema, group, rank, reserved, elements, code_bytes = HEADER.unpack_from(data)
    if magic != MAGIC or schema != SCHEMA or reserved or not 1 <= rank <= 6:
        raise ValueError("unsupported vq artifact header")
    shape = struct.unpack_from("<" + "Q" * rank, data, HEADER.size)
    lay = layout(shape, group)
    if elements != lay["elements"] or code_bytes != lay["code_bytes"] or len(data) != lay["serialized_bytes"]:
        raise ValueError("vq header disagrees with its dimensions")
    start = HEADER.size + 8 * rank
    book = np.frombuffer(data, "<f4", ENTRIES * group, start).reshape(ENTRIES, group).astype(np.float32)
    codes = np.frombuffer(data, "<u4", lay["code_bytes"] // 4, start + 64 * group).astype(np.uint32)
    return tuple(int(d) for d in shape), group, codes, book


# ------------------------------------------------------------ encode/decode ----

def decode(codes: np.ndarray, book: np.ndarray, elements: int, group: int) -> np.ndarray:
    """Gather one code vector per group and trim the tail (vq.py:117-121)."""
    vectors = (elements + group - 1) // group
    idx = unpack(codes, vectors)
    return np.asarray(book, np.float32)[idx].reshape(-1)[:elements].copy()


def nearest(values: np.ndarray, book: np.ndarray, group: int) -> np.ndarray:
    """Per-vector index of the float64-nearest code vector (vq.py:161-174).

    Distances are accumulated in component order j = 0..g-1 as float64
    `d += (v_j - b_j) * (v_j - b_j)`, exactly as the reference's numpy loop
    does; ties keep the lowest index (`np.argmin`). A partial final vector
    compares only its valid components (`vq.py:171-172`).
    """
    x = np.asarray(values, dtype=np.float32).reshape(-1)
    vectors = (x.size + group - 1) // group
    padded = np.zeros(vectors * group, dtype=np.float32)
    padded[:x.size] = x
    v = padded.reshape(-1, group)
    b = np.asarray(book, np.float32).astype(np.float64)
    tail = x.size % group
    chosen = np.empty(vectors, dtype=np.uint32)
    step = 8192
    for start in range(0, vectors, step):
        chunk = v[start:start + step].astype(np.float64)
        dist = np.zeros((len(chunk), ENTRIES), dtype=np.float64)
        last = start + len(chunk) == vectors
        for j in range(group):
            delta = chunk[:, j, None] - b[None, :, j]
            if last and tail and j >= tail:
                delta[-1] = 0.0
            dist += delta * delta
        chosen[start:start + len(chunk)] = np.argmin(dist, axis=1).astype(np.uint32)
    return chosen


def encode(values: np.ndarray, book: np.ndarray, group: int) -> np.ndarray:
    """Packed u32 code image of `values` (vq.py:154-179)."""
    return pack(nearest(values, book, group))


def nearest_fp32_shader(values: np.ndarray, book: np.ndarray, group: int) -> np.ndarray:
    """The shader's FP32 encode (vq4.comp:118-144): sequential `precise`
    float32 sum of rounded squares, strict `<` so ties keep the lowest index.
    Pinned to the compiled shader (`vq4_ref.encode`)."""
    x = np.asarray(values, dtype=np.float32).reshape(-1)
    vectors = (x.size + group - 1) // group
    padded = np.zeros(vectors * group, dtype=np.float32)
    padded[:x.size] = x
    v = padded.reshape(-1, group)
    b = np.asarray(book, np.float32)
    tail = x.size % group
    dist = np.zeros((vectors, ENTRIES), dtype=np.float32)
    for j in range(group):
        delta = (v[:, j, None] - b[None, :, j]).astype(np.float32)
        sq = (delta * delta).astype(np.float32)
        if tail and j >= tail:
            sq[-1] = 0.0
        dist = (dist + sq).astype(np.float32)
    return np.argmin(dist, axis=1).astype(np.uint32)


def near_ties(values, book, group, rel=1e-6):
    """Indices of vectors whose best and second-best float64 distances are
    within `rel` of each other: where FP32 and FP64 encoders may disagree."""
    x = np.asarray(values, dtype=np.float32).reshape(-1)
    vectors = x.size // group
    v = x[:vectors * group].reshape(-1, group).astype(np.float64)
    b = np.asarray(book, np.float32).astype(np.float64)
    d = ((v[:, None, :] - b[None, :, :]) ** 2).sum(-1)
    d.sort(axis=1)
    gap = d[:, 1] - d[:, 0]
    return np.nonzero(gap <= rel * np.maximum(d[:, 1], 1e-300))[0]


# ------------------------------------------------------------ codebook fit ----

def _reseed(sample: np.ndarray, book: np.ndarray) -> np.ndarray:
    """The sample vector farthest from the current book (vq.py:232-257)."""
    gap = ((sample.astype(np.float64)[:, None, :] - book.astype(np.float64)[None, :, :]) ** 2).sum(-1).min(1)
    return sample[int(gap.argmax())]


def fit_codebook(values, group: int = 16, iterations: int = 4, sample_vectors: int = 4096,
                 init=None) -> np.ndarray:
    """Lloyd fit with farthest-point reseed and warm start (vq.py:182-229)."""
    x = np.asarray(values, dtype=np.float32).reshape(-1)
    complete = x[:x.size // group * group].reshape(-1, group)
    pick = np.linspace(0, len(complete) - 1, min(len(complete), sample_vectors), dtype=np.int64)
    sample = complete[pick]
    if init is None:
        book = sample[np.linspace(0, len(sample) - 1, ENTRIES, dtype=np.int64)].copy()
    else:
        book = np.array(init, dtype=np.float32).reshape(ENTRIES, group).copy()
    for _ in range(iterations):
        idx = nearest(sample, book, group)
        kept = set()
        empty = set(range(ENTRIES)) - set(np.unique(idx).tolist())
        reachable = [e for e in empty if not any(np.array_equal(book[e], book[j]) for j in range(e))]
        if init is not None and len(sample) < len(complete) and reachable:
            kept = set(np.unique(nearest(complete, book, group)).tolist())
        for entry in range(ENTRIES):
            selected = sample[idx == entry]
            if len(selected):
                book[entry] = selected.mean(axis=0, dtype=np.float64).astype(np.float32)
            elif entry not in kept:
                book[entry] = _reseed(sample, book)
    return book


# ------------------------------------------------------ shader arithmetic ----

def matmul_shader(a_codes, a_book, b_codes, b_book, m, n, k, group, flags) -> np.ndarray:
    """vq4.comp op 2 (165-176): C[row,col] = sum over inner in order of
    fl32(a*b), accumulated with a separately rounded FP32 add. Flag bit 0: A
    is stored K x M; bit 1: B is stored N x K. Pinned to the compiled shader
    (`vq4_ref.matmul`)."""
    a = decode(a_codes, a_book, m * k, group)
    b = decode(b_codes, b_book, k * n, group)
    A = a.reshape(k, m).T if flags & 1 else a.reshape(m, k)
    B = b.reshape(n, k).T if flags & 2 else b.reshape(k, n)
    total = np.zeros((m, n), dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        for inner in range(k):
            product = (A[:, inner, None] * B[None, inner, :]).astype(np.float32)
            total = (total + product).astype(np.float32)
    return total


def adamw_shader(w, m, v, g, coefficients) -> tuple:
    """vq4.comp op 3, `adamw_value` (87-116), in FP32 with every operation
    rounded on its own (`precise`, no fused multiply-add): returns
    (w', m', v') as float32 arrays. Pinned to the compiled shader
    (`vq4_ref.adamw`)."""
    f32 = np.float32
    lr, b1, b2, eps, decay, c1, c2 = (f32(c) for c in coefficients)
    one = f32(1.0)
    w, m, v, g = (np.asarray(t, f32) for t in (w, m, v, g))
    with np.errstate(all="ignore"):
        next_m = (b1 * m) + ((one - b1) * g)                 # vq4.comp:103
        next_v = (b2 * v) + ((one - b2) * (g * g))           # vq4.comp:104
        corrected_m = next_m / c1                            # vq4.comp:105
        corrected_v = next_v / c2                            # vq4.comp:106
        denominator = np.sqrt(corrected_v) + eps             # vq4.comp:107
        decayed = w * (one - lr * decay)                     # vq4.comp:108
        next_w = decayed - (lr * corrected_m) / denominator  # vq4.comp:109
    return (next_w.astype(f32), next_m.astype(f32), next_v.astype(f32))


def adamw_coefficients(lr, beta1, beta2, eps, weight_decay, step) -> np.ndarray:
    """The seven FP32 coefficients the host passes (vq.py:357-358)."""
    return np.array([lr, beta1, beta2, eps, weight_decay, 1 - beta1 ** step, 1 - beta2 ** step],
                    dtype=np.float32)


# ------------------------------------------------- float64 product references ----

def dense_nt_f64(x: np.ndarray, w_codes, w_book, n: int, k: int, group: int) -> np.ndarray:
    """Y = X @ decode(W).T in float64, W stored N x K (north-star op A7)."""
    wd = decode(w_codes, w_book, n * k, group).reshape(n, k).astype(np.float64)
    return np.asarray(x, np.float64) @ wd.T


def coded_f64(a_codes, a_book, b_codes, b_book, m, n, k, group, flags) -> np.ndarray:
    """decode(A) @ decode(B) in float64 with the op-2 transpose flags."""
    a = decode(a_codes, a_book, m * k, group).astype(np.float64)
    b = decode(b_codes, b_book, k * n, group).astype(np.float64)
    A = a.reshape(k, m).T if flags & 1 else a.reshape(m, k)
    B = b.reshape(n, k).T if flags & 2 else b.reshape(k, n)
    return A @ B


def normwise_error(y, y64, absolute_products) -> float:
    """max |y - y64| / sum_k |a_k b_k|, the GEMM tolerance metric."""
    denom = np.maximum(np.asarray(absolute_products, np.float64), 1e-300)
    return float(np.max(np.abs(np.asarray(y, np.float64) - y64) / denom))


# ----------------------------------------------------------- seeded inputs ----

def gaussian(shape, std, seed) -> np.ndarray:
    """N(0, std^2) float32 draws from `default_rng(seed)`."""
    return (np.random.default_rng(seed).standard_normal(shape) * std).astype(np.float32)


def block_normalised(values: np.ndarray, group: int) -> np.ndarray:
    """Each consecutive `group`-value block divided by its L2 norm (cfg 2, cfg 5a)."""
    x = np.asarray(values, np.float32).reshape(-1, group).astype(np.float64)
    norm = np.linalg.norm(x, axis=1, keepdims=True)
    norm[norm == 0] = 1.0
    return (x / norm).astype(np.float32).reshape(np.shape(values))


def duplicate_heavy(count_vectors: int, group: int, seed: int = 10) -> np.ndarray:
    """16 exact atoms, atom 0 at 85% occupancy and atoms 1..15 sharing 15%,
    shuffled with a fixed seed (cfg 5b)."""
    rng = np.random.default_rng(seed)
    atoms = rng.standard_normal((ENTRIES, group)).astype(np.float32)
    rare = int(round(count_vectors * 0.15))
    idx = np.zeros(count_vectors, dtype=np.int64)
    idx[:rare] = 1 + (np.arange(rare) % (ENTRIES - 1))
    rng.shuffle(idx)
    return atoms[idx].reshape(-1)
