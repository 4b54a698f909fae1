"""Vector-coded tensors (vq4/v1) and their B200 operations.

Drop-in for the reference's `vq` module (`src/alelyon_compute_kit/_kit/python/
vq.py`): the same format and public names (`storage_layout`, `VQArray`,
`encode`, `fit_codebook`, `VQDevice`, `VQAdamW`), the same validation and
refusal messages, the same bounds on the schema-1 device calls.

Each 4-bit index selects one of 16 FP32 code vectors of 8, 16 or 32 values;
one codebook per tensor; eight indices per little-endian u32 word.

CPU work, as in the reference: `fit_codebook` (Lloyd iterations on a strided
calibration sample) and the module-level `encode`, which `fit_codebook` uses
on that sample. Device work goes through `VQDevice` and the C ABI; there is
no CPU fallback on that path.

Additions, all on `VQDevice` and none changing an existing signature:
`matmul_dense` / `matmul_dense_grouped` (FP32 activations times coded
weights), `matmul_coded` (both operands coded, no MAC bound),
`encode_large` / `decode_large` (64-bit value counts), and `adamw_fused`,
which `VQAdamW.step` uses to update, refit and re-encode all three states
with one device round trip per phase instead of seven.
"""
from __future__ import annotations

import ctypes
import math
import operator
import struct
from contextlib import ExitStack
from dataclasses import dataclass

import numpy as np

from . import ack

SCHEMA = 1
GROUPS = (8, 16, 32)
ENTRIES = 16
MAX_ELEMENTS = 1 << 28          # values of one coded tensor (the reference's bound)
MAX_MATMUL_MACS = 1 << 28       # multiply-adds of one schema-1 product

# schema-2 operations of ack_vq2 (include/alelyon_compute_kit.h)
OP_DENSE, OP_CODED, OP_ADAMW_SAMPLE, OP_ADAMW_USAGE, OP_ADAMW_ENCODE, OP_ENCODE, OP_DECODE, OP_REPACK, OP_FIT, \
    OP_FIT_VALUES = range(16, 26)
DENSE_TC_MIN_ROWS = 40   # rows of X from which the dense product runs on the tensor cores


# ------------------------------------------------------------ argument checks ----

def _integer(value, name: str, minimum: int, maximum: int) -> int:
    """An integral value (bools refused) within [minimum, maximum]."""
    if isinstance(value, (bool, np.bool_)):
        raise ValueError(f"{name} must be an integer")
    try:
        number = operator.index(value)
    except TypeError as exc:
        raise ValueError(f"{name} must be an integer") from exc
    if number < minimum or number > maximum:
        raise ValueError(f"{name} must be in {minimum}..{maximum}")
    return number


def _shape(shape) -> tuple[int, ...]:
    dims = tuple(_integer(d, "dimension", 1, MAX_ELEMENTS) for d in shape)
    if len(dims) < 1 or len(dims) > 6 or math.prod(dims) > MAX_ELEMENTS:
        raise ValueError("vq shape requires rank 1..6 and a bounded element count")
    return dims


def _group(group) -> int:
    g = _integer(group, "group", 8, 32)
    if g not in GROUPS:
        raise ValueError("vq group must be 8, 16 or 32")
    return g


def _float_array(value, name: str) -> np.ndarray:
    a = np.asarray(value)
    if a.dtype != np.float32 or not np.isfinite(a).all():
        raise ValueError(f"{name} must contain finite float32 values")
    return np.ascontiguousarray(a)


def _book(value, group: int) -> np.ndarray:
    book = _float_array(value, "codebook")
    if book.shape != (ENTRIES, group):
        raise ValueError(f"codebook must have shape (16, {group})")
    return book


# -------------------------------------------------------------- the format ----
#
# A coded tensor of n values in groups of g: V = ceil(n / g) vectors, one
# 4-bit entry index each; index v is nibble v % 8 (bits 4 (v % 8) ..) of the
# little-endian u32 word v // 8; the unused high nibbles of the last word are
# zero. Its wire image is a 40-byte header (<8sIIIIQQ: magic "ACKVQ4\0\0",
# schema 1, group, rank, reserved 0, n, code bytes), the rank dimensions as
# u64, the 16 x g FP32 codebook and the code words, all little-endian.

def storage_layout(shape, group: int = 16) -> dict:
    """Byte accounting of one coded tensor, padding and codebook included."""
    shape, group = _shape(shape), _group(group)
    n = math.prod(shape)
    vectors = -(-n // group)
    code_bytes = 4 * -(-vectors // 8)
    book_bytes = 4 * ENTRIES * group
    meta = _WireHeader.SIZE + 8 * len(shape)
    total = code_bytes + book_bytes + meta
    return {"elements": n, "vectors": vectors, "code_bytes": code_bytes, "codebook_bytes": book_bytes,
            "metadata_bytes": meta, "serialized_bytes": total, "payload_bytes": code_bytes + book_bytes,
            "bits_per_value": 8 * total / n, "sub_bit": 8 * total < n}


class _WireHeader:
    """The fixed header of a wire image."""

    LAYOUT = struct.Struct("<8sIIIIQQ")
    SIZE = LAYOUT.size
    MAGIC = b"ACKVQ4\0\0"

    @classmethod
    def pack(cls, shape: tuple, group: int, layout: dict) -> bytes:
        head = cls.LAYOUT.pack(cls.MAGIC, SCHEMA, group, len(shape), 0, layout["elements"], layout["code_bytes"])
        return head + struct.pack(f"<{len(shape)}Q", *shape)

    @classmethod
    def unpack(cls, view: memoryview) -> tuple[tuple, int, dict, int]:
        """(shape, group, layout, offset of the codebook) of a whole image."""
        magic, schema, group, rank, reserved, n, code_bytes = cls.LAYOUT.unpack_from(view)
        if magic != cls.MAGIC or schema != SCHEMA or reserved or rank < 1 or rank > 6:
            raise ValueError("unsupported vq artifact header")
        start = cls.SIZE + 8 * rank
        if view.nbytes < start:
            raise ValueError("truncated vq dimensions")
        shape = struct.unpack_from(f"<{rank}Q", view, cls.SIZE)
        layout = storage_layout(shape, group)
        if n != layout["elements"] or code_bytes != layout["code_bytes"]:
            raise ValueError("vq header disagrees with its dimensions")
        if view.nbytes != layout["serialized_bytes"]:
            raise ValueError("vq artifact length mismatch")
        return shape, group, layout, start


def _pack(indices: np.ndarray) -> np.ndarray:
    """Entry indices -> u32 code words (eight nibbles per word, vector v in
    nibble v % 8 of word v // 8; the last word zero-padded)."""
    idx = np.zeros(-(-indices.size // 8) * 8, dtype=np.uint32)
    idx[:indices.size] = indices
    shifts = np.arange(0, 32, 4, dtype=np.uint32)
    return np.bitwise_or.reduce(idx.reshape(-1, 8) << shifts, axis=1).astype(np.uint32)


def _indices(codes: np.ndarray, vectors: int) -> np.ndarray:
    """The first `vectors` entry indices of a code-word image."""
    shifts = np.arange(0, 32, 4, dtype=np.uint32)
    return ((np.asarray(codes, np.uint32)[:, None] >> shifts) & np.uint32(15)).reshape(-1)[:vectors]


@dataclass(frozen=True, init=False)
class VQArray:
    """An owned, read-only coded tensor on the host: shape, group, the code
    words and the codebook (the reference's `VQArray`)."""

    shape: tuple[int, ...]
    group: int
    codes: np.ndarray
    codebook: np.ndarray

    def __init__(self, shape, group, codes, codebook):
        shape, group = _shape(shape), _group(group)
        layout = storage_layout(shape, group)
        words = np.asarray(codes)
        if words.dtype != np.uint32 or words.shape != (layout["code_bytes"] // 4,):
            raise ValueError("vq codes must be the exact uint32 word image")
        used = layout["vectors"] % 8
        if used and int(words[-1]) >> (4 * used):
            raise ValueError("vq unused codeword bits must be zero")
        book = _book(codebook, group)
        frozen = []
        for a in (words, book):
            a = a.copy()
            a.flags.writeable = False
            frozen.append(a)
        for name, value in (("shape", shape), ("group", group), ("codes", frozen[0]), ("codebook", frozen[1])):
            object.__setattr__(self, name, value)

    @property
    def layout(self) -> dict:
        return storage_layout(self.shape, self.group)

    def decode(self) -> np.ndarray:
        lay = self.layout
        values = self.codebook[_indices(self.codes, lay["vectors"])].reshape(-1)
        return values[:lay["elements"]].reshape(self.shape).copy()

    def to_bytes(self) -> bytes:
        return (_WireHeader.pack(self.shape, self.group, self.layout) + self.codebook.astype("<f4").tobytes()
                + self.codes.astype("<u4").tobytes())

    @classmethod
    def from_bytes(cls, data, *, max_bytes: int = 128 * 1024 * 1024) -> "VQArray":
        limit = _integer(max_bytes, "max_bytes", _WireHeader.SIZE, 1 << 32)
        view = memoryview(data).cast("B")
        if view.nbytes < _WireHeader.SIZE or view.nbytes > limit:
            raise ValueError("vq artifact byte limit or truncated header")
        shape, group, layout, at = _WireHeader.unpack(view)
        book_end = at + layout["codebook_bytes"]
        book = np.frombuffer(view[at:book_end], dtype="<f4").astype(np.float32).reshape(ENTRIES, group)
        codes = np.frombuffer(view[book_end:], dtype="<u4").astype(np.uint32)
        return cls(shape, group, codes, book)


def _nearest(vectors: np.ndarray, book: np.ndarray, valid_last: int | None = None) -> np.ndarray:
    """float64 nearest entry per row, components summed in order, lowest
    index on ties; `valid_last` limits the last row to its valid components."""
    group = book.shape[1]
    b = book.astype(np.float64)
    chosen = np.empty(len(vectors), dtype=np.uint32)
    step = 16384
    for start in range(0, len(vectors), step):
        v = vectors[start:start + step].astype(np.float64)
        distances = np.zeros((len(v), ENTRIES), dtype=np.float64)
        last = start + len(v) == len(vectors)
        for j in range(group):
            delta = v[:, j, None] - b[None, :, j]
            if last and valid_last is not None and j >= valid_last:
                delta[-1] = 0
            distances += delta * delta
        chosen[start:start + len(v)] = np.argmin(distances, axis=1).astype(np.uint32)
    return chosen


def encode(values, codebook, *, group: int = 16) -> VQArray:
    """CPU encoder: nearest code vector in float64, lowest index on ties.

    The reference's CPU encoder (its results define the device encoder's:
    `VQDevice.encode` returns the same bytes). `fit_codebook` uses it on its
    calibration sample; device-sized work belongs on `VQDevice`."""
    group = _group(group)
    x = _float_array(values, "values")
    shape = _shape(x.shape)
    book = _book(codebook, group)
    layout = storage_layout(shape, group)
    padded = np.zeros(layout["vectors"] * group, dtype=np.float32)
    padded[:x.size] = x.reshape(-1)
    tail = x.size % group
    chosen = _nearest(padded.reshape(-1, group), book, tail if tail else None)
    return VQArray(shape, group, _pack(chosen), book)


def _reseed(sample: np.ndarray, book: np.ndarray) -> np.ndarray:
    """The sample vector the current book serves worst (farthest point)."""
    gap = ((sample.astype(np.float64)[:, None, :] - book.astype(np.float64)[None, :, :]) ** 2).sum(-1).min(1)
    return sample[int(gap.argmax())]


def _sample_positions(complete: int, sample_vectors: int) -> np.ndarray:
    return np.linspace(0, complete - 1, min(complete, sample_vectors), dtype=np.int64)


def _fit(sample: np.ndarray, complete: int, group: int, iterations: int, init, whole_usage) -> np.ndarray:
    """Lloyd iterations on the calibration sample. `whole_usage(book)` returns
    the entries the whole tensor selects; it is asked only on a warm start
    whose sample is smaller than the tensor and leaves empty an entry no lower
    row duplicates (the kept-entry rule of the reference fit)."""
    if init is None:
        book = sample[np.linspace(0, len(sample) - 1, ENTRIES, dtype=np.int64)].copy()
    else:
        book = _book(init, group).copy()
    for _ in range(iterations):
        _book(book, group)
        idx = _nearest(sample, book)
        kept = set()
        empty = set(range(ENTRIES)) - set(np.unique(idx).tolist())
        reachable = [e for e in empty if not any(np.array_equal(book[e], book[j]) for j in range(e))]
        if init is not None and len(sample) < complete and reachable:
            kept = set(whole_usage(book))
        for entry in range(ENTRIES):
            selected = sample[idx == entry]
            if len(selected):
                book[entry] = selected.mean(axis=0, dtype=np.float64).astype(np.float32)
            elif entry not in kept:
                book[entry] = _reseed(sample, book)
    return book


def fit_codebook(values, *, group: int = 16, iterations: int = 4,
                 sample_vectors: int = 4096, init=None) -> np.ndarray:
    """Bounded deterministic calibration on the CPU; does not establish task quality.

    Lloyd iterations on a strided sample of at most `sample_vectors`
    complete vectors; an entry a iteration leaves empty is reseeded with the
    sample vector the book serves worst, unless (warm start from `init`, the
    sample smaller than the tensor) the whole tensor still selects it."""
    group = _group(group)
    iterations = _integer(iterations, "iterations", 0, 32)
    sample_vectors = _integer(sample_vectors, "sample_vectors", ENTRIES, 65536)
    x = _float_array(values, "values").reshape(-1)
    if x.size < group:
        raise ValueError("codebook calibration needs at least one complete vector")
    complete = x[:x.size // group * group].reshape(-1, group)
    sample = complete[_sample_positions(len(complete), sample_vectors)]

    def whole_usage(book):
        return np.unique(_nearest(complete, book)).tolist()

    return _fit(sample, len(complete), group, iterations, init, whole_usage)


class ResidentStack:
    """A `VQStack` held in device memory (see `VQDevice.resident`): codes
    (canonical or tile32) and books uploaded once, plus per-M activation,
    output and status buffers reused across calls. `free()` (or leaving a
    `with` block) releases the device memory."""

    def __init__(self, backend: "VQDevice", stack: "VQStack", layout: str) -> None:
        if layout not in ("tile32", "canonical"):
            raise ValueError(f"unknown code layout {layout!r}")
        if len(stack.shape) != 2:
            raise ValueError("vq matmul requires matrices")
        n, k = stack.shape
        if layout == "tile32" and (k % stack.group or (k // stack.group) % 32):
            raise ValueError("the tile32 layout needs (K / group) % 32 == 0 for a stored N x K matrix")
        self.backend, self.shape, self.group, self.layout = backend, stack.shape, stack.group, layout
        self.count = len(stack)
        device = backend.device
        self._buffers = []
        with device._lock:
            device._require_open()
            canon = device.buffer(stack.codes.nbytes)
            self._buffers.append(canon)
            canon.upload(stack.codes)
            books = device.buffer(stack.books.nbytes)
            self._buffers.append(books)
            books.upload(stack.books)
            self.books = books
            if layout == "tile32":
                words = (n + 31) // 32 * 32 * (k // stack.group) // 8
                tiled = device.buffer(self.count * words * 4)
                self._buffers.append(tiled)
                status = self._status()
                plan = backend._plan2(OP_REPACK, n, 1, k, stack.group, batch=self.count)
                backend._launch2(plan, [canon, None, None, None, None, tiled, None, status])
                self._check(status)
                canon.free()
                self._buffers.remove(canon)
                self.codes = tiled
            else:
                self.codes = canon

    def __len__(self) -> int:
        return self.count

    def _status(self):
        status = self.backend.device.buffer(4)
        self._buffers.append(status)
        status.upload(np.zeros(1, dtype=np.uint32))
        return status

    @staticmethod
    def _check(status) -> None:
        flags = int(status.download(np.uint32)[0])
        if flags:
            names = [name for bit, name in ((1, "nonfinite"), (2, "layout"), (4, "optimizer"), (8, "stalled"))
                     if flags & bit]
            raise ack.AckError(f"vq device arithmetic refused: status={flags} ({', '.join(names) or 'unknown'})")

    def matmul(self, xs, *, transpose_b: bool = True, out: np.ndarray | None = None,
               parts: int = 0) -> np.ndarray:
        """Y = X . op(decode W) for every resident matrix, X and Y in host
        memory. One pipelined library call (`ack_vq2_dense_host`): the
        experts run in `parts` ranges (0: the library's choice) whose copies
        in, products and copies out overlap; page-locked `xs` and `out`
        (e.g. from a pinned allocator) let the copies run asynchronously.
        With 64 or more rows of X on canonical codes the product runs on the
        tensor cores."""
        if self.layout == "tile32" and not transpose_b:
            raise ValueError("the tile32 layout holds W stored N x K (transpose_b=True)")
        backend, device = self.backend, self.backend.device
        # finiteness is checked on the device (the kernels flag nonfinite
        # products in the status word), not by a host pass over X
        x = np.asarray(xs)
        if x.dtype != np.float32:
            raise ValueError("activations must contain finite float32 values")
        x = np.ascontiguousarray(x)
        if x.ndim != 3 or x.shape[0] != self.count:
            raise ValueError("activations must be (count, M, K) with one matrix per coded weight")
        e, m, k = x.shape
        n, k2 = self.shape if transpose_b else self.shape[::-1]
        if k != k2:
            raise ValueError("vq matmul dimensions are incompatible or exceed bounds")
        flags = (2 if transpose_b else 0) | (4 if self.layout == "tile32" else 0)
        if (self.layout == "canonical" and transpose_b and m >= DENSE_TC_MIN_ROWS and k % self.group == 0
                and (k // self.group) % 32 == 0):
            flags |= 8
        y = np.empty((e, m, n), dtype=np.float32) if out is None else out
        if y.dtype != np.float32 or y.shape != (e, m, n) or not y.flags.c_contiguous:
            raise ValueError("out must be a C-contiguous (count, M, N) float32 array")
        plan = struct.pack("<16I", *backend._plan2(OP_DENSE, m, n, k, self.group, flags=flags, batch=e))
        status = ctypes.c_uint32(0)
        with device._lock:
            device._require_open()
            if not self.codes._handle:
                raise ack.AckError("resident stack has been freed")
            fn = device._lib.cdll.ack_vq2_dense_host
            fn.restype = ctypes.c_int32
            fn.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p,
                           ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32)]
            rc = fn(device._handle, plan, len(plan), self.codes._handle, self.books._handle, x.ctypes.data,
                    y.ctypes.data, int(parts), ctypes.byref(status))
            if rc != ack.ACK_OK:
                raise ack._kit_error("vq2", rc, device._lib.last_error())
        if status.value == 1:
            raise ValueError("activations must contain finite float32 values (or the products overflowed): "
                             "device status=1")
        if status.value:
            raise ack.AckError(f"vq device arithmetic refused: status={status.value}")
        return y

    def free(self) -> None:
        for b in self._buffers:
            b.free()
        self._buffers = []

    def __enter__(self) -> "ResidentStack":
        return self

    def __exit__(self, *exc) -> None:
        self.free()


@dataclass(frozen=True, init=False)
class VQStack:
    """E coded matrices of one shape and group, stored contiguously: codes
    (E, words) and books (E, 16, group). The operand of the grouped product;
    build it once for weights that are used many times."""

    shape: tuple[int, ...]
    group: int
    codes: np.ndarray
    books: np.ndarray

    def __init__(self, shape, group, codes, books):
        shape, group = _shape(shape), _group(group)
        layout = storage_layout(shape, group)
        codes = np.asarray(codes)
        books = np.asarray(books)
        if codes.dtype != np.uint32 or codes.ndim != 2 or codes.shape[1] != layout["code_bytes"] // 4:
            raise ValueError("stacked codes must be a (count, words) uint32 array")
        if books.dtype != np.float32 or books.shape != (codes.shape[0], ENTRIES, group):
            raise ValueError(f"stacked books must be a (count, 16, {group}) float32 array")
        if not codes.flags.c_contiguous or not books.flags.c_contiguous:
            raise ValueError("stacked codes and books must be C-contiguous")
        object.__setattr__(self, "shape", shape)
        object.__setattr__(self, "group", group)
        object.__setattr__(self, "codes", codes)
        object.__setattr__(self, "books", books)

    @classmethod
    def from_arrays(cls, arrays) -> "VQStack":
        arrays = list(arrays)
        if not arrays or any(a.shape != arrays[0].shape or a.group != arrays[0].group for a in arrays):
            raise ValueError("a stack needs one or more VQArrays of one shape and group")
        return cls(arrays[0].shape, arrays[0].group, np.stack([a.codes for a in arrays]),
                   np.stack([a.codebook for a in arrays]))

    def __len__(self) -> int:
        return self.codes.shape[0]

    def __getitem__(self, i) -> VQArray:
        return VQArray(self.shape, self.group, self.codes[i], self.books[i])


class VQDevice:
    """Synchronous, status-checked vq4 operations on an open `ack.Device`.

    Each call allocates its device buffers, uploads its inputs, enqueues the
    kernel, reads the status word and then the output, and frees the buffers
    -- the reference's `VQDevice._run` contract (vq.py:283-308)."""

    def __init__(self, device: ack.Device):
        self.device = device
        with device._lock:
            device._require_open()
            lib = device._lib.cdll
            try:
                schema = lib.ack_vq_schema
                self._call = lib.ack_vq
                self._call2 = lib.ack_vq2
            except AttributeError as exc:
                raise ack.AckUnavailable("library lacks the optional vq4/v1 extension") from exc
            if schema() != SCHEMA:
                raise ack.AckUnavailable("incompatible vq4 extension schema")

    # -- transport ------------------------------------------------------------------

    @staticmethod
    def _refuse_status(status) -> None:
        """Raise if the kernel set a status bit (vq4.comp:5-8): the output
        must not be used."""
        flags = int(status.download(np.uint32)[0])
        if flags:
            names = [name for bit, name in ((1, "nonfinite"), (2, "layout"), (4, "optimizer"), (8, "stalled"))
                     if flags & bit]
            raise ack.AckError(f"vq device arithmetic refused: status={flags} ({', '.join(names) or 'unknown'})")

    def _run(self, words, inputs, output_bytes: int, dtype):
        """One schema-1 `ack_vq` call on fresh device buffers: the inputs
        staged (an unread input slot names the first input again: the ABI
        wants every slot live), the output and a cleared status word
        allocated, the status checked, the output downloaded."""
        dev = self.device
        with dev._lock, ExitStack() as owned:
            dev._require_open()

            def fresh(nbytes: int, content=None):
                b = dev.buffer(nbytes)
                owned.callback(b.free)
                if content is not None:
                    b.upload(content)
                return b

            slots = [fresh(a.nbytes, a) for a in inputs]
            slots += [slots[0]] * (4 - len(slots))
            out = fresh(output_bytes)
            status = fresh(4, np.zeros(1, dtype=np.uint32))
            plan = struct.pack("<8I", *words)
            rc = self._call(dev._handle, *(b._handle for b in slots), out._handle, status._handle, plan, len(plan))
            if rc != ack.ACK_OK:
                raise ack._kit_error("vq", rc, dev._lib.last_error())
            self._refuse_status(status)
            return out.download(dtype)

    def _launch2(self, plan_words, slots) -> None:
        """Enqueue one schema-2 operation on live buffers (slot order
        in0..in4, out0, out1, status; None for an unused slot)."""
        device = self.device
        plan = struct.pack("<16I", *plan_words)
        handles = (ctypes.c_void_p * 8)(*[(b._handle if b is not None else None) for b in slots])
        rc = self._call2(device._handle, handles, 8, plan, len(plan))
        if rc != ack.ACK_OK:
            raise ack._kit_error("vq2", rc, device._lib.last_error())

    @staticmethod
    def _plan2(op, m, n, k, group, flags=0, batch=1, aux0=0, aux1=0, aux2=0):
        return (op, m, n, k, group, ENTRIES, flags, 0, batch, aux0, aux1, aux2, 0, 0, 0, 0)

    def _run2(self, plan_words, inputs, outputs):
        """Upload `inputs` (up to five arrays; None skips a slot), run, check
        status, download `outputs` [(nbytes, dtype), ...] (up to two)."""
        device = self.device
        with device._lock, ExitStack() as cleanup:
            device._require_open()
            slots = [None] * 8
            for i, array in enumerate(inputs):
                if array is None:
                    continue
                b = device.buffer(array.nbytes)
                cleanup.callback(b.free)
                b.upload(array)
                slots[i] = b
            outs = []
            for i, (nbytes, _) in enumerate(outputs):
                b = device.buffer(nbytes)
                cleanup.callback(b.free)
                slots[5 + i] = b
                outs.append(b)
            status = device.buffer(4)
            cleanup.callback(status.free)
            status.upload(np.zeros(1, dtype=np.uint32))
            slots[7] = status
            self._launch2(plan_words, slots)
            self._refuse_status(status)
            return tuple(b.download(dtype) for b, (_, dtype) in zip(outs, outputs))

    # -- the reference's operations (schema 1) ----------------------------------
    #
    # Each is one `ack_vq` call with the reference's 8-word plan [op, m, n, k,
    # group, 16, flags, 0] and bounds (2^28 values, 2^28 multiply-adds).

    def _op1(self, op: int, m: int, n: int, k: int, group: int, flags: int, inputs, out_bytes: int, dtype):
        return self._run((op, m, n, k, group, ENTRIES, flags, 0), inputs, out_bytes, dtype)

    def encode(self, values, codebook, *, group: int = 16) -> VQArray:
        group = _group(group)
        x = _float_array(values, "values")
        book = _book(codebook, group)
        words = self._op1(0, x.size, 1, 1, group, 0, (x, book), storage_layout(x.shape, group)["code_bytes"],
                          np.uint32)
        return VQArray(x.shape, group, words, book)

    def decode(self, value: VQArray) -> np.ndarray:
        n = value.layout["elements"]
        out = self._op1(1, n, 1, 1, value.group, 0, (value.codes, value.codebook), 4 * n, np.float32)
        return out.reshape(value.shape)

    @staticmethod
    def _product_geometry(a: VQArray, b: VQArray, transpose_a, transpose_b) -> tuple[int, int, int, int]:
        """(m, n, k, flags) of op(a) @ op(b), refused as the reference refuses."""
        if type(transpose_a) is not bool or type(transpose_b) is not bool:
            raise ValueError("transpose flags must be boolean")
        if len(a.shape) != 2 or len(b.shape) != 2 or a.group != b.group:
            raise ValueError("vq matmul requires two matrices using the same vector group")
        (m, k) = (a.shape[1], a.shape[0]) if transpose_a else a.shape
        (k_b, n) = (b.shape[1], b.shape[0]) if transpose_b else b.shape
        return m, n, k if k == k_b else -1, int(transpose_a) | (int(transpose_b) << 1)

    def matmul(self, a: VQArray, b: VQArray, *, transpose_a=False, transpose_b=False) -> np.ndarray:
        m, n, k, flags = self._product_geometry(a, b, transpose_a, transpose_b)
        if k < 0 or max(m, n, k) > 65536 or m * n > MAX_ELEMENTS:
            raise ValueError("vq matmul dimensions are incompatible or exceed bounds")
        if m * n * k > MAX_MATMUL_MACS:
            raise ValueError("vq-matmul-work-limit: split the product into bounded calls")
        out = self._op1(2, m, n, k, a.group, flags, (a.codes, a.codebook, b.codes, b.codebook), 4 * m * n,
                        np.float32)
        return out.reshape(m, n)

    def adamw(self, weight: VQArray, momentum: VQArray, variance: VQArray,
              gradient: VQArray, *, lr: float, beta1: float, beta2: float,
              eps: float, weight_decay: float, step: int) -> tuple[np.ndarray, ...]:
        """vq4.comp op 3: W', M', V' as FP32 arrays from the four coded states."""
        states = (weight, momentum, variance, gradient)
        coefficients = _adamw_coefficients(states, lr, beta1, beta2, eps, weight_decay, step)
        n = weight.layout["elements"]
        if 3 * n > MAX_ELEMENTS:
            raise ValueError("vq AdamW active scratch exceeds element bound")
        inputs = (np.concatenate([s.codes for s in states]),
                  np.concatenate([s.codebook.reshape(-1) for s in states]), coefficients)
        out = self._op1(3, n, 1, 1, weight.group, 0, inputs, 12 * n, np.float32)
        return tuple(part.reshape(weight.shape) for part in out.reshape(3, n))

    # -- B200 extension operations (schema 2) ----------------------------------

    def encode_large(self, values, codebook, *, group: int = 16) -> np.ndarray:
        """Packed code words of a 1-D float32 array of any length (beyond the
        2^28-value bound of `encode`); returns the uint32 word image."""
        group = _group(group)
        x = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        if not x.size:
            raise ValueError("nothing to encode")
        book = _book(codebook, group)
        words = ((x.size + group - 1) // group + 7) // 8
        plan = self._plan2(OP_ENCODE, x.size & 0xFFFFFFFF, 1, 1, group, aux0=x.size >> 32)
        (codes,) = self._run2(plan, (x, book), [(words * 4, np.uint32)])
        return codes

    def decode_large(self, codes, codebook, count: int, *, group: int = 16) -> np.ndarray:
        group = _group(group)
        count = _integer(count, "count", 1, 1 << 36)
        book = _book(codebook, group)
        words = ((count + group - 1) // group + 7) // 8
        codes = np.ascontiguousarray(codes, dtype=np.uint32).reshape(-1)
        if codes.size != words:
            raise ValueError("code image does not match the value count")
        plan = self._plan2(OP_DECODE, count & 0xFFFFFFFF, 1, 1, group, aux0=count >> 32)
        (out,) = self._run2(plan, (codes, book), [(count * 4, np.float32)])
        return out

    def matmul_dense(self, x, w: VQArray, *, transpose_b: bool = True) -> np.ndarray:
        """FP32 activations times coded weights.

        `transpose_b=True`: `w` is stored (N, K) with its vectors along K and
        the result is `x @ decode(w).T`; `False`: `w` is stored (K, N) and the
        result is `x @ decode(w)`. `x` is (M, K) float32."""
        return self.matmul_dense_grouped(np.asarray(x)[None], VQStack.from_arrays([w]),
                                         transpose_b=transpose_b)[0]

    def fit_codebook(self, values, *, group: int = 16, iterations: int = 4, sample_vectors: int = 4096,
                     init=None) -> np.ndarray:
        """`fit_codebook` computed on the device: the same arguments, the
        same refusals and bit for bit the same book as the CPU function (the
        sample's nearest entries by the certified search, float64 means in
        sample order, the farthest-point reseed, the warm start's kept-entry
        rule over the whole tensor)."""
        group = _group(group)
        iterations = _integer(iterations, "iterations", 0, 32)
        sample_vectors = _integer(sample_vectors, "sample_vectors", ENTRIES, 65536)
        x = _float_array(values, "values").reshape(-1)
        if x.size < group:
            raise ValueError("codebook calibration needs at least one complete vector")
        complete = x.size // group
        positions = _sample_positions(complete, sample_vectors)
        s = len(positions)
        rows = np.linspace(0, s - 1, ENTRIES, dtype=np.int64)
        index = np.concatenate([positions, rows]).astype(np.uint32)
        book = None if init is None else _book(init, group)
        flags = 0 if book is None else 1
        plan = self._plan2(OP_FIT_VALUES, x.size & 0xFFFFFFFF, 1, 1, group, flags=flags, aux0=s, aux1=iterations,
                           aux2=x.size >> 32)
        device = self.device
        with device._lock, ExitStack() as cleanup:
            device._require_open()

            def buffer_of(array):
                b = device.buffer(array.nbytes)
                cleanup.callback(b.free)
                b.upload(array)
                return b

            slots = [buffer_of(x), buffer_of(book) if book is not None else None, buffer_of(index), None]
            workspace = device.buffer(s * group * 4 + (s + 15) // 16 * 16 + 160)
            cleanup.callback(workspace.free)
            out = device.buffer(ENTRIES * group * 4)
            cleanup.callback(out.free)
            status = buffer_of(np.zeros(1, dtype=np.uint32))
            self._launch2(plan, slots + [workspace, out, None, status])
            flags = int(status.download(np.uint32)[0])
            if flags:
                raise ack.AckError(f"vq device arithmetic refused: status={flags}")
            return out.download(np.float32).reshape(ENTRIES, group)

    def resident(self, stack: "VQStack", *, layout: str = "tile32") -> "ResidentStack":
        """Upload a `VQStack` once and keep it on the device: the weights of
        a grouped product that runs many times (serving, a training step).
        `layout="tile32"` (matrices stored N x K with (K / group) % 32 == 0)
        repacks the codes on the device into the layout whose rows a warp
        reads as coalesced lines; "canonical" keeps the wire layout. For
        single-row products (M = 1) with K a multiple of 256 * group the
        canonical layout is the faster one: it feeds the byte-pair table
        kernel (one lookup per code byte); tile32 is faster for M >= 2."""
        return ResidentStack(self, stack, layout)

    def matmul_dense_grouped(self, xs, ws, *, transpose_b: bool = True, out: np.ndarray | None = None,
                             parts: int = 0) -> np.ndarray:
        """E independent products in one launch: `xs` is (E, M, K) float32
        (or a sequence of (M, K)), `ws` a `VQStack` (or a sequence of
        VQArray) of E matrices of one shape and group, or a `ResidentStack`
        (then only X and Y cross the bus, into `out` when given: a
        contiguous (E, M, N) float32 array, ideally in pinned memory; the
        copies and products overlap over `parts` ranges of the experts).
        Returns (E, M, N)."""
        if type(transpose_b) is not bool:
            raise ValueError("transpose flags must be boolean")
        if isinstance(ws, ResidentStack):
            return ws.matmul(xs, transpose_b=transpose_b, out=out, parts=parts)
        stack = ws if isinstance(ws, VQStack) else VQStack.from_arrays(ws)
        if len(stack.shape) != 2:
            raise ValueError("vq matmul requires matrices")
        x = np.asarray(xs) if not isinstance(xs, (list, tuple)) else np.stack([np.asarray(v) for v in xs])
        x = _float_array(x, "activations")
        if x.ndim != 3 or x.shape[0] != len(stack):
            raise ValueError("activations must be (count, M, K) with one matrix per coded weight")
        e, m, k = x.shape
        n, k2 = stack.shape if transpose_b else stack.shape[::-1]
        if k != k2:
            raise ValueError("vq matmul dimensions are incompatible or exceed bounds")
        plan = self._plan2(OP_DENSE, m, n, k, stack.group, flags=2 if transpose_b else 0, batch=e)
        (y,) = self._run2(plan, (x, stack.codes, stack.books), [(e * m * n * 4, np.float32)])
        return y.reshape(e, m, n)

    def matmul_coded(self, a: VQArray, b: VQArray, *, transpose_a=False, transpose_b=False) -> np.ndarray:
        """`op(decode a) @ op(decode b)` without the 2^28-MAC bound of `matmul`.

        With `a` stored (M, K) and `b` stored (N, K) (`transpose_b=True`) and
        K a multiple of the group, each group's dot product is a lookup in the
        16x16 table of codebook inner products."""
        m, n, k, flags = self._product_geometry(a, b, transpose_a, transpose_b)
        if k < 0:
            raise ValueError("vq matmul dimensions are incompatible or exceed bounds")
        plan = self._plan2(OP_CODED, m, n, k, a.group, flags=flags)
        (y,) = self._run2(plan, (a.codes, a.codebook, b.codes, b.codebook), [(m * n * 4, np.float32)])
        return y.reshape(m, n)

    def adamw_fused(self, weight: VQArray, momentum: VQArray, variance: VQArray, gradient: VQArray, *,
                    lr: float, beta1: float, beta2: float, eps: float, weight_decay: float, step: int,
                    sample_vectors: int = 4096, iterations: int = 4, fit: str = "host"):
        """One VQAdamW step without FP32 scratch: the device computes the
        AdamW values of the calibration sample (the same values op 3 would
        produce), `fit_codebook`'s Lloyd iterations run on the CPU with the
        whole-tensor entry check answered by the device (fit="host"), or on
        the device, bit for bit the same books (fit="device"), then one device
        pass decodes, updates and re-encodes W, M and V with the fitted books.

        Returns ((W', M', V') as VQArrays, changed weight values, bytes the
        device produced)."""
        if fit not in ("host", "device"):
            raise ValueError(f"fit must be 'host' or 'device', not {fit!r}")
        states = (weight, momentum, variance, gradient)
        coefficients = _adamw_coefficients(states, lr, beta1, beta2, eps, weight_decay, step)
        group = weight.group
        count = weight.layout["elements"]
        complete = count // group
        if complete < 1:
            raise ValueError("codebook calibration needs at least one complete vector")
        positions = _sample_positions(complete, sample_vectors)
        s = len(positions)
        codes = np.concatenate([st.codes for st in states])
        books = np.concatenate([st.codebook.reshape(-1) for st in states])
        words = weight.codes.size
        device = self.device
        with device._lock, ExitStack() as cleanup:
            device._require_open()

            def buffer_of(array):
                b = device.buffer(array.nbytes)
                cleanup.callback(b.free)
                b.upload(array)
                return b

            b_codes, b_books, b_coefs = buffer_of(codes), buffer_of(books), buffer_of(coefficients)
            b_pos = buffer_of(positions.astype(np.uint32))
            status = buffer_of(np.zeros(1, dtype=np.uint32))

            def check():
                flags = int(status.download(np.uint32)[0])
                if flags:
                    raise ack.AckError(f"vq device arithmetic refused: status={flags}")

            sample_out = device.buffer(3 * s * group * 4)
            cleanup.callback(sample_out.free)
            self._launch2(self._plan2(OP_ADAMW_SAMPLE, count, 1, 1, group, batch=1, aux0=s),
                          [b_codes, b_books, b_coefs, b_pos, None, sample_out, None, status])
            if fit == "device":
                stride = ((s + 15) // 16 * 16 + 160)
                workspace = device.buffer(3 * stride)
                cleanup.callback(workspace.free)
                b_new = device.buffer(3 * ENTRIES * group * 4)
                cleanup.callback(b_new.free)
                self._launch2(self._plan2(OP_FIT, count, 1, 1, group, flags=1, batch=1, aux0=s, aux1=iterations),
                              [b_codes, b_books, b_coefs, sample_out, workspace, b_new, None, status])
                check()
                new_books = b_new.download(np.float32).reshape(3, ENTRIES, group)
                produced = new_books.nbytes
                return self._adamw_encode(weight, count, group, words, b_codes, b_books, b_coefs, b_new, new_books,
                                          status, check, cleanup, produced)
            check()
            samples = sample_out.download(np.float32).reshape(3, s, group)

            trial = device.buffer(ENTRIES * group * 4)
            cleanup.callback(trial.free)
            usage_out = device.buffer(ENTRIES * 4)
            cleanup.callback(usage_out.free)
            fitted = []
            for which, state in enumerate((weight, momentum, variance)):
                def whole_usage(book, which=which):
                    trial.upload(np.ascontiguousarray(book, dtype=np.float32))
                    self._launch2(self._plan2(OP_ADAMW_USAGE, count, 1, 1, group, batch=1, aux0=which, aux1=0),
                                  [b_codes, b_books, b_coefs, trial, None, usage_out, None, status])
                    check()
                    return np.nonzero(usage_out.download(np.uint32))[0].tolist()

                fitted.append(_fit(samples[which], complete, group, iterations, state.codebook, whole_usage))
            new_books = np.ascontiguousarray(np.stack(fitted), dtype=np.float32)
            b_new = buffer_of(new_books)
            return self._adamw_encode(weight, count, group, words, b_codes, b_books, b_coefs, b_new, new_books,
                                      status, check, cleanup, samples.nbytes)

    def _adamw_encode(self, weight, count, group, words, b_codes, b_books, b_coefs, b_new, new_books, status, check,
                      cleanup, produced):
        """The fused step's last pass: decode, update and re-encode W, M, V
        with the fitted books `b_new` (device) / `new_books` (host copy)."""
        device = self.device
        out_codes = device.buffer(3 * words * 4)
        cleanup.callback(out_codes.free)
        changed = device.buffer(4)
        cleanup.callback(changed.free)
        self._launch2(self._plan2(OP_ADAMW_ENCODE, count, 1, 1, group, batch=1),
                      [b_codes, b_books, b_coefs, b_new, None, out_codes, changed, status])
        check()
        image = out_codes.download(np.uint32).reshape(3, words)
        n_changed = int(changed.download(np.uint32)[0])
        encoded = tuple(VQArray(weight.shape, group, image[i], new_books[i]) for i in range(3))
        return encoded, n_changed, produced + image.nbytes


def _adamw_coefficients(states, lr, beta1, beta2, eps, weight_decay, step) -> np.ndarray:
    """The reference's argument checks and its seven FP32 coefficients (vq.py:345-360)."""
    weight = states[0]
    if any(s.shape != weight.shape or s.group != weight.group for s in states):
        raise ValueError("vq AdamW states must have identical shapes and groups")
    step = _integer(step, "step", 1, 1 << 53)
    values = (lr, beta1, beta2, eps, weight_decay)
    if any(isinstance(x, (bool, np.bool_)) or not math.isfinite(float(x)) for x in values):
        raise ValueError("vq AdamW coefficients must be finite numbers")
    if lr < 0 or not 0 <= beta1 < 1 or not 0 <= beta2 < 1 or eps <= 0 or weight_decay < 0:
        raise ValueError("vq AdamW coefficients outside their domains")
    coefficients = np.array([lr, beta1, beta2, eps, weight_decay,
                             1 - beta1 ** step, 1 - beta2 ** step], dtype=np.float32)
    if not np.isfinite(coefficients).all() or coefficients[3] <= 0 or (coefficients[5:] <= 0).any():
        raise ValueError("vq AdamW coefficients are not representable in float32")
    return coefficients


class VQAdamW:
    """Optimizer with coded persistent weights and both moments.

    The AdamW arithmetic is FP32 in the reference shader's order; codebooks
    are refitted on the CPU; re-encoding is lossy. A failed step leaves the
    three state images and the step counter unchanged."""

    def __init__(self, backend, weight: VQArray, *, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0,
                 fit: str = "host"):
        """`fit` chooses where a backend with the fused step (`adamw_fused`)
        refits the codebooks: "host" (the CPU, as the reference) or "device"
        (the same books bit for bit, computed on the GPU)."""
        if fit not in ("host", "device"):
            raise ValueError(f"fit must be 'host' or 'device', not {fit!r}")
        self.fit = fit
        self.backend = backend
        self.weight = weight
        zeros = np.zeros_like(weight.codes)
        zero_book = np.zeros((ENTRIES, weight.group), dtype=np.float32)
        self.momentum = VQArray(weight.shape, weight.group, zeros, zero_book)
        self.variance = VQArray(weight.shape, weight.group, zeros, zero_book)
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        self.steps = 0

    def step(self, gradient: VQArray) -> dict:
        next_step = self.steps + 1
        fused = getattr(self.backend, "adamw_fused", None)
        if fused is not None:
            encoded, changed, produced = fused(
                self.weight, self.momentum, self.variance, gradient, lr=self.lr, beta1=self.betas[0],
                beta2=self.betas[1], eps=self.eps, weight_decay=self.weight_decay, step=next_step,
                **({"fit": self.fit} if self.fit != "host" else {}))
            encoded = list(encoded)
        else:
            scratch = self.backend.adamw(self.weight, self.momentum, self.variance, gradient,
                                         lr=self.lr, beta1=self.betas[0], beta2=self.betas[1],
                                         eps=self.eps, weight_decay=self.weight_decay, step=next_step)
            # each array warm-starts from its own state's codebook: the pairing must be exact
            if len(scratch) != 3:
                raise ValueError(f"vq AdamW update returned {len(scratch)} arrays, not 3")
            encoded = []
            for value, state in zip(scratch, (self.weight, self.momentum, self.variance)):
                book = fit_codebook(value, group=self.weight.group, init=state.codebook)
                encoded.append(self.backend.encode(value, book, group=self.weight.group))
            changed = int(np.count_nonzero(encoded[0].decode() != self.weight.decode()))
            produced = sum(s.nbytes for s in scratch)
        self.weight, self.momentum, self.variance = encoded
        self.steps = next_step
        return {"step": self.steps, "changed_weight_values": changed,
                "persistent_state_bytes": sum(s.layout["serialized_bytes"] for s in encoded),
                "gradient_bytes": gradient.layout["serialized_bytes"],
                "native_update_output_bytes": produced,
                "calibration": ("device float32/float64, bit for bit the CPU fit" if fused is not None and self.fit == "device"
                                else "CPU float32/float64 temporary arrays"),
                "model_quality_validated": False}
