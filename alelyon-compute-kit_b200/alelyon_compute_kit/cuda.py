"""vq4 operations on device-resident PyTorch tensors.

The same kernels, plans and admission as `VQDevice`, reached through the C
ABI's device-pointer entry `ack_vq_launch`: operands are CUDA tensors (code
words as int32 bit patterns), work is enqueued on the current PyTorch stream
of the tensors' device, nothing is copied to or from the host and nothing
synchronises unless asked (`check`). PyTorch supplies device memory,
streams and `torch.distributed`; the arithmetic is the library's.

Every function refuses, by raising, when the library is missing or a tensor
is not on a CUDA device: there is no CPU path here.
"""
from __future__ import annotations

import ctypes
import struct

import torch

from . import ack

ENTRIES = 16
OP_ENCODE1, OP_DECODE1, OP_MATMUL1, OP_ADAMW1 = 0, 1, 2, 3
(OP_DENSE, OP_CODED, OP_ADAMW_SAMPLE, OP_ADAMW_USAGE, OP_ADAMW_ENCODE, OP_ENCODE, OP_DECODE, OP_REPACK, OP_FIT,
 OP_FIT_VALUES, OP_RESIDUAL, OP_CLIP) = range(16, 28)
REDUCE_WORKSPACE_BYTES = (1024 + 1) * 8   # float64 partials of ops 26 and 27, then their total


def words_for(count: int, group: int) -> int:
    """u32 words of the packed image of `count` values."""
    return ((count + group - 1) // group + 7) // 8


def tile32_words(rows: int, cols: int, group: int) -> int:
    """u32 words of the tile32 layout of a coded rows x cols matrix."""
    return (rows + 31) // 32 * 32 * (cols // group) // 8


def plan1(op, m, n, k, group, flags=0) -> bytes:
    return struct.pack("<8I", op, m, n, k, group, ENTRIES, flags, 0)


def plan2(op, m, n, k, group, flags=0, batch=1, aux0=0, aux1=0, aux2=0) -> bytes:
    return struct.pack("<16I", op, m, n, k, group, ENTRIES, flags, 0, batch, aux0, aux1, aux2, 0, 0, 0, 0)


def _nbytes(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.numel() * t.element_size()


def launch(plan: bytes, slots, stream: torch.cuda.Stream | None = None) -> None:
    """Enqueue one plan. `slots` lists the operand tensors in the plan's slot
    order (6 for a 32-byte plan, 8 for a 64-byte plan); None = unused."""
    lib = ack._lib()
    ops = ack.AckVqOperands()
    ops.size = ctypes.sizeof(ops)
    ops.nslots = len(slots)
    device = None
    for i, t in enumerate(slots):
        if t is None:
            continue
        if not t.is_cuda:
            raise ack.AckError(f"vq operand {i} is not a CUDA tensor")
        if not t.is_contiguous():
            raise ack.AckError(f"vq operand {i} is not contiguous")
        device = device or t.device
        if t.device != device:
            raise ack.AckError("vq operands live on different devices")
        ops.ptr[i] = t.data_ptr()
        ops.bytes[i] = _nbytes(t)
    if device is None:
        raise ack.AckError("vq launch without operands")
    with torch.cuda.device(device):
        s = stream if stream is not None else torch.cuda.current_stream(device)
        rc = lib.cdll.ack_vq_launch(plan, len(plan), ctypes.byref(ops), ctypes.c_void_p(s.cuda_stream))
    if rc != ack.ACK_OK:
        raise ack._kit_error("vq", rc, lib.last_error())


def status_word(device) -> torch.Tensor:
    """A cleared status word (the caller clears it, vq4.comp:5-8)."""
    return torch.zeros(1, dtype=torch.int32, device=device)


STATUS_BITS = {1: "nonfinite", 2: "layout", 4: "optimizer", 8: "stalled"}


def check(status: torch.Tensor) -> None:
    """Synchronise on the status word and raise on any set bit (vq4.comp:5-8
    bits 1/2/4; bit 8: a pipelined kernel's bounded wait ran out)."""
    flags = int(status.item()) & 0xFFFFFFFF
    if flags:
        names = ", ".join(name for bit, name in STATUS_BITS.items() if flags & bit) or "unknown"
        raise ack.AckError(f"vq device arithmetic refused: status={flags} ({names})")


def decode(codes, book, count: int, group: int, *, out=None, status=None):
    """Dense float32 values of a packed image (64-bit count)."""
    out = torch.empty(count, dtype=torch.float32, device=codes.device) if out is None else out
    status = status_word(codes.device) if status is None else status
    launch(plan2(OP_DECODE, count & 0xFFFFFFFF, 1, 1, group, aux0=count >> 32),
           [codes, book, None, None, None, out, None, status])
    return out, status


def encode(x, book, group: int, *, out=None, status=None):
    """Packed image of a float32 tensor; the reference CPU encoder's bytes."""
    count = x.numel()
    out = torch.empty(words_for(count, group), dtype=torch.int32, device=x.device) if out is None else out
    status = status_word(x.device) if status is None else status
    launch(plan2(OP_ENCODE, count & 0xFFFFFFFF, 1, 1, group, aux0=count >> 32),
           [x, book, None, None, None, out, None, status])
    return out, status


def repack_tile32(codes, n: int, k: int, group: int, *, out=None, status=None):
    """The tile32 layout of E canonical n x k images (vectors along k,
    (k / group) % 32 == 0): `codes` (E, words) int32 -> (E, tile32 words).
    Static weights are repacked once; `dense(..., layout="tile32")` then reads
    each warp's 32 rows as coalesced 512-byte lines."""
    e = codes.shape[0]
    out = torch.empty((e, tile32_words(n, k, group)), dtype=torch.int32, device=codes.device) if out is None else out
    status = status_word(codes.device) if status is None else status
    launch(plan2(OP_REPACK, n, 1, k, group, batch=e), [codes, None, None, None, None, out, None, status])
    return out, status


# The dense product runs on the tensor cores from this many activation rows
# (canonical layout, W stored n x k, (k / group) % 32 == 0). The tensor-core
# kernel computes 64 rows of X per tile whatever M is, so its time is flat up
# to 64 rows; the shared-memory lookup-table kernels grow with M (cfg2
# measured: M=32 8.5 ms LUT against 8.9 ms; M=48 12.8 ms against 8.7 ms;
# M=64 16.9 ms against 9.0 ms).
DENSE_TC_MIN_ROWS = 40
DENSE_TC_MAX_ROWS = 128   # rows of X per pass of the tensor-core kernel


def dense_tc_workspace_bytes(m: int, k: int, group: int, batch: int) -> int:
    """Bytes of the tensor-core dense product's workspace: the projections of
    one pass of at most 128 rows of X on every codebook entry, as bf16 hi and
    lo rows, 128 rows per 64-row tile of X, 16 k / group values each, per
    expert."""
    rows = min(m, DENSE_TC_MAX_ROWS)
    return batch * ((rows + 63) // 64) * 128 * 16 * (k // group) * 2


def dense_engine(m: int, k: int, group: int, *, transpose_b: bool = True, layout: str = "canonical") -> str:
    """"tensor" when the tensor-core kernel applies and pays, else "lut"."""
    if (transpose_b and layout == "canonical" and m >= DENSE_TC_MIN_ROWS and k % group == 0
            and (k // group) % 32 == 0):
        return "tensor"
    return "lut"


def dense(x, codes, books, n: int, group: int, *, transpose_b: bool = True, layout: str = "canonical", out=None,
          status=None, engine: str = "auto", workspace=None):
    """Y[e] = X[e] @ decode(W[e]).T (W[e] stored n x k) for e < E, one launch.
    `x` (E, M, K) float32; `codes` (E, words) int32, canonical or (layout
    "tile32", from `repack_tile32`); `books` (E, 16, group).

    `engine`: "tensor" runs the tcgen05 kernel (one-hot codes times the
    entries' projections, needs the canonical layout, transpose_b and
    (k / group) % 32 == 0; its workspace, `dense_tc_workspace_bytes`, is
    allocated here unless given); "lut" the lookup-table kernels; "auto"
    picks by `dense_engine`."""
    e, m, k = x.shape
    out = torch.empty((e, m, n), dtype=torch.float32, device=x.device) if out is None else out
    status = status_word(x.device) if status is None else status
    flags = 2 if transpose_b else 0
    if layout == "tile32":
        if not transpose_b:
            raise ack.AckError("the tile32 layout holds W stored n x k (transpose_b=True)")
        flags |= 4
    elif layout != "canonical":
        raise ack.AckError(f"unknown code layout {layout!r}")
    if engine == "auto":
        engine = dense_engine(m, k, group, transpose_b=transpose_b, layout=layout)
    if engine == "tensor":
        flags |= 8
        if workspace is None:
            workspace = torch.empty(dense_tc_workspace_bytes(m, k, group, e), dtype=torch.uint8, device=x.device)
    elif engine != "lut":
        raise ack.AckError(f"unknown dense engine {engine!r}")
    else:
        workspace = None
    launch(plan2(OP_DENSE, m, n, k, group, flags=flags, batch=e), [x, codes, books, None, workspace, out, None, status])
    return out, status


def coded(a_codes, a_book, b_codes, b_book, m: int, n: int, k: int, group: int, *, flags: int = 2,
          out=None, status=None):
    """C = op(decode A) @ op(decode B); flags bit 0: A stored K x M, bit 1: B stored N x K."""
    out = torch.empty((m, n), dtype=torch.float32, device=a_codes.device) if out is None else out
    status = status_word(a_codes.device) if status is None else status
    launch(plan2(OP_CODED, m, n, k, group, flags=flags), [a_codes, a_book, b_codes, b_book, None, out, None, status])
    return out, status


def matmul_exact(a_codes, a_book, b_codes, b_book, m: int, n: int, k: int, group: int, *, flags: int = 0,
                 out=None, status=None):
    """The reference's bounded packed-pair product (schema-1 op 2)."""
    out = torch.empty((m, n), dtype=torch.float32, device=a_codes.device) if out is None else out
    status = status_word(a_codes.device) if status is None else status
    launch(plan1(OP_MATMUL1, m, n, k, group, flags), [a_codes, a_book, b_codes, b_book, out, status])
    return out, status


def adamw_sample(codes, books, coefs, positions, count: int, group: int, *, batch: int = 1, out=None, status=None):
    """AdamW values of the sample vectors `positions` for each expert: (E, 3, S, group)."""
    s = positions.numel()
    out = torch.empty((batch, 3, s, group), dtype=torch.float32, device=codes.device) if out is None else out
    status = status_word(codes.device) if status is None else status
    launch(plan2(OP_ADAMW_SAMPLE, count, 1, 1, group, batch=batch, aux0=s),
           [codes, books, coefs, positions, None, out, None, status])
    return out, status


def adamw_usage(codes, books, coefs, trial, count: int, group: int, state: int, expert: int = 0, *, batch: int = 1,
                out=None, status=None):
    """How many complete vectors of one updated state each entry of `trial` wins."""
    out = torch.empty(ENTRIES, dtype=torch.int32, device=codes.device) if out is None else out
    status = status_word(codes.device) if status is None else status
    launch(plan2(OP_ADAMW_USAGE, count, 1, 1, group, batch=batch, aux0=state, aux1=expert),
           [codes, books, coefs, trial, None, out, None, status])
    return out, status


def adamw_encode(codes, books, coefs, new_books, count: int, group: int, *, batch: int = 1, out=None, changed=None,
                 status=None):
    """Decode, update and re-encode W, M, V of each expert: codes (E, 3, words), changed (E,)."""
    words = words_for(count, group)
    dev = codes.device
    out = torch.empty((batch, 3, words), dtype=torch.int32, device=dev) if out is None else out
    changed = torch.empty(batch, dtype=torch.int32, device=dev) if changed is None else changed
    status = status_word(dev) if status is None else status
    launch(plan2(OP_ADAMW_ENCODE, count, 1, 1, group, batch=batch),
           [codes, books, coefs, new_books, None, out, changed, status])
    return out, changed, status


def fit_workspace_bytes(samples: int) -> int:
    """Workspace bytes of `adamw_fit` per fitted book."""
    return (samples + 15) // 16 * 16 + 160


def adamw_fit(codes, books, coefs, samples, count: int, group: int, *, iterations: int = 4, batch: int = 1, out=None,
              workspace=None, status=None):
    """fit_codebook of W', M', V' for each expert on the device, warm-started
    from the current books: `samples` is `adamw_sample`'s output (E, 3, S,
    group); returns the fitted books (E, 3, 16, group), bit for bit the CPU
    fit of the same sample."""
    s = samples.shape[2]
    dev = codes.device
    out = torch.empty((batch, 3, ENTRIES, group), dtype=torch.float32, device=dev) if out is None else out
    if workspace is None:
        workspace = torch.empty(batch * 3 * fit_workspace_bytes(s), dtype=torch.uint8, device=dev)
    status = status_word(dev) if status is None else status
    launch(plan2(OP_FIT, count, 1, 1, group, flags=1, batch=batch, aux0=s, aux1=iterations),
           [codes, books, coefs, samples, workspace, out, None, status])
    return out, status


def fit_codebook(x, group: int, *, iterations: int = 4, sample_vectors: int = 4096, init=None, out=None, status=None):
    """`fit_codebook` of a float32 CUDA tensor on its device, bit for bit the
    CPU function's book (16, group); `init` (16, group) warm-starts it."""
    import numpy as np
    count = x.numel()
    complete = count // group
    if complete < 1:
        raise ack.AckError("codebook calibration needs at least one complete vector")
    s = min(complete, sample_vectors)
    positions = np.linspace(0, complete - 1, s, dtype=np.int64)
    rows = np.linspace(0, s - 1, ENTRIES, dtype=np.int64)
    index = torch.from_numpy(np.concatenate([positions, rows]).astype(np.uint32).view(np.int32)).to(x.device)
    out = torch.empty((ENTRIES, group), dtype=torch.float32, device=x.device) if out is None else out
    workspace = torch.empty(s * group * 4 + fit_workspace_bytes(s), dtype=torch.uint8, device=x.device)
    status = status_word(x.device) if status is None else status
    launch(plan2(OP_FIT_VALUES, count & 0xFFFFFFFF, 1, 1, group, flags=0 if init is None else 1, aux0=s,
                 aux1=iterations, aux2=count >> 32),
           [x, init, index, None, workspace, out, None, status])
    return out, status


def _f32_bits(value: float) -> int:
    return struct.unpack("<I", struct.pack("<f", value))[0]


def residual(prediction, target_codes, target_book, group: int, scale: float, *, out=None, sumsq=None,
             workspace=None, status=None):
    """The harness residual on the device: r = prediction - decode(target)
    (FP32, elementwise), returned scaled by fl32(scale), and the float64 sum
    of r^2 in `sumsq` (one value): the MSE loss is sumsq / count."""
    count = prediction.numel()
    dev = prediction.device
    out = torch.empty_like(prediction) if out is None else out
    sumsq = torch.empty(1, dtype=torch.float64, device=dev) if sumsq is None else sumsq
    workspace = torch.empty(REDUCE_WORKSPACE_BYTES // 8, dtype=torch.float64, device=dev) if workspace is None \
        else workspace
    status = status_word(dev) if status is None else status
    launch(plan2(OP_RESIDUAL, count, 1, 1, group, aux0=_f32_bits(scale)),
           [prediction, target_codes, target_book, None, workspace, out, sumsq, status])
    return out, sumsq, status


def clip_norm(gradient, max_norm: float, *, out=None, stats=None, workspace=None, status=None):
    """The harness's global-norm clip on the device: norm = ||g||_2 in
    float64, scale = min(1, max_norm / (norm + 1e-6)), out = g * fl32(scale);
    `stats` (two float64) receives [norm, scale]."""
    count = gradient.numel()
    dev = gradient.device
    out = torch.empty_like(gradient) if out is None else out
    stats = torch.empty(2, dtype=torch.float64, device=dev) if stats is None else stats
    workspace = torch.empty(REDUCE_WORKSPACE_BYTES // 8, dtype=torch.float64, device=dev) if workspace is None \
        else workspace
    status = status_word(dev) if status is None else status
    lo, hi = struct.unpack("<II", struct.pack("<d", float(max_norm)))
    launch(plan2(OP_CLIP, count, 1, 1, 8, aux0=lo, aux1=hi), [gradient, None, None, None, workspace, out, stats, status])
    return out, stats, status
