"""The reference's own vq4 compute shader, compiled for the host CPU --
TEST INFRASTRUCTURE ONLY, like everything under `oracle/`.

`oracle/Makefile` (target `ref`) compiles the unchanged GLSL source of
`src/alelyon_compute_kit/_kit/kernels/vq4.comp` as C++ through the shim in
`oracle/vq4_shim.h`, into `oracle/_ref/libvq4_ref.so`. This module runs one
dispatch of it over numpy arrays. The tests use it to pin the numpy
restatements of the shader (`vq_oracle.matmul_shader`, `adamw_shader`,
`nearest_fp32_shader`): op 2, op 3 and op 0 (`vq4.comp:87-176`).

The shader is executed one invocation at a time, with IEEE FP32 arithmetic,
every operation rounded on its own (the `precise` qualifier, no fused
multiply-add), in the shader's own source order.

The library is built only where the reference checkout exists. The built
file travels with the repository; where it is missing, `available()` is
False and callers skip.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_ref" / "libvq4_ref.so"
_LIB = None


def build(reference: str | None = None) -> bool:
    """Build the shader library from a reference checkout; True if it exists after."""
    reference = reference or os.environ.get("ACK_REFERENCE_ROOT")
    if reference and Path(reference).is_dir():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REFERENCE={reference}"], check=True)
    return LIBRARY.exists()


def available() -> bool:
    return LIBRARY.exists()


def lib():
    global _LIB
    if _LIB is None:
        c = ctypes.CDLL(str(LIBRARY))
        p, u = ctypes.c_void_p, ctypes.c_uint32
        c.vq4_ref_run.argtypes = [p, p, u, p, u, p, u, p, u, p, u, p, u, u]
        c.vq4_ref_run.restype = ctypes.c_int
        _LIB = c
    return _LIB


def _words(a) -> np.ndarray:
    if a is None:
        return np.zeros(1, np.uint32)
    a = np.ascontiguousarray(a)
    if a.dtype == np.float32:
        a = a.view(np.uint32)
    return np.ascontiguousarray(a.astype(np.uint32, copy=False).reshape(-1))


def run(plan, b0, b1, b2=None, b3=None, out_words: int = 1):
    """One shader dispatch. `plan` is the 8-word push block
    `[op, m, n, k, group, entries, flags, reserved]`. Returns (dst as u32
    words, status word). The workgroup count is ceil(invocations / 64), the
    one the reference's planner records (`vq4_ops.rs:173-175`)."""
    plan = np.asarray(plan, np.uint32)
    op, m, n = int(plan[0]), int(plan[1]), int(plan[2])
    invocations = {0: (m + 8 * int(plan[4]) - 1) // (8 * int(plan[4])), 1: m, 2: m * n, 3: m}.get(op, m)
    groups = max(1, (invocations + 63) // 64)
    bufs = [_words(b) for b in (b0, b1, b2, b3)]
    dst = np.zeros(max(1, out_words), np.uint32)
    status = np.zeros(1, np.uint32)
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    bad = lib().vq4_ref_run(ptr(plan), ptr(bufs[0]), bufs[0].size, ptr(bufs[1]), bufs[1].size,
                            ptr(bufs[2]), bufs[2].size, ptr(bufs[3]), bufs[3].size,
                            ptr(dst), dst.size, ptr(status), status.size, groups)
    if bad:
        raise IndexError("the shader indexed past a binding")
    return dst, int(status[0])


def matmul(a_codes, a_book, b_codes, b_book, m, n, k, group, flags):
    """Op 2 (`vq4.comp:165-176`): C[m, n] as float32, and the status word."""
    dst, status = run([2, m, n, k, group, 16, flags, 0], a_codes, a_book, b_codes, b_book, m * n)
    return dst.view(np.float32).reshape(m, n), status


def adamw(state_codes, books, coefficients, n, group):
    """Op 3 (`vq4.comp:87-116`): the four code images [W, M, V, G] back to
    back, their four books, the seven coefficients. Returns (w', m', v'),
    status."""
    codes = np.concatenate([np.asarray(c, np.uint32).reshape(-1) for c in state_codes])
    book = np.concatenate([np.asarray(b, np.float32).reshape(-1) for b in books])
    coefs = np.asarray(coefficients, np.float32)
    dst, status = run([3, n, 1, 1, group, 16, 0, 0], codes, book, coefs, None, 3 * n)
    out = dst.view(np.float32)
    return (out[:n], out[n:2 * n], out[2 * n:]), status


def encode(values, book, group):
    """Op 0 (`vq4.comp:118-144`), the shader's FP32 encoder: packed code
    words and the status word."""
    x = np.ascontiguousarray(values, np.float32).reshape(-1)
    words = ((x.size + group - 1) // group + 7) // 8
    dst, status = run([0, x.size, 1, 1, group, 16, 0, 0], x, np.asarray(book, np.float32), None, None, words)
    return dst, status


def decode(codes, book, n, group):
    """Op 1 (`vq4.comp:161-162`): n float32 values and the status word."""
    dst, status = run([1, n, 1, 1, group, 16, 0, 0], codes, np.asarray(book, np.float32), None, None, n)
    return dst.view(np.float32), status
