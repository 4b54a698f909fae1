"""The reference's NF4 shaders compiled for the host (oracle/Makefile `ref`,
nf4_shim.h): nf4_decode.comp for output storage 0/1/2 and nf4_gemv.comp for
bf16 (0) and fp16 (1) operands. TEST INFRASTRUCTURE ONLY: a checker of
nf4_oracle.py; nothing in the product loads it.

The call builds the push words and grid the reference's planner records
(nf4_ops.rs) from the same arrays nf4_oracle takes, and runs every
invocation of the dispatch on the host."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

import nf4_oracle as no

HERE = Path(__file__).resolve().parent


def _lib(name: str):
    path = HERE / "_ref" / name
    return ctypes.CDLL(str(path)) if path.exists() else None


def available() -> bool:
    return all((HERE / "_ref" / f).exists() for f in
               ("libnf4_decode_ref0.so", "libnf4_decode_ref1.so", "libnf4_decode_ref2.so",
                "libnf4_gemv_ref0.so", "libnf4_gemv_ref1.so"))


def _words(data: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(data).view(np.uint8).tobytes()
    return np.frombuffer(raw + b"\0" * (-len(raw) % 4), np.uint32).copy()


def _arg(arr: np.ndarray):
    return arr.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(arr.size)


def decode(packed, absmax_q, absmax2, tables, starts, offsets, n, *, ids=None, member_values=0, src_base=0,
           storage=0) -> np.ndarray:
    lib = _lib(f"libnf4_decode_ref{storage}.so")
    pw, qw = _words(np.asarray(packed, np.uint8)), _words(np.asarray(absmax_q, np.uint8))
    a2 = np.ascontiguousarray(absmax2, np.float32)
    tb = np.ascontiguousarray(tables, np.float32)
    sw = _words(np.ascontiguousarray(starts, np.int64))
    ov = np.ascontiguousarray(offsets, np.float32)
    iw = _words(np.ascontiguousarray(ids, np.int64)) if ids is not None else np.zeros(2, np.uint32)
    plan = no.decode_plan(n, len(ov), 0 if ids is None else len(ids), member_values, src_base,
                          no.values_covered(len(packed), len(absmax_q), 4 * len(a2)), storage)
    push = np.array([plan[k] for k in ("n", "words", "members", "selected", "member_values", "src_base",
                                       "src_limit")], np.uint32)
    out = np.zeros(n, np.float32 if storage == 0 else np.uint16)
    groups = (plan["words"] + 255) // 256
    gx = min(groups, no.MAX_GRID)
    gy = (groups + gx - 1) // gx
    args = [push.ctypes.data_as(ctypes.c_void_p)]
    for arr in (pw, qw, a2, tb, sw, ov, iw, out):
        args += list(_arg(arr))
    lib.nf4_decode_ref_run.restype = ctypes.c_int
    bad = lib.nf4_decode_ref_run(*args, ctypes.c_uint32(gx), ctypes.c_uint32(gy))
    assert bad == 0, "the shader indexed past a binding"
    return out


def gemv(a16, packed, absmax_q, absmax2, tables, starts, offsets, groups, *, rows, n, k, lda=0, src_base=0,
         elem=0, c=None) -> np.ndarray:
    lib = _lib(f"libnf4_gemv_ref{elem}.so")
    gt = np.ascontiguousarray(groups, np.uint32).reshape(-1, 3)
    max_rows = int(gt[:, 1].max())
    a2 = np.ascontiguousarray(absmax2, np.float32)
    plan = no.gemv_plan(rows, max_rows, n, k, lda, len(gt), len(offsets), src_base,
                        no.values_covered(len(packed), len(absmax_q), 4 * len(a2)), elem)
    push = np.array([plan[x] for x in ("n", "k", "lda", "rows", "src_base", "src_limit", "members")], np.uint32)
    a_words = _words(np.ascontiguousarray(a16, np.uint16).reshape(-1))
    a_words = np.concatenate([a_words, np.zeros(-len(a_words) % 4, np.uint32)])
    out = np.zeros(rows * n, np.float32) if c is None else np.array(c, np.float32).reshape(-1)
    arrays = (a_words, _words(np.asarray(packed, np.uint8)), out, _words(np.asarray(absmax_q, np.uint8)), a2,
              np.ascontiguousarray(tables, np.float32), _words(np.ascontiguousarray(starts, np.int64)),
              np.ascontiguousarray(offsets, np.float32), gt.reshape(-1).copy())
    args = [push.ctypes.data_as(ctypes.c_void_p)]
    for i, arr in enumerate(arrays):
        ptr, count = _arg(arr)
        args += [ptr, ctypes.c_uint64(count.value // 4) if i == 0 else count]   # A in uvec4 units
    gx = min(n, no.MAX_GRID)
    gy = (n + no.MAX_GRID - 1) // no.MAX_GRID
    lib.nf4_gemv_ref_run.restype = ctypes.c_int
    bad = lib.nf4_gemv_ref_run(*args, ctypes.c_uint32(gx), ctypes.c_uint32(gy), ctypes.c_uint32(len(gt)))
    assert bad == 0, "the shader indexed past a binding"
    return out.reshape(rows, n)
