"""ctypes loader for the C oracle (`oracle/libvq_oracle.so`) -- TEST
INFRASTRUCTURE ONLY, like everything under `oracle/`."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return HERE / "libvq_oracle.so"


def lib():
    global _LIB
    if _LIB is None:
        path = HERE / "libvq_oracle.so"
        if not path.exists():
            build()
        c = ctypes.CDLL(str(path))
        p = ctypes.c_void_p
        c.vqo_threads.restype = ctypes.c_int
        c.vqo_decode.argtypes = [p, p, ctypes.c_uint64, ctypes.c_uint32, p]
        c.vqo_encode.argtypes = [p, ctypes.c_uint64, p, ctypes.c_uint32, p]
        c.vqo_dense_nt.argtypes = [p, ctypes.c_uint32, ctypes.c_uint32, p, p, ctypes.c_uint32,
                                   ctypes.c_uint32, p]
        c.vqo_adamw.argtypes = [p, p, p, p, ctypes.c_uint64, p, p, p, p]
        _LIB = c
    return _LIB


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def threads() -> int:
    return int(lib().vqo_threads())


def decode(codes, book, n, group, out=None):
    codes = np.ascontiguousarray(codes, np.uint32)
    book = np.ascontiguousarray(book, np.float32)
    out = np.empty(n, np.float32) if out is None else out
    lib().vqo_decode(_ptr(codes), _ptr(book), n, group, _ptr(out))
    return out


def encode(values, book, group):
    values = np.ascontiguousarray(values, np.float32).reshape(-1)
    book = np.ascontiguousarray(book, np.float32)
    words = ((values.size + group - 1) // group + 7) // 8
    out = np.empty(words, np.uint32)
    lib().vqo_encode(_ptr(values), values.size, _ptr(book), group, _ptr(out))
    return out


def dense_nt(x, codes, book, n, group):
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    codes = np.ascontiguousarray(codes, np.uint32)
    book = np.ascontiguousarray(book, np.float32)
    y = np.empty((m, n), np.float32)
    lib().vqo_dense_nt(_ptr(x), m, k, _ptr(codes), _ptr(book), n, group, _ptr(y))
    return y


def adamw(w, m, v, g, coefficients):
    arrs = [np.ascontiguousarray(t, np.float32).reshape(-1) for t in (w, m, v, g)]
    c = np.ascontiguousarray(coefficients, np.float32)
    outs = [np.empty_like(arrs[0]) for _ in range(3)]
    lib().vqo_adamw(*(_ptr(a) for a in arrs), arrs[0].size, _ptr(c), *(_ptr(o) for o in outs))
    return tuple(outs)
