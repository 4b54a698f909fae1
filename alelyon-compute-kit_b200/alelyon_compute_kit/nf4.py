"""The NF4 comparator on device-resident PyTorch tensors: nf4-decode/v1 and
nf4-gemv/v1 of the reference kit (its `ack_nf4_decode` / `ack_gemv_nf4`,
ffi.rs:7365 and :8017; the law in kernels/nf4_decode.comp and
nf4_gemv.comp), through the library's device-pointer entries
`ack_nf4_decode_launch` / `ack_gemv_nf4_launch`: the same admission and
refusal names as the handle entries, work on the current PyTorch stream.

The stored form (bitsandbytes' NF4 with double quantisation): `packed`
uint8, two 4-bit indices a byte with the first value in the high nibble;
`absmax_q` uint8, one index a block of 64 values into the 256-entry map;
`absmax2` float32, one value a nested block of 256 blocks; `tables`
float32[272], the 16 code values then the 256 map values; `starts` int64,
each member's first value (ascending from 0, on whole nested blocks);
`offsets` float32, one a member.

A comparator for the vq4 path, not part of it: the same 4-bit weight budget
in another format, measured on the same shapes.
"""
from __future__ import annotations

import ctypes

import torch

from . import ack

STORAGE = {"f32": 0, "bf16": 1, "f16": 2}
ELEM = {"bf16": 0, "f16": 1}


def _operands(tensors):
    ptrs = (ctypes.c_void_p * len(tensors))()
    sizes = (ctypes.c_uint64 * len(tensors))()
    device = None
    for i, t in enumerate(tensors):
        if t is None:
            continue
        if not t.is_cuda or not t.is_contiguous():
            raise ack.AckError(f"nf4 operand {i} must be a contiguous CUDA tensor")
        device = device or t.device
        if t.device != device:
            raise ack.AckError("nf4 operands live on different devices")
        ptrs[i] = t.data_ptr()
        sizes[i] = t.numel() * t.element_size()
    return ptrs, sizes, device


def decode(packed, absmax_q, absmax2, tables, starts, offsets, n: int, *, ids=None, member_values: int = 0,
           src_base: int = 0, storage: str = "f32", out=None) -> torch.Tensor:
    """nf4-decode/v1 of `n` values: the whole source member by member, or
    (with `ids`, int64) the selected members of `member_values` each; float32
    output, or the 16-bit words of bf16 / fp16 as int16."""
    code = STORAGE[storage]
    if out is None:
        out = torch.empty(n, dtype=torch.float32 if code == 0 else torch.int16, device=packed.device)
    selected = 0 if ids is None else ids.numel()
    ptrs, sizes, device = _operands([packed, absmax_q, absmax2, tables, starts, offsets, ids, out])
    lib = ack._lib()
    with torch.cuda.device(device):
        rc = lib.cdll.ack_nf4_decode_launch(ptrs, sizes, n, offsets.numel(), selected, member_values, src_base, code,
                                            ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    if rc != ack.ACK_OK:
        raise ack._kit_error("nf4-decode", rc, lib.last_error())
    return out


def gemv(a16, packed, absmax_q, absmax2, tables, starts, offsets, groups, *, rows: int, n: int, k: int,
         lda: int = 0, src_base: int = 0, elem: str = "bf16", max_rows: int | None = None,
         out=None) -> torch.Tensor:
    """nf4-gemv/v1: for each group (first row, rows, weight base) of `groups`
    (int32, G x 3), C[first row + m, :] = A[first row + m, :] . W^T with W
    the n x k weight at the base; `a16` holds A's 16-bit words (rows x lda);
    C is float32 rows x n (rows no group writes are left as they are)."""
    table = groups.reshape(-1, 3)
    if max_rows is None:
        max_rows = int(table[:, 1].max().item())
    if out is None:
        out = torch.zeros((rows, n), dtype=torch.float32, device=a16.device)
    ptrs, sizes, device = _operands([a16, packed, absmax_q, absmax2, tables, starts, offsets, table, out])
    lib = ack._lib()
    with torch.cuda.device(device):
        rc = lib.cdll.ack_gemv_nf4_launch(ptrs, sizes, rows, max_rows, n, k, lda, table.shape[0], offsets.numel(),
                                          src_base, ELEM[elem],
                                          ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    if rc != ack.ACK_OK:
        raise ack._kit_error("nf4-gemv", rc, lib.last_error())
    return out
