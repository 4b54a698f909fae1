"""ctypes helpers for the host-only ABI tests: plan blocks and the planner
probes of libalelyon_compute_kit.so. Nothing here touches a device."""
import ctypes
import struct

from alelyon_compute_kit import ack

MAX_VALUES = 1 << 28
MAX_DIM = 65536


def lib():
    return ack._lib()


def block(words) -> bytes:
    return struct.pack(f"<{len(words)}I", *words)


def last_error() -> str:
    return lib().last_error()


def probe(words):
    """(code, required_bytes[8], work_items, dispatch[3]) of a plan."""
    plan = block(words)
    req = (ctypes.c_uint64 * 8)()
    work = ctypes.c_uint32()
    disp = (ctypes.c_uint32 * 3)()
    rc = lib().cdll.ack_vq_plan_probe(plan, len(plan), req, ctypes.byref(work), disp)
    return rc, list(req), work.value, list(disp)


def required(words):
    rc, req, _, _ = probe(words)
    assert rc == 0, last_error()
    return req[:6] if len(words) == 8 else req


def validate_buffers(words, capacities, ids):
    plan = block(words)
    caps = (ctypes.c_uint64 * len(capacities))(*capacities)
    idv = (ctypes.c_uint64 * len(ids))(*ids)
    return lib().cdll.ack_vq_plan_validate_buffers(plan, len(plan), caps, idv, len(ids))


def validate_dispatch(words, limits):
    plan = block(words)
    lim = (ctypes.c_uint32 * 3)(*limits)
    return lib().cdll.ack_vq_plan_validate_dispatch(plan, len(plan), lim)


def refusal(words):
    """(code, message) of a plan the probe refuses."""
    rc, _, _, _ = probe(words)
    return rc, last_error()
